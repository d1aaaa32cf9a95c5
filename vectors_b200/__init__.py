"""vectors_b200: the integrallis/vectors batch distance + top-k scan on NVIDIA B200 (sm_100a).

The scans (FLAT exact search, the SQ8 / FP16 / sign-bit BQ quantized scans and the IVF-PQ ADC
list scan) run as hand-written CUDA kernels in ``libvx.so``; this package is the host-side
mirror of the reference's index SPI over that library's C ABI (include/vx.h).
"""
from ._native import VxError, device_count, kernel_launches, lib  # noqa: F401
from .index_spi import (  # noqa: F401
    FlatScanAdapter,
    GpuUnavailableException,
    IOException,
    IllegalArgumentException,
    IndexSpi,
    IvfFlatAdapter,
    IvfPqAdapter,
    NullPointerException,
    QuantizedFlatScanAdapter,
    SearchOutcome,
    SimilarityFunction,
    UnsupportedOperationException,
    ivf_graph_info,
    merge_shards_device,
    quantized_bin_info,
    shard_offsets,
)

__all__ = [
    "FlatScanAdapter",
    "QuantizedFlatScanAdapter",
    "IvfPqAdapter",
    "IvfFlatAdapter",
    "IndexSpi",
    "SearchOutcome",
    "SimilarityFunction",
    "IllegalArgumentException",
    "NullPointerException",
    "GpuUnavailableException",
    "UnsupportedOperationException",
    "IOException",
    "quantized_bin_info",
    "ivf_graph_info",
    "merge_shards_device",
    "shard_offsets",
    "device_count",
    "kernel_launches",
    "lib",
    "VxError",
]
