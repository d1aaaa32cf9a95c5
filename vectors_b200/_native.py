"""ctypes binding of libvx.so (include/vx.h).

The library is built in-tree (``vectors_b200/libvx.so``).  Loading fails loudly when it is
missing: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvx.so")

VX_OK = 0
VX_ERR_INVALID_ARGUMENT = 1
VX_ERR_NULL_POINTER = 2
VX_ERR_GPU_UNAVAILABLE = 3
VX_ERR_CUDA = 4
VX_ERR_OUT_OF_MEMORY = 5
VX_ERR_UNSUPPORTED = 6
VX_ERR_DEVICE_TIMEOUT = 7
VX_ERR_FORMAT = 8

VX_KIND_FLAT, VX_KIND_FP16, VX_KIND_SQ8, VX_KIND_BQ, VX_KIND_IVFPQ, VX_KIND_IVFFLAT, VX_KIND_SQ4, VX_KIND_BBQ, VX_KIND_PQ = range(9)

_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64
_F32 = C.c_float
_PP = C.POINTER(C.c_void_p)

# name -> (argtypes); every function returns int (vx_status) except vx_last_error.
SIGNATURES = {
    "vx_abi_version": [],
    "vx_device_count": [_P],
    "vx_kernel_launches": [_P],
    "vx_debug_fail_next": [_I32],
    "vx_debug_wait_timeout": [_I32, _I32],
    "vx_profile_enable": [_I32],
    "vx_profile_read": [_I32, _P, _P],
    "vx_profile_reset": [],
    "vx_flat_build": [_I32, _P, _I64, _I32, _I64, _I32, _PP],
    "vx_fp16_build": [_I32, _P, _I64, _I32, _I32, _P, _I64, _PP],
    "vx_sq8_build": [_I32, _P, _P, _I64, _I32, _F32, _F32, _I32, _P, _I64, _PP],
    "vx_sq4_build": [_I32, _P, _P, _I64, _I32, _F32, _F32, _I32, _P, _I64, _PP],
    "vx_bq_build": [_I32, _P, _I64, _I32, _I32, _P, _I64, _PP],
    "vx_bbq_build": [_I32, _P, _P, _P, _I64, _I32, _I32, _P, _I64, _PP],
    "vx_pq_build": [_I32, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _P, _I64, _PP],
    "vx_ivfpq_build": [_I32, _P, _I32, _I32, _P, _P, _I32, _I32, _P, _P, _I64, _I32, _P, _I32, _I32, _PP],
    "vx_quantized_bin_info": [_P, _I64, _P, _P, _P],
    "vx_quantized_bin_build": [_I32, _P, _I64, _I32, _P, _I64, _PP],
    "vx_ivf_graph_info": [_P, _I64, _P, _P, _P, _P, _P],
    "vx_ivf_graph_build": [_I32, _P, _I64, _I32, _P, _I64, _I64, _I32, _I32, _PP],
    "vx_ivfflat_build": [_I32, _P, _I32, _I32, _P, _P, _P, _I64, _I64, _I32, _I32, _PP],
    "vx_ivf_set_buoy": [_P, _P, _P],
    "vx_ivf_set_gamma": [_P, _F32],
    "vx_ivf_set_key_dims": [_P, _P],
    "vx_index_info": [_P, _P, _P, _P, _P],
    "vx_index_free": [_P],
    "vx_search_batch": [_P, _P, _I32, _I32, _I32, _I32, _F32, _P, _P, _P],
    "vx_search_batch_device": [_P, _P, _I32, _I32, _I32, _I32, _F32, _P, _P, _P, _P],
    "vx_scan_candidates": [_P, _P, _I32, _I32, _I32, _P, _P, _P],
    "vx_scan_candidates_device": [_P, _P, _I32, _I32, _I32, _P, _P, _P, _P],
    "vx_ivfpq_search": [_P, _P, _I32, _I32, _I32, _I32, _I32, _F32, _P, _P, _P],
    "vx_ivfpq_search_device": [_P, _P, _I32, _I32, _I32, _I32, _I32, _F32, _P, _P, _P, _P],
    "vx_ivf_route_device": [_P, _P, _I32, _I32, _I32, _P, _P],
    "vx_ivfpq_search_routed_device": [_P, _P, _I32, _I32, _I32, _I32, _I32, _F32, _P, _P, _P, _P, _P],
    "vx_ivf_route_dist_device": [_P, _P, _I32, _I32, _I32, _P, _P, _P],
    "vx_ivfflat_scan_pairs_device": [_P, _P, _I32, _I32, _I32, _I32, _P, _P, _P, _P],
    "vx_ivfflat_merge_pairs_device": [_P, _I32, _I32, _I32, _P, _P, _P, _P, _F32, _P, _P, _P, _P],
    "vx_merge_shards_device": [_I32, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _P, _P, _P, _P],
    "vx_bq_scan_candidates_noalloc": [_P, _P, _I32, _I32, _I32, _P, _P, _P, _P],
}

_lib = None
_lock = threading.Lock()


class VxError(RuntimeError):
    """A vx_* call failed; ``status`` is the vx_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[vx status {status}] {message}")
        self.status = status


def lib() -> C.CDLL:
    """Loads libvx.so once (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libvx.so not found at {LIB_PATH}; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` or `make -C vectors_b200/csrc`"
                )
            h = C.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(h, name)
                fn.argtypes = args
                fn.restype = C.c_int
            h.vx_last_error.argtypes = []
            h.vx_last_error.restype = C.c_char_p
            _lib = h
    return _lib


def last_error() -> str:
    return (lib().vx_last_error() or b"").decode("utf-8", "replace")


def check(status: int) -> None:
    if status != VX_OK:
        raise VxError(status, last_error())


def exported_symbols() -> list[str]:
    return sorted(list(SIGNATURES) + ["vx_last_error"])


def device_count() -> int:
    c = C.c_int32(0)
    check(lib().vx_device_count(C.byref(c)))
    return int(c.value)


PROFILE_SLOTS = {
    "gemm_scan": 0,
    "merge": 1,
    "rescore": 2,
    "fallback": 3,
    "bq_scan": 4,
    "adc_scan": 5,
    "route": 6,
    "pilot": 7,
}


def profile_enable(on: bool = True) -> None:
    check(lib().vx_profile_enable(1 if on else 0))


def profile_reset() -> None:
    check(lib().vx_profile_reset())


def profile_read() -> dict:
    """{slot name: (total device ms, launches)} accumulated since the last reset."""
    out = {}
    for name, slot in PROFILE_SLOTS.items():
        ms, n = C.c_double(0), C.c_int64(0)
        check(lib().vx_profile_read(slot, C.byref(ms), C.byref(n)))
        out[name] = (ms.value, n.value)
    return out


def kernel_launches() -> int:
    c = C.c_int64(0)
    check(lib().vx_kernel_launches(C.byref(c)))
    return int(c.value)
