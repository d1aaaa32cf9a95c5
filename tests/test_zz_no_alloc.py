"""The BQ candidate scan that allocates no device memory (vx_bq_scan_candidates_noalloc).

It exists for callers that must not allocate device memory while searching (a host that
reserves and accounts its whole device budget up front, or a latency-critical loop where an
allocation would block on the allocator or synchronise the device).  Its scratch is a
statically sized device array shared by every call, placed on the device when a BQ index is
built there.  This file checks that:
  * two calls in a row return, bit for bit (the BQ path's tolerance), what the allocating
    entry point returns;
  * a call, the first one after the build included, changes neither the device's free memory
    nor the stream-ordered pool's reserved or peak-used bytes;
  * an oversized batch is refused with a message giving the largest batch that fits;
  * host-side fault injection reaches the call like every other entry point.

This file is collected last on purpose: a failure here leaves every other test already run.
"""
import ctypes as C

import numpy as np
import pytest

import vectors_b200 as vx
from vectors_b200 import _native as N

pytestmark = pytest.mark.gpu

# CUmemPool_attribute values (cuda.h)
_RESERVED_MEM_CURRENT = 5
_USED_MEM_CURRENT = 7
_USED_MEM_HIGH = 8


class _Pool:
    """The device's default stream-ordered pool (the one cudaMallocAsync draws on), read through
    the driver API."""

    def __init__(self, device):
        self.cu = C.CDLL("libcuda.so.1")
        dev = C.c_int()
        assert self.cu.cuDeviceGet(C.byref(dev), device) == 0
        self.pool = C.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(C.byref(self.pool), dev) == 0

    def get(self, attr):
        v = C.c_uint64()
        assert self.cu.cuMemPoolGetAttribute(self.pool, attr, C.byref(v)) == 0
        return v.value

    def reset_peak(self):
        zero = C.c_uint64(0)
        assert self.cu.cuMemPoolSetAttribute(self.pool, _USED_MEM_HIGH, C.byref(zero)) == 0


def _bq_index(rng, n, dim, metric):
    db = rng.standard_normal((n, dim)).astype(np.float32)
    words = np.zeros((n, dim // 64), np.uint64)
    bits = (db >= 0).astype(np.uint64)
    for w in range(dim // 64):
        for b in range(64):
            words[:, w] |= bits[:, 64 * w + b] << np.uint64(b)
    index = vx.QuantizedFlatScanAdapter()
    index.build_bq(words, dim, metric)
    return index


def _outputs(nq, k):
    import torch

    return (torch.empty((nq, k), dtype=torch.int32, device="cuda"),
            torch.empty((nq, k), dtype=torch.float32, device="cuda"),
            torch.empty((nq,), dtype=torch.int32, device="cuda"))


def _call(index, q, k, outs):
    import torch

    ids, sc, cnt = outs
    st = torch.cuda.current_stream(q.device).cuda_stream
    return N.lib().vx_bq_scan_candidates_noalloc(index._h.ptr, C.c_void_p(q.data_ptr()), q.shape[0], q.shape[1],
                                                 k, C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                 C.c_void_p(cnt.data_ptr()), C.c_void_p(st))


def test_no_alloc_scan_matches_allocating_scan_twice():
    import torch

    rng = np.random.default_rng(7)
    n, dim, k, nq = 30000, 1024, 100, 200
    for metric in (vx.SimilarityFunction.COSINE, vx.SimilarityFunction.EUCLIDEAN):
        index = _bq_index(rng, n, dim, metric)
        outs = _outputs(nq, k)
        for call in range(2):
            q = torch.from_numpy(rng.standard_normal((nq, dim)).astype(np.float32)).cuda()
            N.check(_call(index, q, k, outs))
            torch.cuda.synchronize()
            ids, sc, cnt = (t.cpu().numpy() for t in outs)
            ref_ids, ref_sc, ref_cnt = index.scan_candidates_device(q, k)
            torch.cuda.synchronize()
            assert np.array_equal(cnt, ref_cnt.cpu().numpy()), (metric, call)
            assert np.array_equal(ids, ref_ids.cpu().numpy()), (metric, call)
            assert np.array_equal(sc, ref_sc.cpu().numpy()), (metric, call)
        index.close()


def test_no_alloc_scan_allocates_nothing():
    import torch

    rng = np.random.default_rng(9)
    n, dim, k, nq = 50000, 1024, 100, 128
    index = _bq_index(rng, n, dim, vx.SimilarityFunction.DOT_PRODUCT)
    outs = _outputs(nq, k)
    q = torch.from_numpy(rng.standard_normal((nq, dim)).astype(np.float32)).cuda()
    pool = _Pool(torch.cuda.current_device())
    torch.cuda.synchronize()
    for call in range(2):  # the first call after the build, then a second one
        free0 = torch.cuda.mem_get_info()[0]
        reserved0 = pool.get(_RESERVED_MEM_CURRENT)
        used0 = pool.get(_USED_MEM_CURRENT)
        pool.reset_peak()
        N.check(_call(index, q, k, outs))
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0, call
        assert pool.get(_RESERVED_MEM_CURRENT) == reserved0, call
        assert pool.get(_USED_MEM_HIGH) == used0, call
    index.close()


def test_no_alloc_scan_rejects_oversized_batch():
    import torch

    rng = np.random.default_rng(8)
    words = rng.integers(0, 2**63, size=(5000, 16), dtype=np.uint64)
    index = vx.QuantizedFlatScanAdapter()
    index.build_bq(words, 1024, vx.SimilarityFunction.COSINE)
    q = torch.zeros((20000, 1024), dtype=torch.float32, device="cuda")
    with pytest.raises(vx.VxError, match=r"at most \d+ queries fit"):
        N.check(_call(index, q, 500, _outputs(20000, 500)))
    index.close()


def test_no_alloc_scan_sees_injected_failure():
    import torch

    rng = np.random.default_rng(10)
    words = rng.integers(0, 2**63, size=(1000, 16), dtype=np.uint64)
    index = vx.QuantizedFlatScanAdapter()
    index.build_bq(words, 1024, vx.SimilarityFunction.COSINE)
    q = torch.zeros((4, 1024), dtype=torch.float32, device="cuda")
    N.lib().vx_debug_fail_next(4)  # VX_ERR_CUDA
    assert _call(index, q, 10, _outputs(4, 10)) == 4
    assert _call(index, q, 10, _outputs(4, 10)) == 0  # the injected failure fires once
    index.close()
