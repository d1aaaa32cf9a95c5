"""The BQ candidate scan that allocates no device memory (vx_bq_scan_candidates_noalloc).

It exists for callers that must not allocate device memory while searching (a host that
reserves and accounts its whole device budget up front, or a latency-critical loop where an
allocation would block on the allocator or synchronise the device).  Its scratch is a
statically sized device array shared by every call, so this test runs two calls in a row and
checks both against the allocating entry point, bit for bit (the BQ path's tolerance), and
that an oversized batch is refused with a clear message.

This file is collected last on purpose: a failure here leaves every other test already run.
"""
import ctypes as C

import numpy as np
import pytest

import vectors_b200 as vx
from vectors_b200 import _native as N

pytestmark = pytest.mark.gpu


def _noalloc(index, q, k):
    import torch

    nq, dim = q.shape
    ids = torch.empty((nq, k), dtype=torch.int32, device=q.device)
    sc = torch.empty((nq, k), dtype=torch.float32, device=q.device)
    cnt = torch.empty((nq,), dtype=torch.int32, device=q.device)
    st = torch.cuda.current_stream(q.device).cuda_stream
    N.check(N.lib().vx_bq_scan_candidates_noalloc(index._h.ptr, C.c_void_p(q.data_ptr()), nq, dim, k,
                                                  C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                  C.c_void_p(cnt.data_ptr()), C.c_void_p(st)))
    torch.cuda.synchronize()
    return ids.cpu().numpy(), sc.cpu().numpy(), cnt.cpu().numpy()


def test_no_alloc_scan_matches_allocating_scan_twice():
    import torch

    rng = np.random.default_rng(7)
    n, dim, k = 30000, 1024, 100
    db = rng.standard_normal((n, dim)).astype(np.float32)
    words = np.zeros((n, dim // 64), np.uint64)
    bits = (db >= 0).astype(np.uint64)
    for w in range(dim // 64):
        for b in range(64):
            words[:, w] |= bits[:, 64 * w + b] << np.uint64(b)
    for metric in (vx.SimilarityFunction.COSINE, vx.SimilarityFunction.EUCLIDEAN):
        index = vx.QuantizedFlatScanAdapter()
        index.build_bq(words, dim, metric)
        for call in range(2):
            q = torch.from_numpy(rng.standard_normal((200, dim)).astype(np.float32)).cuda()
            ref_ids, ref_sc, ref_cnt = index.scan_candidates_device(q, k)
            torch.cuda.synchronize()
            ids, sc, cnt = _noalloc(index, q, k)
            assert np.array_equal(cnt, ref_cnt.cpu().numpy()), (metric, call)
            assert np.array_equal(ids, ref_ids.cpu().numpy()), (metric, call)
            assert np.array_equal(sc, ref_sc.cpu().numpy()), (metric, call)
        index.close()


def test_no_alloc_scan_rejects_oversized_batch():
    import torch

    rng = np.random.default_rng(8)
    words = rng.integers(0, 2**63, size=(5000, 16), dtype=np.uint64)
    index = vx.QuantizedFlatScanAdapter()
    index.build_bq(words, 1024, vx.SimilarityFunction.COSINE)
    q = torch.zeros((20000, 1024), dtype=torch.float32, device="cuda")
    with pytest.raises(vx.VxError, match="scratch"):
        _noalloc(index, q, 500)
    index.close()
