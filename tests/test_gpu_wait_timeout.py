"""The device-side wait limit (VX_ERR_DEVICE_TIMEOUT) on a GPU, without a fault.

Every spin-wait of the scan kernels is bounded: when a wait runs out, the kernel records the
timeout, unwinds and returns, and the call reports VX_ERR_DEVICE_TIMEOUT with the context still
usable.  vx_debug_wait_timeout runs that bounded wait on a barrier nothing completes, so the wait
runs out by design; a search on the same device afterwards must still return the oracle's
results.
"""
import time

import numpy as np
import pytest

import vectors_b200 as vx
from vectors_b200 import _native as N

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_the_context_stays_usable(oracle):
    for limit_ms in (20, 200):
        t = time.perf_counter()
        status = N.lib().vx_debug_wait_timeout(0, limit_ms)
        waited = time.perf_counter() - t
        assert status == 7, (status, N.last_error())  # VX_ERR_DEVICE_TIMEOUT
        assert "time budget" in N.last_error()
        assert waited >= limit_ms / 1e3 * 0.9, waited
    db = oracle.gen_mixture(3000, 64, 8, 0.3, 1, 2, True)
    q = oracle.gen_mixture(16, 64, 8, 0.3, 1, 3, True)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction.COSINE)
    ids, sc, cnt = oracle.flat_search(db, q, oracle.COSINE, 10)
    for i, o in enumerate(f.search_batch(q, 10)):
        assert list(o.ordinals) == list(ids[i, :cnt[i]])
    f.close()


def test_wait_limit_is_validated():
    assert N.lib().vx_debug_wait_timeout(0, 0) == 1
    assert N.lib().vx_debug_wait_timeout(0, 20000) == 1
