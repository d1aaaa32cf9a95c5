"""Child process for test_gpu_scan_variants.py: the scan variant is chosen by environment
variables that the library reads once per process (VX_GEMM_1SM, VX_SCAN_PILOT, VX_SCAN_POOL,
VX_BQ_TENSOR_BYTES, VX_BQ_WINDOW_BYTES, VX_ADC_GROUPED, VX_EPI_WARPS), so each variant runs in a process of its own.
Exits 0 when FLAT, SQ8, BQ and BBQ results (or, with the argument "ivf", IVF-PQ results) match
the oracle."""
import os
import sys

import numpy as np

import vectors_b200 as vx
from oracle import oracle as O


def ivf():
    """IVF-PQ (8-dim subspaces, 256 centroids): the ADC scan variants."""
    db = O.gen_mixture(20_000, 128, 32, 0.3, 0xC0FFEE03, 0xC0FFEE01, False)
    q = O.gen_mixture(300, 128, 32, 0.3, 0xC0FFEE03, 0xC0FFEE02, False)
    cent = O.kmeans_train(db[:5000], 8, 10, 42)
    assign = O.kmeans_assign(db, cent)
    off, ords = O.build_ivf_lists(assign, 8)
    resid = db - cent[assign]
    cb = O.pq_train(resid, 16, 256)
    codes = O.pq_encode_all(resid, 16, 256, cb)
    for metric in (0, 1):
        a = vx.IvfPqAdapter(nprobe=4)
        a.build_prebuilt(cent, off, ords, cb, codes, 16, 256, vx.SimilarityFunction(metric), vectors=db)
        got = a.ivf_search(q, 10, 4)
        ids, sc, cnt = O.ivfpq_search(cent, off, ords, 16, 256, cb, codes, q, metric, 10, 4)
        for i, o in enumerate(got):
            assert list(o.ordinals) == list(ids[i, : cnt[i]]), f"ivfpq m={metric} query {i}"
            assert np.array_equal(o.scores, sc[i, : cnt[i]]), f"ivfpq m={metric} query {i} scores"
        a.close()
    print("variant ok")
    return 0


def main():
    if sys.argv[1:] == ["ivf"]:
        return ivf()
    db = O.gen_mixture(120_000, 96, 8, 0.3, 0xC0FFEE03, 0xC0FFEE01, True)
    q = O.gen_mixture(300, 96, 8, 0.3, 0xC0FFEE03, 0xC0FFEE02, True)
    for metric in (0, 2):
        f = vx.FlatScanAdapter()
        f.build(db, vx.SimilarityFunction(metric))
        # k = 10, 100, 300: streams of 288, 544 and 1056 keys (544 on the 8-epilogue-warp build by
        # default, on the 4-warp one under VX_EPI_WARPS=4)
        for k in (10, 100, 300):
            got = f.search_batch(q, k)
            ids, sc, cnt = O.flat_search(db, q, metric, k)
            for i, o in enumerate(got):
                assert list(o.ordinals) == list(ids[i, : cnt[i]]), f"flat m={metric} k={k} query {i}"
                np.testing.assert_allclose(o.scores, sc[i, : cnt[i]], rtol=1e-4, atol=0)
        f.close()
    lo, hi = O.sq8_train(db)
    codes, corr = O.sq8_encode_all(lo, hi, db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction.DOT_PRODUCT)
    got = a.scan_candidates(q, 100)
    ids, sc, cnt = O.sq8_search(codes, corr, lo, hi, q, O.DOT_PRODUCT, 100)
    for i, o in enumerate(got):
        assert list(o.ordinals) == list(ids[i, : cnt[i]]), f"sq8 query {i}"
        assert np.array_equal(o.scores, sc[i, : cnt[i]]), f"sq8 query {i} scores"
    words = O.bq_encode_all(db)
    b = vx.QuantizedFlatScanAdapter()
    b.build_bq(words, 96, vx.SimilarityFunction.DOT_PRODUCT)
    # k = 1,200: wider than one candidate stream (1,023 keys), so the tensor scan takes two passes
    # (the popcount scan keeps up to 1,023 keys and refuses it)
    popcount = os.environ.get("VX_BQ_TENSOR_BYTES") == "0" and os.environ.get("VX_BQ_WINDOW_BYTES") == "0"
    for k in (100,) if popcount else (100, 1200):
        got = b.scan_candidates(q, k)
        ids, sc, cnt = O.bq_search(words, 96, q, O.DOT_PRODUCT, k)
        for i, o in enumerate(got):
            assert list(o.ordinals) == list(ids[i, : cnt[i]]), f"bq k={k} query {i}"
            assert np.array_equal(o.scores, sc[i, : cnt[i]]), f"bq k={k} query {i} scores"
    cent = db.mean(0).astype(np.float32)
    bw, bc = O.bbq_encode_all(db, cent)
    for metric in (0, 2):
        b = vx.QuantizedFlatScanAdapter()
        b.build_bbq(bw, bc, cent, 96, vx.SimilarityFunction(metric))
        got = b.scan_candidates(q, 100)
        ids, sc, cnt = O.bbq_search(bw, bc, cent, 96, q, metric, 100)
        for i, o in enumerate(got):
            assert list(o.ordinals) == list(ids[i, : cnt[i]]), f"bbq m={metric} query {i}"
            assert np.array_equal(o.scores, sc[i, : cnt[i]]), f"bbq m={metric} query {i} scores"
        b.close()
    print("variant ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
