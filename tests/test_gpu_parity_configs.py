"""GPU parity at the benchmark workloads' own shapes (not toy sizes), against the CPU oracle.

* FLAT COSINE fp32, 100,000 x 768 from a 64-component mixture (sigma 0.3, L2-normalised),
  1,000 queries, k = 10: the whole workload, every query.
* IVF-PQ with the benchmark's table shape: 768 dims, M = 96 subspaces of 8 dims x 256
  centroids (uint8 codes, residual encoding), nlist 256, nprobe 32, on 200,000 rows of a
  1,024-component mixture; rescore 1 (pure ADC, bit-exact) and 4 (exact fp32 re-score).
* SQ8 DOT at the benchmark's 1,000,000 x 768 (the reference's global-quantile encoding),
  256 queries, k = 100, bit-exact.
* BQ sign-bit Hamming at 1,000,000 x 1,024 bits (256-component mixture, sigma 0.5), 256 queries,
  k = 100, bit-exact.
* FP16 DOT with fp32 queries (the reference's Fp16QuantizedVectors scoring) on 200,000 x 768
  L2-normalised rows, 512 queries, k = 100.

Bars as in test_gpu_parity.py: bit-exact ordinals and scores on the integer / code paths;
identical ordinals and scores within 1e-4 relative on the fp32 / fp16 paths.  The IVF-PQ
codebooks are drawn from residual sub-vectors instead of trained (training is an offline step;
the scan's arithmetic does not depend on how the codebook was made), so the case runs in
seconds.
"""
import numpy as np
import pytest

import vectors_b200 as vx

pytestmark = pytest.mark.gpu

SEED_C, SEED_DB, SEED_Q = 0xC0FFEE03, 0xC0FFEE01, 0xC0FFEE02
REL = 1e-4


def _check(got, ids, sc, cnt, tag, exact):
    bad = []
    for i, o in enumerate(got):
        c = cnt[i]
        if len(o.ordinals) != c or list(o.ordinals) != list(ids[i, :c]):
            bad.append(i)
            continue
        if exact:
            assert np.array_equal(o.scores, sc[i, :c]), f"{tag}: query {i} scores differ"
        else:
            np.testing.assert_allclose(o.scores, sc[i, :c], rtol=REL, atol=0, err_msg=f"{tag}: query {i}")
    assert not bad, f"{tag}: {len(bad)} of {len(got)} queries differ in ids, first {bad[:5]}"


def test_flat_cosine_100k_x_768_1000_queries(oracle):
    db = oracle.gen_mixture(100_000, 768, 64, 0.3, SEED_C + 1, SEED_DB + 1, True)
    q = oracle.gen_mixture(1000, 768, 64, 0.3, SEED_C + 1, SEED_Q + 1, True)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction.COSINE)
    got = f.search_batch(q, 10)
    ids, sc, cnt = oracle.flat_search(db, q, oracle.COSINE, 10)
    _check(got, ids, sc, cnt, "FLAT 100k x 768 COSINE", exact=False)
    f.close()


@pytest.fixture(scope="module")
def ivfpq_768(oracle):
    n, dim, nlist, m, ks = 200_000, 768, 256, 96, 256
    db = oracle.gen_mixture(n, dim, 1024, 0.3, SEED_C + 4, SEED_DB + 4, False)
    q = oracle.gen_mixture(500, dim, 1024, 0.3, SEED_C + 4, SEED_Q + 4, False)
    cent = oracle.kmeans_train(db[::8], nlist, 5, 42)
    assign = oracle.kmeans_assign(db, cent)
    off, ords = oracle.build_ivf_lists(assign, nlist)
    resid = db - cent[assign]
    pick = np.random.default_rng(5).choice(n, ks, replace=False)
    # codebooks concatenated per subspace: [m][ks][8]
    cb = np.ascontiguousarray(resid[pick].reshape(ks, m, dim // m).transpose(1, 0, 2)).reshape(-1)
    codes = oracle.pq_encode_all(resid, m, ks, cb)
    return db, q, cent, off, ords, cb, codes


@pytest.mark.parametrize("metric", [0, 1])
def test_ivfpq_m96_dim768_nlist256_nprobe32(oracle, ivfpq_768, metric):
    db, q, cent, off, ords, cb, codes = ivfpq_768
    a = vx.IvfPqAdapter(nprobe=32)
    a.build_prebuilt(cent, off, ords, cb, codes, 96, 256, vx.SimilarityFunction(metric), vectors=db)
    got = a.ivf_search(q, 10, 32)
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 96, 256, cb, codes, q, metric, 10, 32)
    _check(got, ids, sc, cnt, f"IVF-PQ M=96 m={metric}", exact=True)
    got = a.ivf_search(q, 10, 32, rescore_factor=4)
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 96, 256, cb, codes, q, metric, 10, 32, 4, db)
    _check(got, ids, sc, cnt, f"IVF-PQ M=96 rescore 4 m={metric}", exact=False)
    a.close()


def test_sq8_dot_1M_x_768_k100(oracle):
    n, dim = 1_000_000, 768
    db = oracle.gen_mixture(n, dim, 64, 0.3, SEED_C + 2, SEED_DB + 2, False)
    q = oracle.gen_mixture(256, dim, 64, 0.3, SEED_C + 2, SEED_Q + 2, False)
    lo, hi = oracle.sq8_train(db)
    codes, corr = oracle.sq8_encode_all(lo, hi, db)
    del db
    a = vx.QuantizedFlatScanAdapter()
    a.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction.DOT_PRODUCT)
    got = a.scan_candidates(q, 100)
    ids, sc, cnt = oracle.sq8_search(codes, corr, lo, hi, q, oracle.DOT_PRODUCT, 100)
    _check(got, ids, sc, cnt, "SQ8 1M x 768 DOT k=100", exact=True)
    a.close()


def test_bq_hamming_1M_x_1024_bits_k100(oracle):
    n, dim, chunk = 1_000_000, 1024, 125_000
    words = np.empty((n, dim // 64), np.uint64)
    for r in range(0, n, chunk):  # generated in slices: the fp32 rows are not kept
        part = oracle.gen_mixture(chunk, dim, 256, 0.5, SEED_C + 3, SEED_DB + 3, False, first_row=r)
        words[r:r + chunk] = oracle.bq_encode_all(part)
    q = oracle.gen_mixture(256, dim, 256, 0.5, SEED_C + 3, SEED_Q + 3, False)
    for metric in (oracle.DOT_PRODUCT, oracle.EUCLIDEAN):
        a = vx.QuantizedFlatScanAdapter()
        a.build_bq(words, dim, vx.SimilarityFunction(metric))
        got = a.scan_candidates(q, 100)
        ids, sc, cnt = oracle.bq_search(words, dim, q, metric, 100)
        _check(got, ids, sc, cnt, f"BQ 1M x 1024 bits m={metric} k=100", exact=True)
        a.close()


def test_fp16_dot_200k_x_768_k100(oracle):
    db = oracle.gen_mixture(200_000, 768, 4096, 0.3, SEED_C + 5, SEED_DB + 5, True)
    q = oracle.gen_mixture(512, 768, 4096, 0.3, SEED_C + 5, SEED_Q + 5, True)
    codes = oracle.fp16_encode_all(db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_fp16(codes, vx.SimilarityFunction.DOT_PRODUCT)
    got = a.scan_candidates(q, 100)
    ids, sc, cnt = oracle.fp16_search(codes, q, oracle.DOT_PRODUCT, 100)
    _check(got, ids, sc, cnt, "FP16 200k x 768 DOT k=100", exact=False)
    a.close()
