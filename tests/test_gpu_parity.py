"""GPU parity: the CUDA scans (through the C ABI) against the CPU oracle on seeded inputs.

Bar: bit-exact ordinals and scores for the integer / code paths (SQ8, BQ, IVF-PQ ADC); for the
fp32 / fp16 paths identical ordinals and scores within 1e-4 relative (the exact re-score runs
in the reference's operation order, so scores are expected to agree to the bit as well).
"""
import numpy as np
import pytest

import vectors_b200 as vx

pytestmark = pytest.mark.gpu

SEED_C, SEED_DB, SEED_Q = 0xC0FFEE03, 0xC0FFEE01, 0xC0FFEE02
REL = 1e-4


def _check_float(got, ids, sc, cnt, tag, exact_scores=False):
    for i, o in enumerate(got):
        c = cnt[i]
        assert len(o.ordinals) == c, f"{tag}: query {i} count {len(o.ordinals)} != {c}"
        assert list(o.ordinals) == list(ids[i, :c]), f"{tag}: query {i} ids {o.ordinals[:8]} vs {ids[i, :8]}"
        if exact_scores:
            assert np.array_equal(o.scores, sc[i, :c]), f"{tag}: query {i} scores differ"
        else:
            np.testing.assert_allclose(o.scores, sc[i, :c], rtol=REL, atol=0, err_msg=tag)


def _data(O, n, dim, nq, comps=16, sigma=0.3, normalize=True):
    db = O.gen_mixture(n, dim, comps, sigma, SEED_C, SEED_DB, normalize)
    q = O.gen_mixture(nq, dim, comps, sigma, SEED_C, SEED_Q, normalize)
    return db, q


# ------------------------------------------------------------------ FLAT
@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("n,dim,nq,k", [(5000, 128, 64, 10), (3000, 100, 33, 7), (1000, 768, 10, 100), (257, 64, 130, 5)])
def test_flat_matches_oracle(oracle, metric, n, dim, nq, k):
    db, q = _data(oracle, n, dim, nq, normalize=(metric != 3))
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction(metric))
    got = f.search_batch(q, k)
    ids, sc, cnt = oracle.flat_search(db, q, metric, k)
    _check_float(got, ids, sc, cnt, f"flat m={metric} n={n} dim={dim}")
    f.close()


@pytest.mark.parametrize("metric", [0, 2])
def test_flat_large_with_pilot_floors(oracle, metric):
    # more rows than the pilot sweep, several query blocks: exercises the shared admission
    # floors and the floor-filtered merge
    db, q = _data(oracle, 120_000, 96, 300, comps=8)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction(metric))
    got = f.search_batch(q, 10)
    ids, sc, cnt = oracle.flat_search(db, q, metric, 10)
    _check_float(got, ids, sc, cnt, f"flat pilot m={metric}")


def test_sq8_large_with_pilot_floors(oracle):
    db, q = _data(oracle, 120_000, 128, 260, comps=8)
    lo, hi = oracle.sq8_train(db)
    codes, corr = oracle.sq8_encode_all(lo, hi, db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction.DOT_PRODUCT)
    got = a.scan_candidates(q, 100)
    ids, sc, cnt = oracle.sq8_search(codes, corr, lo, hi, q, oracle.DOT_PRODUCT, 100)
    _check_float(got, ids, sc, cnt, "sq8 pilot", exact_scores=True)


@pytest.mark.parametrize("metric", [0, 2])
def test_flat_wide_rows(oracle, metric):
    # 1536 dims: 24 K chunks per tile
    db, q = _data(oracle, 4000, 1536, 20, normalize=(metric != 3))
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction(metric))
    got = f.search_batch(q, 10)
    ids, sc, cnt = oracle.flat_search(db, q, metric, 10)
    _check_float(got, ids, sc, cnt, f"flat 1536 m={metric}")


def test_k_larger_than_index(oracle):
    # every row is returned, in canonical order, for FLAT, SQ8 and BQ
    db, q = _data(oracle, 50, 64, 7)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction.COSINE)
    ids, sc, cnt = oracle.flat_search(db, q, oracle.COSINE, 100)
    _check_float(f.search_batch(q, 100), ids, sc, cnt, "flat k > n")
    lo, hi = oracle.sq8_train(db)
    codes, corr = oracle.sq8_encode_all(lo, hi, db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction.DOT_PRODUCT)
    ids, sc, cnt = oracle.sq8_search(codes, corr, lo, hi, q, oracle.DOT_PRODUCT, 100)
    _check_float(a.scan_candidates(q, 100), ids, sc, cnt, "sq8 k > n", exact_scores=True)
    words = oracle.bq_encode_all(db)
    b = vx.QuantizedFlatScanAdapter()
    b.build_bq(words, 64, vx.SimilarityFunction.EUCLIDEAN)
    ids, sc, cnt = oracle.bq_search(words, 64, q, oracle.EUCLIDEAN, 100)
    _check_float(b.scan_candidates(q, 100), ids, sc, cnt, "bq k > n", exact_scores=True)


def test_flat_single_query_and_small_index(oracle):
    db, q = _data(oracle, 5, 32, 3)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction.COSINE)
    got = f.search_batch(q, 10)  # k > n
    ids, sc, cnt = oracle.flat_search(db, q, oracle.COSINE, 10)
    _check_float(got, ids, sc, cnt, "flat k>n")
    one = f.search(q[0], 3)
    assert list(one.ordinals) == list(ids[0, :3])


def test_flat_duplicates_take_exact_fallback(oracle):
    # many identical rows: the approximate window cannot separate them, so the exact scan
    # decides and ties resolve to the lowest ordinals
    rng = np.random.default_rng(0)
    base = rng.standard_normal((1, 64)).astype(np.float32)
    db = np.repeat(base, 600, axis=0)
    db[::7] += 0.5 * rng.standard_normal((len(db[::7]), 64)).astype(np.float32)
    q = base + 0.01 * rng.standard_normal((4, 64)).astype(np.float32)
    for metric in (1, 2):
        f = vx.FlatScanAdapter()
        f.build(db, vx.SimilarityFunction(metric))
        got = f.search_batch(q, 20)
        ids, sc, cnt = oracle.flat_search(db, q, metric, 20)
        _check_float(got, ids, sc, cnt, f"flat duplicates m={metric}")


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_flat_near_duplicates_take_second_pass(oracle, metric):
    # 500 rows within 1e-4 of each other around the queries: the 128-candidate window cannot
    # prove completeness, the 1000-candidate second pass can
    rng = np.random.default_rng(1)
    base = rng.standard_normal((1, 96)).astype(np.float32)
    near = base + 1e-4 * rng.standard_normal((500, 96)).astype(np.float32)
    far = rng.standard_normal((4000, 96)).astype(np.float32)
    db = np.concatenate([far[:2000], near, far[2000:]])
    q = base + 1e-3 * rng.standard_normal((6, 96)).astype(np.float32)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction(metric))
    got = f.search_batch(q, 10)
    ids, sc, cnt = oracle.flat_search(db, q, metric, 10)
    _check_float(got, ids, sc, cnt, f"flat near-duplicates m={metric}")


def test_flat_many_duplicates_exact_fallback(oracle):
    rng = np.random.default_rng(2)
    base = rng.standard_normal((1, 64)).astype(np.float32)
    db = np.concatenate([rng.standard_normal((3000, 64)).astype(np.float32), np.repeat(base, 2500, axis=0)])
    q = base + 0.01 * rng.standard_normal((3, 64)).astype(np.float32)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction.DOT_PRODUCT)
    got = f.search_batch(q, 10)
    ids, sc, cnt = oracle.flat_search(db, q, oracle.DOT_PRODUCT, 10)
    _check_float(got, ids, sc, cnt, "flat many duplicates")


def test_flat_empty_index(oracle):
    f = vx.FlatScanAdapter()
    f.build(np.zeros((0, 0), np.float32), vx.SimilarityFunction.COSINE)
    out = f.search_batch(np.ones((2, 8), np.float32), 4)
    assert [len(o.ordinals) for o in out] == [0, 0]


def test_flat_dimension_mismatch(oracle):
    db, q = _data(oracle, 100, 16, 2)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction.COSINE)
    with pytest.raises(vx.IllegalArgumentException, match="dimension"):
        f.search_batch(np.ones((2, 17), np.float32), 4)


# ------------------------------------------------------------------ SQ8
@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("n,dim,nq,k", [(6000, 768, 40, 100), (2500, 100, 129, 10)])
def test_sq8_bit_exact(oracle, metric, n, dim, nq, k):
    db, q = _data(oracle, n, dim, nq)
    lo, hi = oracle.sq8_train(db)
    codes, corr = oracle.sq8_encode_all(lo, hi, db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction(metric))
    got = a.scan_candidates(q, k)
    ids, sc, cnt = oracle.sq8_search(codes, corr, lo, hi, q, metric, k)
    _check_float(got, ids, sc, cnt, f"sq8 m={metric}", exact_scores=True)


def test_sq8_two_pass(oracle):
    db, q = _data(oracle, 4000, 128, 20)
    lo, hi = oracle.sq8_train(db)
    codes, corr = oracle.sq8_encode_all(lo, hi, db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction.DOT_PRODUCT, vectors=db)
    got = a.search_batch(q, 10, 0, 4.0)
    ids, sc, cnt = oracle.quantized_two_pass(0, codes, corr, lo, hi, db, q, oracle.DOT_PRODUCT, 10, 4.0)
    _check_float(got, ids, sc, cnt, "sq8 two-pass")
    got = a.search_batch(q, 10, 0, 1.0)  # oqf <= 1 delegates to the exact scan
    ids, sc, cnt = oracle.flat_search(db, q, oracle.DOT_PRODUCT, 10)
    _check_float(got, ids, sc, cnt, "sq8 exact delegate")


# ------------------------------------------------------------------ BQ
@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("n,dim,nq,k", [(20000, 1024, 300, 100), (3000, 100, 17, 10), (999, 64, 5, 3)])
def test_bq_bit_exact(oracle, metric, n, dim, nq, k):
    db, q = _data(oracle, n, dim, nq, sigma=0.5, normalize=False)
    words = oracle.bq_encode_all(db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_bq(words, dim, vx.SimilarityFunction(metric))
    got = a.scan_candidates(q, k)
    ids, sc, cnt = oracle.bq_search(words, dim, q, metric, k)
    _check_float(got, ids, sc, cnt, f"bq m={metric} dim={dim}", exact_scores=True)


def test_bq_all_equal_rows_ties_by_ordinal(oracle):
    db = np.ones((5000, 128), np.float32)
    q = np.ones((3, 128), np.float32)
    words = oracle.bq_encode_all(db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_bq(words, 128, vx.SimilarityFunction.COSINE)
    got = a.scan_candidates(q, 50)
    for o in got:
        assert list(o.ordinals) == list(range(50))


# ------------------------------------------------------------------ FP16
@pytest.mark.parametrize("metric", [0, 1, 2, 3])
def test_fp16_candidates_match_oracle(oracle, metric):
    db, q = _data(oracle, 6000, 256, 50, normalize=(metric != 3))
    codes = oracle.fp16_encode_all(db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_fp16(codes, vx.SimilarityFunction(metric))
    got = a.scan_candidates(q, 100)
    ids, sc, cnt = oracle.fp16_search(codes, q, metric, 100)
    _check_float(got, ids, sc, cnt, f"fp16 m={metric}")


# ------------------------------------------------------------------ IVF-PQ
def _ivf(oracle, n=20000, dim=64, nlist=64, m=8, ks=256, comps=32):
    db = oracle.gen_mixture(n, dim, comps, 0.3, SEED_C, SEED_DB, False)
    q = oracle.gen_mixture(40, dim, comps, 0.3, SEED_C, SEED_Q, False)
    cent = oracle.kmeans_train(db[:5000], nlist, 10, 42)
    assign = oracle.kmeans_assign(db, cent)
    off, ords = oracle.build_ivf_lists(assign, nlist)
    resid = db - cent[assign]
    cb = oracle.pq_train(resid, m, ks)
    codes = oracle.pq_encode_all(resid, m, ks, cb)
    return db, q, cent, off, ords, cb, codes


@pytest.mark.parametrize("metric", [0, 1])
@pytest.mark.parametrize("dim,nlist", [(64, 64), (96, 30)])
def test_ivfpq_bit_exact(oracle, metric, dim, nlist):
    # (64, 64): tiled routing; (96, 30): per-row routing (dim not a multiple of 64) with two
    # centroids outside the 4-row groups, 12-dim subspaces on the general ADC kernel
    db, q, cent, off, ords, cb, codes = _ivf(oracle, dim=dim, nlist=nlist)
    a = vx.IvfPqAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, cb, codes, 8, 256, vx.SimilarityFunction(metric), vectors=db)
    got = a.ivf_search(q, 10, 8)
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 8, 256, cb, codes, q, metric, 10, 8)
    _check_float(got, ids, sc, cnt, f"ivfpq m={metric}", exact_scores=True)
    got = a.ivf_search(q, 10, 8, rescore_factor=4)
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 8, 256, cb, codes, q, metric, 10, 8, 4, db)
    _check_float(got, ids, sc, cnt, f"ivfpq rescore m={metric}")


@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("nlist", [32, 4])
def test_ivfpq_grouped_bit_exact(oracle, metric, nlist):
    # 8-dim subspaces, 256 centroids, M a multiple of 16: the grouped ADC kernel (up to four
    # queries per list, chunked tables); nlist=4 gives lists longer than one row pass
    db, q, cent, off, ords, cb, codes = _ivf(oracle, n=20000, dim=128, nlist=nlist, m=16)
    a = vx.IvfPqAdapter(nprobe=4)
    a.build_prebuilt(cent, off, ords, cb, codes, 16, 256, vx.SimilarityFunction(metric), vectors=db)
    got = a.ivf_search(q, 10, 4)
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 16, 256, cb, codes, q, metric, 10, 4)
    _check_float(got, ids, sc, cnt, f"ivfpq grouped m={metric} nlist={nlist}", exact_scores=True)
    got = a.ivf_search(q, 10, 4, rescore_factor=4)
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 16, 256, cb, codes, q, metric, 10, 4, 4, db)
    _check_float(got, ids, sc, cnt, f"ivfpq grouped rescore m={metric} nlist={nlist}")


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_ivfpq_many_queries_per_list_bit_exact(oracle, metric):
    # 400 queries x 8 probes over 16 lists: ~200 pairs per list, so ~50 four-query groups
    # scan each list one after another and every query's floor is carried across its eight
    # lists; rescore 2 and 4 widen the kept candidates (K = 20, 40).
    db, _, cent, off, ords, cb, codes = _ivf(oracle, n=20000, dim=128, nlist=16, m=16)
    q = oracle.gen_mixture(400, 128, 32, 0.3, SEED_C, SEED_Q + 7, False)
    a = vx.IvfPqAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, cb, codes, 16, 256, vx.SimilarityFunction(metric), vectors=db)
    got = a.ivf_search(q, 10, 8)
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 16, 256, cb, codes, q, metric, 10, 8)
    _check_float(got, ids, sc, cnt, f"ivfpq many m={metric}", exact_scores=True)
    for rf in (2, 4):
        got = a.ivf_search(q, 10, 8, rescore_factor=rf)
        ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 16, 256, cb, codes, q, metric, 10, 8, rf, db)
        _check_float(got, ids, sc, cnt, f"ivfpq many rescore {rf} m={metric}")


# ------------------------------------------------------------------ SQ4
@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("n,dim,nq,k", [(6000, 768, 40, 100), (2500, 101, 65, 10)])
def test_sq4_bit_exact(oracle, metric, n, dim, nq, k):
    # ScalarQuantizedVectors INT4: nibble codes unpacked to bytes, the exact int8 tensor scan
    # with the INT4 constants (maxValue 15); odd dim leaves the last byte's high nibble unused
    db, q = _data(oracle, n, dim, nq, normalize=(metric != 3))
    lo, hi = oracle.sq8_train(db)
    packed, corr = oracle.sq4_encode_all(lo, hi, db)
    a = vx.QuantizedFlatScanAdapter()
    a.build_sq4(packed, corr, dim, lo, hi, vx.SimilarityFunction(metric), vectors=db)
    got = a.scan_candidates(q, k)
    ids, sc, cnt = oracle.sq4_search(packed, corr, dim, lo, hi, q, metric, k)
    _check_float(got, ids, sc, cnt, f"sq4 m={metric} dim={dim}", exact_scores=True)
    # the two-pass contract (candidates re-scored in fp32) on top of the SQ4 scan
    two = a.search_batch(q, 10, over_query_factor=4.0)
    ci, cs, cc = oracle.sq4_search(packed, corr, dim, lo, hi, q, metric, oracle.candidate_k(10, 4.0))
    ids, sc, cnt = oracle.rescore_candidates(db, q, metric, ci, cc, 10)
    _check_float(two, ids, sc, cnt, f"sq4 two-pass m={metric} dim={dim}")
    a.close()


# ------------------------------------------------------------------ BBQ
@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("n,dim,nq,k", [(6000, 768, 40, 100), (2500, 100, 65, 10), (1000, 1024, 20, 5),
                                        (90000, 256, 300, 100), (3000, 1536, 30, 10), (2000, 2048, 20, 10)])
def test_bbq_bit_exact(oracle, metric, n, dim, nq, k):
    # BinaryQuantizedVectors BBQ: 4-bit query codes against centroid-relative sign bits, the
    # exact asymmetric dot (int8 tensor cores), computeBbqDot and the metric transform in Java's
    # order; 90,000 rows also take the pilot sweep's floors and several row tiles per unit
    db, q = _data(oracle, n, dim, nq, normalize=(metric == 2))
    cent = db.mean(0).astype(np.float32)
    words, corr = oracle.bbq_encode_all(db, cent)
    a = vx.QuantizedFlatScanAdapter()
    a.build_bbq(words, corr, cent, dim, vx.SimilarityFunction(metric), vectors=db)
    got = a.scan_candidates(q, k)
    ids, sc, cnt = oracle.bbq_search(words, corr, cent, dim, q, metric, k)
    _check_float(got, ids, sc, cnt, f"bbq m={metric} dim={dim}", exact_scores=True)
    two = a.search_batch(q, 5, over_query_factor=4.0)
    ci, cs, cc = oracle.bbq_search(words, corr, cent, dim, q, metric, oracle.candidate_k(5, 4.0))
    ids, sc, cnt = oracle.rescore_candidates(db, q, metric, ci, cc, 5)
    _check_float(two, ids, sc, cnt, f"bbq two-pass m={metric} dim={dim}")
    a.close()


# ------------------------------------------------------------------ IVF-flat
@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("dim,nq,k", [(128, 400, 10), (96, 50, 50), (100, 40, 10), (7, 30, 5)])
def test_ivfflat_matches_oracle(oracle, metric, dim, nq, k):
    # dims: whole 64-dim chunks, a zero-padded last chunk, 4 dims after the 8-lane part, no
    # lane part at all; 400 queries x 8 probes over 16 lists puts several 64-query groups on
    # each list; every list ends in a batch whose count % 4 rows take the scalar functions
    n, nlist = 9000, 16
    db = oracle.gen_mixture(n, dim, 12, 0.3, SEED_C, SEED_DB, metric == 2)
    q = oracle.gen_mixture(nq, dim, 12, 0.3, SEED_C, SEED_Q, metric == 2)
    cent = oracle.kmeans_train(db[:3000], nlist, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), nlist)
    a = vx.IvfFlatAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction(metric))
    got = a.ivf_search(q, k, 8)
    # the reference's search in full: EUCLIDEAN stops early against the partitions' radii
    radii = oracle.ivf_radii(cent, off, ords, db)
    ids, sc, cnt = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, metric, k, 8)
    for i, o in enumerate(got):
        c = cnt[i]
        assert list(o.ordinals) == list(ids[i, :c]), f"ivfflat m={metric} dim={dim} query {i}"
        if metric == 2:
            np.testing.assert_allclose(o.scores, sc[i, :c], rtol=1e-6, atol=0)
        else:
            assert np.array_equal(o.scores, sc[i, :c]), f"ivfflat m={metric} dim={dim} query {i} scores"
    # IndexSpi.searchBatch: the adapter's nprobe, and overQueryFactor widening the probes
    _same_outcomes(a.search_batch(q, k), got, "ivfflat searchBatch")
    # IvfFlatAdapter.search: candidateK = ceil(k * 1.5) hits from ceil(8 * 1.5) probes, trimmed to k
    wide = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, metric, oracle.candidate_k(k, 1.5), 12)
    got2 = a.search_batch(q, k, over_query_factor=1.5)
    for i, o in enumerate(got2):
        assert list(o.ordinals) == list(wide[0][i, : min(k, wide[2][i])]), f"ivfflat oqf query {i}"
    a.close()


@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("k", [10, 100])
def test_ivfflat_long_lists_in_row_parts_match_oracle(oracle, metric, k):
    # lists of ~5,000 rows: each is scanned as row parts of 1,024 rows (several groups per list,
    # a part's K best merged per pair afterwards), and the last part holds the list's trailing
    # batch; the EUCLIDEAN early exit then runs on the merged per-list results
    n, nlist, dim = 40_000, 8, 64
    db = oracle.gen_mixture(n, dim, 8, 0.3, SEED_C, SEED_DB, metric == 2)
    q = oracle.gen_mixture(150, dim, 8, 0.3, SEED_C, SEED_Q, metric == 2)
    cent = oracle.kmeans_train(db[:8000], nlist, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), nlist)
    assert np.diff(off).max() > 2048
    a = vx.IvfFlatAdapter(nprobe=4)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction(metric))
    got = a.ivf_search(q, k, 4)
    radii = oracle.ivf_radii(cent, off, ords, db)
    ids, sc, cnt = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, metric, k, 4)
    for i, o in enumerate(got):
        c = cnt[i]
        assert list(o.ordinals) == list(ids[i, :c]), f"ivfflat parts m={metric} k={k} query {i}"
        if metric == 2:
            np.testing.assert_allclose(o.scores, sc[i, :c], rtol=1e-6, atol=0)
        else:
            assert np.array_equal(o.scores, sc[i, :c]), f"ivfflat parts m={metric} k={k} query {i} scores"
    a.close()


def _same_outcomes(x, y, tag):
    for i, (u, v) in enumerate(zip(x, y)):
        assert np.array_equal(u.ordinals, v.ordinals) and np.array_equal(u.scores, v.scores), f"{tag} query {i}"


@pytest.mark.parametrize("metric", [0, 1, 2])
@pytest.mark.parametrize("dim,nlist", [(64, 64), (96, 30)])
def test_ivf_route_device_matches_oracle_and_routed_search(oracle, metric, dim, nlist):
    import torch

    db, q, cent, off, ords, cb, codes = _ivf(oracle, dim=dim, nlist=nlist)
    a = vx.IvfPqAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, cb, codes, 8, 256, vx.SimilarityFunction(metric))
    qd = torch.from_numpy(q).cuda()
    lists = a.route_device(qd, 8)
    torch.cuda.synchronize()
    ref, _ = oracle.route(cent, q, metric, 8)
    assert np.array_equal(lists.cpu().numpy(), ref), "routing differs from the oracle"
    # routed search over the same lists == the one-call search
    i1, s1, c1 = a.ivf_search_device(qd, 10, 8)
    i2, s2, c2 = a.ivf_search_routed_device(qd, 10, 8, lists)
    torch.cuda.synchronize()
    assert torch.equal(i1, i2) and torch.equal(s1, s2) and torch.equal(c1, c2)
    bad = lists.clone()
    bad[0, 0] = nlist + 5
    with pytest.raises(vx.IllegalArgumentException):
        a.ivf_search_routed_device(qd, 10, 8, bad)


@pytest.mark.parametrize("m,dim", [(16, 128), (8, 96)])
def test_ivfpq_list_sharded_equals_unsharded(oracle, m, dim):
    # two indexes holding the even / odd lists (global ordinals, the other lists empty), searched
    # with the same routed lists and merged with zero offsets == the unsharded index; covers
    # both ADC kernels and the skipping of lists without rows
    import torch

    db, q, cent, off, ords, cb, codes = _ivf(oracle, dim=dim, nlist=32, m=m)
    full = vx.IvfPqAdapter(nprobe=8)
    full.build_prebuilt(cent, off, ords, cb, codes, m, 256, vx.SimilarityFunction.EUCLIDEAN)
    qd = torch.from_numpy(q).cuda()
    lists = full.route_device(qd, 8)
    ref = full.ivf_search_device(qd, 10, 8)
    parts = []
    for r in range(2):
        own = [l for l in range(32) if l % 2 == r]
        sizes = np.zeros(32, np.int64)
        order = []
        for l in own:
            sizes[l] = off[l + 1] - off[l]
            order.append(ords[off[l]:off[l + 1]])
        loff = np.zeros(33, np.int64)
        loff[1:] = np.cumsum(sizes)
        a = vx.IvfPqAdapter(nprobe=8)
        a.build_prebuilt(cent, loff, np.concatenate(order), cb, codes, m, 256, vx.SimilarityFunction.EUCLIDEAN)
        parts.append(a.ivf_search_routed_device(qd, 10, 8, lists))
    ids = torch.stack([p_[0] for p_ in parts])
    sc = torch.stack([p_[1] for p_ in parts])
    cnt = torch.stack([p_[2] for p_ in parts])
    mi, ms, mc = vx.merge_shards_device(ids, sc, cnt, torch.zeros(2, dtype=torch.int64), 10)
    torch.cuda.synchronize()
    assert torch.equal(mi, ref[0]) and torch.equal(ms, ref[1]) and torch.equal(mc, ref[2])


def test_ivfpq_balanced_masks_equal_unsharded(oracle):
    # the replicated-index balanced mode of vectors_b200.sharded.ivf_search_balanced, two ranks
    # emulated on one GPU: lists dealt by assign_lists, each rank scans only its lists' pairs
    import torch

    from vectors_b200.sharded import assign_lists

    db, q, cent, off, ords, cb, codes = _ivf(oracle, dim=128, nlist=32, m=16)
    a = vx.IvfPqAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, cb, codes, 16, 256, vx.SimilarityFunction.EUCLIDEAN)
    qd = torch.from_numpy(q).cuda()
    ref = a.ivf_search_device(qd, 10, 8)
    lists = a.route_device(qd, 8)
    flat = lists.reshape(-1).long()
    rows = torch.from_numpy(np.diff(off)).cuda()
    owner = assign_lists(torch.bincount(flat, minlength=32), rows, 2)
    parts = []
    for r in range(2):
        mine = torch.where(owner[lists.long()] == r, lists, torch.full_like(lists, -1))
        parts.append(a.ivf_search_routed_device(qd, 10, 8, mine))
    ids = torch.stack([p_[0] for p_ in parts])
    sc = torch.stack([p_[1] for p_ in parts])
    cnt = torch.stack([p_[2] for p_ in parts])
    mi, ms, mc = vx.merge_shards_device(ids, sc, cnt, torch.zeros(2, dtype=torch.int64), 10)
    torch.cuda.synchronize()
    assert torch.equal(mi, ref[0]) and torch.equal(ms, ref[1]) and torch.equal(mc, ref[2])


@pytest.mark.parametrize("world", [2, 3])
def test_ivfpq_pair_split_equals_unsplit(oracle, world):
    # vectors_b200.sharded.ivf_search_pair_split, the ranks emulated on one GPU: every list's
    # pairs dealt over the ranks in four-pair table groups, each rank scans its pairs only
    import torch

    from vectors_b200.sharded import deal_pairs

    db, q, cent, off, ords, cb, codes = _ivf(oracle, dim=128, nlist=32, m=16)
    a = vx.IvfPqAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, cb, codes, 16, 256, vx.SimilarityFunction.EUCLIDEAN)
    qd = torch.from_numpy(q).cuda()
    ref = a.ivf_search_device(qd, 10, 8)
    lists = a.route_device(qd, 8)
    parts = [a.ivf_search_routed_device(qd, 10, 8, deal_pairs(lists, r, world)) for r in range(world)]
    ids = torch.stack([p_[0] for p_ in parts])
    sc = torch.stack([p_[1] for p_ in parts])
    cnt = torch.stack([p_[2] for p_ in parts])
    mi, ms, mc = vx.merge_shards_device(ids, sc, cnt, torch.zeros(world, dtype=torch.int64), 10)
    torch.cuda.synchronize()
    assert torch.equal(mi, ref[0]) and torch.equal(ms, ref[1]) and torch.equal(mc, ref[2])
    ids_o, sc_o, cnt_o = oracle.ivfpq_search(cent, off, ords, 16, 256, cb, codes, q, oracle.EUCLIDEAN, 10, 8)
    assert np.array_equal(mc.cpu().numpy(), cnt_o)
    for i in range(q.shape[0]):
        assert list(mi[i, : cnt_o[i]].cpu().numpy()) == list(ids_o[i, : cnt_o[i]])
        assert np.array_equal(ms[i, : cnt_o[i]].cpu().numpy(), sc_o[i, : cnt_o[i]])
    a.close()


def test_ivfpq_routing_matches_oracle(oracle):
    db, q, cent, off, ords, cb, codes = _ivf(oracle)
    lids, _ = oracle.route(cent, q, oracle.EUCLIDEAN, 8)
    ref_lids, _ = oracle.route(cent, q, oracle.EUCLIDEAN, 8, oracle.REFERENCE_HEAP)
    assert np.array_equal(np.sort(lids, 1), np.sort(ref_lids, 1))


# ------------------------------------------------------------------ shards
def test_merge_shards_device(oracle):
    import torch

    db, q = _data(oracle, 3000, 64, 9)
    S = 3
    offs = vx.shard_offsets(3000, S)
    parts = []
    for s in range(S):
        f = vx.FlatScanAdapter()
        f.build(db[offs[s]:offs[s + 1]], vx.SimilarityFunction.COSINE)
        ids, sc, cnt = f.search_batch_device(torch.from_numpy(q).cuda(), 10)
        parts.append((ids, sc, cnt))
        f.close()
    ids = torch.stack([p[0] for p in parts])
    sc = torch.stack([p[1] for p in parts])
    cnt = torch.stack([p[2] for p in parts])
    mi, ms, mc = vx.merge_shards_device(ids, sc, cnt, torch.tensor(offs[:S]), 10)
    torch.cuda.synchronize()
    ref = oracle.flat_search(db, q, oracle.COSINE, 10)
    assert np.array_equal(mi.cpu().numpy(), ref[0])
    np.testing.assert_allclose(ms.cpu().numpy(), ref[1], rtol=REL)


# ------------------------------------------------------------------ threading
def test_concurrent_searches_equal_serial(oracle):
    # an index is safe for concurrent searches from several host threads (the facade's read
    # lock, FlatScanAdapter.java:31-33): two threads searching one FLAT and one SQ8 index at
    # once return what the same calls return one after another
    import threading

    db, q = _data(oracle, 40_000, 256, 300)
    f = vx.FlatScanAdapter()
    f.build(db, vx.SimilarityFunction.COSINE)
    lo, hi = oracle.sq8_train(db)
    codes, corr = oracle.sq8_encode_all(lo, hi, db)
    s = vx.QuantizedFlatScanAdapter()
    s.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction.DOT_PRODUCT, vectors=db)
    calls = [lambda i=i: f.search_batch(q[i::2], 10) for i in range(2)]
    calls += [lambda i=i: s.search_batch(q[i::2], 10, 0, 4.0) for i in range(2)]
    serial = [c() for c in calls]
    results = [[None] * len(calls) for _ in range(3)]
    errors = []

    def run(rep, j):
        try:
            results[rep][j] = calls[j]()
        except Exception as e:  # pragma: no cover - reported below
            errors.append(e)

    for rep in range(3):
        threads = [threading.Thread(target=run, args=(rep, j)) for j in range(len(calls))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
    assert not errors, errors
    for rep in range(3):
        for j in range(len(calls)):
            _same_outcomes(results[rep][j], serial[j], f"concurrent rep {rep} call {j}")
    f.close()
    s.close()


# ------------------------------------------------------------------ wide candidate windows
@pytest.mark.parametrize("kind", ["sq8", "bq", "bbq"])
def test_candidate_windows_wider_than_one_stream(oracle, kind):
    # more candidates per query than one stream keeps (1,023) are taken in passes below the
    # previous pass's smallest key: k = 300 at overQueryFactor 4 (1,200 candidates, two passes)
    # and a 2,100-candidate scan (three passes), against the oracle
    n, dim = 30000, 128 if kind == "sq8" else 256
    db, q = _data(oracle, n, dim, 20, normalize=kind != "bq")
    a = vx.QuantizedFlatScanAdapter()
    if kind == "sq8":
        lo, hi = oracle.sq8_train(db)
        codes, corr = oracle.sq8_encode_all(lo, hi, db)
        a.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction.DOT_PRODUCT, vectors=db)
        scan = lambda kk: oracle.sq8_search(codes, corr, lo, hi, q, oracle.DOT_PRODUCT, kk)  # noqa: E731
    elif kind == "bq":
        words = oracle.bq_encode_all(db)
        a.build_bq(words, dim, vx.SimilarityFunction.DOT_PRODUCT, vectors=db)
        scan = lambda kk: oracle.bq_search(words, dim, q, oracle.DOT_PRODUCT, kk)  # noqa: E731
    else:
        cent = db.mean(0).astype(np.float32)
        words, corr = oracle.bbq_encode_all(db, cent)
        a.build_bbq(words, corr, cent, dim, vx.SimilarityFunction.DOT_PRODUCT, vectors=db)
        scan = lambda kk: oracle.bbq_search(words, corr, cent, dim, q, oracle.DOT_PRODUCT, kk)  # noqa: E731
    got = a.scan_candidates(q, 2100)
    _check_float(got, *scan(2100), f"{kind} 2100 candidates", exact_scores=True)
    two = a.search_batch(q, 300, 0, 4.0)
    ci, cs, cc = scan(oracle.candidate_k(300, 4.0))
    _check_float(two, *oracle.rescore_candidates(db, q, oracle.DOT_PRODUCT, ci, cc, 300), f"{kind} k=300 oqf=4")
    a.close()
