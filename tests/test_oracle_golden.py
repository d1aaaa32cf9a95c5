"""Pins the CPU oracle against the reference's own known-answer tests (re-expressed here) and
published algorithms.  CPU only.

Sources (reference project paths):
  VectorUtilSupportTest.java:423-438,464-476  byte dot / L2 / Hamming known values
  BinaryQuantizerTest.java:55-75,484-532       sign-bit packing, zero -> 1, long packing
  BinaryQuantizerTest.java:150-227             BBQ: bits of v - centroid, (|v-c|^2, vl, width)
  ScalarQuantizerTest.java:606-631             INT4: packed size, nibble layout
  IvfIndexIntegrationTest.java:113-135         probing every list finds the brute-force neighbours
  TopKTest.java:55-135                         canonical top-k, ties by ordinal, infinities, NaN
  IndexSpiSearchBatchTest.java:47-93           batch == sequential
  QuantizedFlatScanAdapter.java:59-95          two-pass contract
"""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_byte_kernels_known_values(oracle):
    assert oracle.byte_dot([1, 2, 3, 4], [5, 6, 7, 8]) == 70
    assert oracle.byte_square_distance([1, 2, 3], [4, 6, 8]) == 50


def test_sq4_nibble_layout_and_size(oracle):
    # fromQuantiles(4, INT4, 0, 15): {0, 5, 10, 15} sit on the levels; low nibble = even dimension
    packed, _ = oracle.sq4_encode_all(0.0, 15.0, np.array([[0.0, 5.0, 10.0, 15.0]], np.float32))
    assert packed.shape == (1, 2)
    assert int(packed[0, 0]) & 0x0F == 0 and int(packed[0, 0]) >> 4 == 5
    assert int(packed[0, 1]) & 0x0F == 10 and int(packed[0, 1]) >> 4 == 15
    # ceil(129 / 2) = 65 bytes per vector
    packed, _ = oracle.sq4_encode_all(-1.0, 1.0, np.zeros((1, 129), np.float32))
    assert packed.shape == (1, 65)


def test_bbq_centres_before_the_sign_bit(oracle):
    # centroid [3, -3]: [2, -2] -> [-1, 1] -> bits 0b10; [4, -4] -> [1, -1] -> bits 0b01
    v = np.array([[2.0, -2.0], [4.0, -4.0]], np.float32)
    words, corr = oracle.bbq_encode_all(v, np.array([3.0, -3.0], np.float32))
    assert int(words[0, 0]) == 0x02 and int(words[1, 0]) == 0x01
    # corrections (|v - c|^2, min centred component, max - min)
    assert corr.tolist() == [[2.0, -1.0, 2.0], [2.0, -1.0, 2.0]]


def test_bbq_corrections_follow_their_definitions(oracle):
    rng = np.random.default_rng(42)
    v = rng.standard_normal((50, 64)).astype(np.float32)
    c = v.mean(0).astype(np.float32)
    _, corr = oracle.bbq_encode_all(v, c)
    x = v - c
    np.testing.assert_allclose(corr[:, 0], (x.astype(np.float64) ** 2).sum(1), rtol=0, atol=1e-3)
    assert np.array_equal(corr[:, 1], x.min(1))
    assert np.array_equal(corr[:, 2], x.max(1) - x.min(1))


def test_hamming_known_values(oracle):
    assert oracle.hamming([0xDEADBEEF, 0xCAFEBABE], [0xDEADBEEF, 0xCAFEBABE]) == 0
    assert oracle.hamming([0], [0xFF]) == 8
    assert oracle.hamming([0], [0xFFFFFFFFFFFFFFFF]) == 64


def test_sign_bit_packing(oracle):
    w = oracle.bq_encode_all(np.array([[1, -1, 1, -1, 1, -1, 1, -1]], np.float32))
    assert int(w[0, 0]) == 0x55
    w = oracle.bq_encode_all(np.array([[0.0, -1.0, 0.0, 1.0]], np.float32))
    assert int(w[0, 0]) == 0x0D  # zero becomes one (BinaryQuantizerTest.java:63)
    w = oracle.bq_encode_all(np.ones((1, 100), np.float32))
    assert int(w[0, 0]) == 0xFFFFFFFFFFFFFFFF and int(w[0, 1]) == (1 << 36) - 1
    assert int(oracle.bq_encode_all(np.full((1, 64), -5.0, np.float32))[0, 0]) == 0


def test_topk_select_reference_cases(oracle):
    assert list(oracle.topk_select([0.5, 0.5, 0.5, 0.5], 2)) == [0, 1]
    assert list(oracle.topk_select([0.5, 0.5, 0.5, 0.5], 4)) == [0, 1, 2, 3]
    assert list(oracle.topk_select([0.9, 0.5, 0.9, 0.3, 0.5], 4)) == [0, 2, 1, 4]
    assert list(oracle.topk_select([-1, 2, -3, 4, 0], 3)) == [3, 1, 4]
    assert list(oracle.topk_select([np.inf, 1, -np.inf, 2], 3)) == [0, 3, 1]
    assert list(oracle.topk_select([42.0], 5)) == [0]
    with pytest.raises(ValueError):
        oracle.topk_select([0.1, np.nan, 0.3], 2)


def test_topk_matches_full_sort(oracle):
    r = oracle.JavaRandom(1234)  # TopKTest.java:79-101
    s = np.array([r.next_float() for _ in range(1000)], np.float32)
    ref = sorted(range(1000), key=lambda i: (-s[i], i))[:10]
    assert list(oracle.topk_select(s, 10)) == ref


def test_java_random_published_values(oracle):
    assert oracle.JavaRandom(42).next_int() == -1170105035
    assert oracle.JavaRandom(0).next_int() == -1155484576
    assert oracle.JavaRandom(42).next_int(10) == 0
    assert oracle.JavaRandom(42).next_double() == 0.7275636800328681


def test_fp16_round_trip(oracle):
    L = oracle.lib()
    for v, h in [(1.0, 0x3C00), (-2.0, 0xC000), (65504.0, 0x7BFF), (65520.0, 0x7C00), (5.96e-8, 0x0001),
                 (0.0, 0x0000), (1.0 + 2 ** -11, 0x3C00), (1.0 + 3 * 2 ** -11, 0x3C02)]:
        assert L.vo_f32_to_f16(v) == h, (v, hex(L.vo_f32_to_f16(v)))
    xs = np.random.default_rng(0).standard_normal(10000).astype(np.float32)
    codes = oracle.fp16_encode_all(xs.reshape(1, -1))
    assert np.array_equal(codes[0], xs.astype(np.float16).view(np.uint16))
    back = np.array([L.vo_f16_to_f32(int(c)) for c in codes[0][:200]], np.float32)
    assert np.array_equal(back, xs[:200].astype(np.float16).astype(np.float32))


def test_bq_score_monotone_in_hamming(oracle):
    # ranking BQ rows by (h asc, id asc) equals ranking by (score desc, id asc)
    for dim in (64, 100, 768, 1024):
        for metric in range(4):
            s = [oracle.bq_score(metric, h, dim) for h in range(dim + 1)]
            assert all(a > b for a, b in zip(s, s[1:])), (dim, metric)


def test_dot_pinned_order_vs_float64(oracle):
    rng = np.random.default_rng(1)
    for n in (3, 16, 17, 31, 32, 33, 100, 768, 1000):
        a = rng.standard_normal(n).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        exact = float(np.dot(a.astype(np.float64), b.astype(np.float64)))
        bound = 1e-6 * float(np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)) * n
        assert abs(oracle.dot(a, b) - exact) <= bound + 1e-12


def test_similarity_transforms(oracle):
    a = np.array([1, 0, 0, 0], np.float32)
    b = np.array([0, 1, 0, 0], np.float32)
    assert oracle.compare(oracle.EUCLIDEAN, a, b) == np.float32(1.0) / np.float32(3.0)
    assert oracle.compare(oracle.DOT_PRODUCT, a, a) == 1.0
    assert oracle.compare(oracle.COSINE, a, b) == 0.5
    assert oracle.compare(oracle.MAXIMUM_INNER_PRODUCT, a, -a) == 0.5


def test_flat_policies_agree_without_ties(oracle):
    db = oracle.gen_mixture(3000, 64, 8, 0.3, 1, 2, True)
    q = oracle.gen_mixture(20, 64, 8, 0.3, 1, 3, True)
    for metric in range(4):
        a = oracle.flat_search(db, q, metric, 10, oracle.CANONICAL)
        b = oracle.flat_search(db, q, metric, 10, oracle.REFERENCE_HEAP)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_reference_heap_tie_semantics(oracle):
    # k=2, scores id0=x, id1=x, id2>x: the reference heap keeps {1, 2}; canonical keeps {2, 0}
    db = np.array([[1.0, 0.0], [1.0, 0.0], [1.0, 1.0]], np.float32)
    q = np.array([[1.0, 1.0]], np.float32)
    ref = oracle.flat_search(db, q, oracle.DOT_PRODUCT, 2, oracle.REFERENCE_HEAP)
    can = oracle.flat_search(db, q, oracle.DOT_PRODUCT, 2, oracle.CANONICAL)
    assert list(ref[0][0]) == [2, 1] and list(can[0][0]) == [2, 0]


def test_sq8_training_and_encoding(oracle):
    data = oracle.gen_mixture(30000, 32, 4, 0.3, 5, 6, False)
    lo, hi = oracle.sq8_train(data)
    assert lo < hi
    codes, corr = oracle.sq8_encode_all(lo, hi, data)
    assert codes.min() >= 0 and codes.max() <= 127
    # scores are reproducible through the per-pair score function
    L = oracle.lib()
    s = L.vo_sq8_score(oracle.DOT_PRODUCT, lo, hi, oracle.P(codes[0]), float(corr[0]), oracle.P(codes[1]),
                       float(corr[1]), 32)
    ids, sc, cnt = oracle.sq8_search(codes, corr, lo, hi, data[:1], oracle.DOT_PRODUCT, 5)
    assert np.isfinite(s) and cnt[0] == 5


def test_two_pass_equals_exact_when_candidates_cover(oracle):
    db = oracle.gen_mixture(500, 32, 4, 0.3, 7, 8, True)
    q = oracle.gen_mixture(5, 32, 4, 0.3, 7, 9, True)
    words = oracle.bq_encode_all(db)
    exact = oracle.flat_search(db, q, oracle.COSINE, 5)
    two = oracle.quantized_two_pass(1, words, None, 0.0, 0.0, db, q, oracle.COSINE, 5, 1000.0)
    assert np.array_equal(exact[0], two[0]) and np.array_equal(exact[1], two[1])


def test_ivfpq_sequential_table_sum(oracle):
    rng = np.random.default_rng(3)
    data = rng.standard_normal((400, 16)).astype(np.float32)
    cb = oracle.pq_train(data, 2, 16)
    codes = oracle.pq_encode_all(data, 2, 16, cb)
    cent = np.zeros((1, 16), np.float32)
    off, ords = oracle.build_ivf_lists(np.zeros(400, np.int32), 1)
    q = data[:3] + 0.01
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 2, 16, cb, codes, q, oracle.EUCLIDEAN, 5, 1)
    for i in range(3):
        t = oracle.pq_adc_table(q[i], 2, 16, cb)
        sums = np.array([np.float32(np.float32(0) + t[0, c[0]]) + t[1, c[1]] for c in codes], np.float32)
        order = sorted(range(400), key=lambda j: (sums[j], j))[:5]
        assert list(ids[i]) == order
        assert np.array_equal(sc[i], -sums[order])


def test_merge_shards_matches_unsharded(oracle):
    db = oracle.gen_mixture(2000, 48, 8, 0.3, 11, 12, True)
    q = oracle.gen_mixture(7, 48, 8, 0.3, 11, 13, True)
    full = oracle.flat_search(db, q, oracle.COSINE, 10)
    S = 4
    offs = [(2000 * i) // S for i in range(S + 1)]
    parts = [oracle.flat_search(db[offs[s]:offs[s + 1]], q, oracle.COSINE, 10) for s in range(S)]
    ids = np.stack([p[0] for p in parts])
    sc = np.stack([p[1] for p in parts])
    cnt = np.stack([p[2] for p in parts])
    m = oracle.merge_shards(np.array(offs[:S]), ids, sc, cnt, 10)
    assert np.array_equal(m[0], full[0]) and np.array_equal(m[1], full[1])


def test_golden_fixtures(oracle):
    """Committed fixtures (tests/golden/make_golden.py) regenerate bit-identically."""
    path = os.path.join(GOLDEN, "golden.json")
    with open(path) as f:
        g = json.load(f)
    from tests.golden.make_golden import compute

    now = compute(oracle)
    assert now == g


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_ivfflat_probing_every_list_is_the_flat_scan(oracle, metric):
    # nprobe = nlist visits every row, so IvfIndex.search returns the FlatScanAdapter neighbours
    # (scores differ in scale: -distance / dot / cosine against SimilarityFunction.compare)
    n, dim, nlist, k = 3000, 24, 8, 10
    db = oracle.gen_mixture(n, dim, 6, 0.3, 0xC0FFEE03, 0xC0FFEE01, False)
    q = oracle.gen_mixture(40, dim, 6, 0.3, 0xC0FFEE03, 0xC0FFEE02, False)
    cent = oracle.kmeans_train(db[:1000], nlist, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), nlist)
    i1, _, c1 = oracle.ivfflat_search(cent, off, ords, db, q, metric, k, nlist)
    i2, _, c2 = oracle.flat_search(db, q, metric, k)
    for j in range(len(q)):
        assert list(i1[j, : c1[j]]) == list(i2[j, : c2[j]]), j
