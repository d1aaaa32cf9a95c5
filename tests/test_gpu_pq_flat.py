"""GPU parity of PQ as a flat quantizer (QuantizerKind.PQ behind QuantizedFlatScanAdapter:
PQVectors.scoreFunctionFor, PQVectors.java:104-191) against the oracle's restatement.

Bit-exact ordinals and scores for the candidate scan (every metric, with and without a global
centroid, on the grouped ADC kernel -- 8-dim subspaces x 256 centroids -- and on the general one);
the two-pass searchBatch (candidates re-scored in fp32) within 1e-4; a quantized.bin PQ payload
opens the same index.
"""
import numpy as np
import pytest

import vectors_b200 as vx
from oracle import formats as F

pytestmark = pytest.mark.gpu

SEED_C, SEED_DB, SEED_Q = 0xC0FFEE03, 0xC0FFEE01, 0xC0FFEE02


def _pq(oracle, n, dim, m, ks, center, normalize):
    db = oracle.gen_mixture(n, dim, 16, 0.3, SEED_C, SEED_DB, normalize)
    q = oracle.gen_mixture(70, dim, 16, 0.3, SEED_C, SEED_Q, normalize)
    gc = db.mean(0).astype(np.float32) if center else None
    x = db - gc if center else db
    cb = oracle.pq_train(x[:4000], m, ks)
    codes = oracle.pq_encode_all(x, m, ks, cb)
    return db, q, gc, cb, codes


def _same(got, ids, sc, cnt, tag, exact=True):
    for i, o in enumerate(got):
        c = cnt[i]
        assert list(o.ordinals) == list(ids[i, :c]), f"{tag}: query {i}"
        if exact:
            assert np.array_equal(o.scores, sc[i, :c]), f"{tag}: query {i} scores"
        else:
            np.testing.assert_allclose(o.scores, sc[i, :c], rtol=1e-4, atol=0, err_msg=f"{tag}: query {i}")


@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("center", [False, True])
@pytest.mark.parametrize("n,dim,m,ks", [(20000, 128, 16, 256), (5000, 96, 8, 256), (3000, 100, 10, 64)])
def test_pq_candidates_bit_exact(oracle, metric, center, n, dim, m, ks):
    # (128, 16, 256): grouped ADC kernel; (96, 8): 12-dim subspaces and (100, 10, 64): 64
    # centroids, both on the general ADC kernel
    db, q, gc, cb, codes = _pq(oracle, n, dim, m, ks, center, metric == 2)
    a = vx.QuantizedFlatScanAdapter()
    a.build_pq(codes, cb, m, ks, vx.SimilarityFunction(metric), global_centroid=gc, vectors=db)
    for k in (10, 100):
        got = a.scan_candidates(q, k)
        _same(got, *oracle.pq_flat_search(cb, codes, dim, m, ks, q, metric, k, global_centroid=gc),
              f"pq m={metric} gc={center} dim={dim} k={k}")
    # the two-pass contract: ceil(k * 4) PQ candidates re-scored with the fp32 rows
    two = a.search_batch(q, 10, 0, 4.0)
    ci, cs, cc = oracle.pq_flat_search(cb, codes, dim, m, ks, q, metric, oracle.candidate_k(10, 4.0), global_centroid=gc)
    _same(two, *oracle.rescore_candidates(db, q, metric, ci, cc, 10), f"pq two-pass m={metric}", exact=False)
    a.close()


def test_pq_quantized_bin_opens_the_same_index(oracle):
    db, q, gc, cb, codes = _pq(oracle, 8000, 128, 16, 256, True, False)
    blob = F.quantized_bin_pq(codes, cb, 128, 16, 256, global_centroid=gc)
    got = vx.QuantizedFlatScanAdapter()
    got.load_quantized_bin(blob, vx.SimilarityFunction.COSINE)
    assert got.kind == "PQ" and got.size() == 8000
    ref = vx.QuantizedFlatScanAdapter()
    ref.build_pq(codes, cb, 16, 256, vx.SimilarityFunction.COSINE, global_centroid=gc)
    a, b = got.scan_candidates(q, 20), ref.scan_candidates(q, 20)
    for i, (u, v) in enumerate(zip(a, b)):
        assert np.array_equal(u.ordinals, v.ordinals) and np.array_equal(u.scores, v.scores), i
    got.close()
    ref.close()


def test_pq_k_larger_than_index_and_empty(oracle):
    db, q, gc, cb, codes = _pq(oracle, 40, 32, 4, 16, False, False)
    a = vx.QuantizedFlatScanAdapter()
    a.build_pq(codes, cb, 4, 16, vx.SimilarityFunction.EUCLIDEAN)
    _same(a.scan_candidates(q, 100), *oracle.pq_flat_search(cb, codes, 32, 4, 16, q, 0, 100), "pq k > n")
    a.close()
    e = vx.QuantizedFlatScanAdapter()
    e.build_pq(np.zeros((0, 4), np.uint8), cb, 4, 16, vx.SimilarityFunction.EUCLIDEAN)
    assert [len(o.ordinals) for o in e.scan_candidates(q[:3], 5)] == [0, 0, 0]
    e.close()
