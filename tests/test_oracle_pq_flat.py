"""The oracle's PQ flat scan (PQVectors.scoreFunctionFor, PQVectors.java:104-191) checked on the CPU.

The reference's PQ tests hold no known-answer scores, only properties (ProductQuantizerTest:
selfScore_isHighForNormalizedVectors, cosineScoring_withGlobalCentroid_usesConsistentNorm), so
the oracle is pinned by those properties and by a second restatement written here in numpy
float32, one Java operation at a time: the ADC table entries come from the oracle's pinned
dotProduct / squareDistance, everything after them (the sequential sum over subspaces, the
centroid norms, the metric transforms, the canonical top-k) is restated independently.
"""
import numpy as np
import pytest

f32 = np.float32


def _pq(oracle, n=600, dim=32, m=4, ks=16, seed=3, offset=0.0, center=False):
    rng = np.random.default_rng(seed)
    data = rng.standard_normal((n, dim)).astype(f32)
    data /= np.linalg.norm(data, axis=1, keepdims=True)
    data += f32(offset)
    gc = data.mean(0).astype(f32) if center else None
    x = data - gc if center else data
    cb = oracle.pq_train(x, m, ks)
    codes = oracle.pq_encode_all(x, m, ks, cb)
    return data, gc, cb, codes


def _scores_numpy(oracle, cb, gc, codes, dim, m, ks, q, metric):
    sub = dim // m
    books = cb.reshape(m, ks, sub)
    qc = (q - gc).astype(f32) if gc is not None else q.astype(f32)
    table = np.empty((m, ks), f32)
    for s in range(m):
        for c in range(ks):
            a = qc[s * sub:(s + 1) * sub]
            table[s, c] = oracle.square_distance(a, books[s, c]) if metric == oracle.EUCLIDEAN else oracle.dot(a, books[s, c])
    n = codes.shape[0]
    acc = np.zeros(n, f32)
    for s in range(m):
        acc = (acc + table[s, codes[:, s]]).astype(f32)
    if metric == oracle.EUCLIDEAN:
        return (f32(1) / (f32(1) + acc)).astype(f32)
    if metric == oracle.MAXIMUM_INNER_PRODUCT:
        return np.array([oracle.lib().vo_scale_mip(float(v)) for v in acc], f32)
    if metric == oracle.COSINE:
        cn = np.zeros((m, ks), f32)
        for s in range(m):
            for d in range(sub):
                cn[s] = (cn[s] + (books[s, :, d] * books[s, :, d]).astype(f32)).astype(f32)
        vsq = np.zeros(n, f32)
        for s in range(m):
            vsq = (vsq + cn[s, codes[:, s]]).astype(f32)
        qsq = f32(0)
        for d in range(dim):
            qsq = f32(qsq + f32(qc[d] * qc[d]))
        qn = f32(np.sqrt(np.float64(qsq)))
        vn = np.sqrt(vsq.astype(np.float64)).astype(f32)
        with np.errstate(divide="ignore", invalid="ignore"):
            cosv = (acc / (qn * vn).astype(f32)).astype(f32)
        out = np.maximum(((f32(1) + cosv) / f32(2)).astype(f32), f32(0))
        out[(vn == 0) | (qn == 0)] = 0
        return out
    return np.maximum(((f32(1) + acc) / f32(2)).astype(f32), f32(0))


@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("center", [False, True])
def test_pq_flat_scores_match_a_second_restatement(oracle, metric, center):
    dim, m, ks, k = 32, 4, 16, 10
    data, gc, cb, codes = _pq(oracle, dim=dim, m=m, ks=ks, center=center)
    q = data[:5] + np.float32(0.01)
    ids, sc, cnt = oracle.pq_flat_search(cb, codes, dim, m, ks, q, metric, k, global_centroid=gc)
    for j in range(len(q)):
        s = _scores_numpy(oracle, cb, gc, codes, dim, m, ks, q[j], metric)
        order = sorted(range(len(s)), key=lambda i: (-s[i], i))[:k]
        assert list(ids[j, :cnt[j]]) == order, (metric, center, j)
        assert np.array_equal(sc[j, :cnt[j]], s[order]), (metric, center, j)


def test_pq_self_score_is_high_for_normalized_vectors(oracle):
    # ProductQuantizerTest.selfScore_isHighForNormalizedVectors: DOT_PRODUCT self score > 0.7
    data, gc, cb, codes = _pq(oracle, n=200, dim=128, m=16, ks=256, seed=42)
    ids, sc, cnt = oracle.pq_flat_search(cb, codes, 128, 16, 256, data[:1], oracle.DOT_PRODUCT, 200)
    assert sc[0][list(ids[0]).index(0)] > 0.7


def test_pq_cosine_with_global_centroid_uses_the_centred_norm(oracle):
    # ProductQuantizerTest.cosineScoring_withGlobalCentroid_usesConsistentNorm: rows shifted by
    # +50, global centring on; the cosine self score uses |q - gc| and stays above 0.5
    data, gc, cb, codes = _pq(oracle, n=100, dim=64, m=8, ks=64, seed=42, offset=50.0, center=True)
    ids, sc, cnt = oracle.pq_flat_search(cb, codes, 64, 8, 64, data[:1], oracle.COSINE, 100, global_centroid=gc)
    assert sc[0][list(ids[0]).index(0)] > 0.5
