"""Persistent files on the GPU: an index opened from quantized.bin or an IVF_PQ graph.bin (in the
layout the reference's encoders write, oracle/formats.py) gives the same results, to the bit, as
the index built from the arrays -- and IVF-PQ the oracle's.  The fp32 rows for the two-pass
rescore come in as a vectors.bin-style view (rows padded to 64 bytes)."""
import numpy as np
import pytest

import vectors_b200 as vx
from oracle import formats as F

pytestmark = pytest.mark.gpu

SEED_C, SEED_DB, SEED_Q = 0xC0FFEE03, 0xC0FFEE01, 0xC0FFEE02


def _vectors_bin_view(db):
    """db rows as they sit in a mapped vectors.bin: stride alignUp(dim * 4, 64) bytes."""
    n, dim = db.shape
    stride = ((dim * 4 + 63) // 64 * 64) // 4
    buf = np.zeros((n, stride), np.float32)
    buf[:, :dim] = db
    return buf[:, :dim]


def _same(a, b, tag):
    assert len(a) == len(b)
    for i, (x, y) in enumerate(zip(a, b)):
        assert np.array_equal(x.ordinals, y.ordinals), f"{tag}: query {i} ids"
        assert np.array_equal(x.scores, y.scores), f"{tag}: query {i} scores"


@pytest.mark.parametrize("metric", [0, 1, 3])
def test_quantized_bin_opens_the_same_index(oracle, metric):
    dim = 100  # rows padded to 112 floats in vectors.bin
    db = oracle.gen_mixture(6000, dim, 16, 0.3, SEED_C, SEED_DB, True)
    q = oracle.gen_mixture(40, dim, 16, 0.3, SEED_C, SEED_Q, True)
    view = _vectors_bin_view(db)
    lo, hi = oracle.sq8_train(db)
    codes, corr = oracle.sq8_encode_all(lo, hi, db)
    packed4, corr4 = oracle.sq4_encode_all(lo, hi, db)
    words = oracle.bq_encode_all(db)
    cent = db.mean(0).astype(np.float32)
    bwords, bcorr = oracle.bbq_encode_all(db, cent)
    f16 = oracle.fp16_encode_all(db)
    cases = [
        ("SQ8", lambda a: a.build_sq8(codes, corr, lo, hi, vx.SimilarityFunction(metric), vectors=db),
         F.quantized_bin_sq8(codes, corr, lo, hi)),
        ("SQ4", lambda a: a.build_sq4(packed4, corr4, dim, lo, hi, vx.SimilarityFunction(metric), vectors=db),
         F.quantized_bin_sq4(packed4, corr4, dim, lo, hi)),
        ("BQ", lambda a: a.build_bq(words, dim, vx.SimilarityFunction(metric), vectors=db), F.quantized_bin_bq(words, dim)),
        ("BBQ", lambda a: a.build_bbq(bwords, bcorr, cent, dim, vx.SimilarityFunction(metric), vectors=db),
         F.quantized_bin_bq(bwords, dim, cent, bcorr)),
        ("FP16", lambda a: a.build_fp16(f16, vx.SimilarityFunction(metric), vectors=db), F.quantized_bin_fp16(f16)),
    ]
    for kind, build, blob in cases:
        ref = vx.QuantizedFlatScanAdapter()
        build(ref)
        got = vx.QuantizedFlatScanAdapter()
        got.load_quantized_bin(blob, vx.SimilarityFunction(metric), vectors=view)
        assert got.kind == kind and got.size() == 6000
        _same(got.scan_candidates(q, 50), ref.scan_candidates(q, 50), f"{kind} candidates m={metric}")
        _same(got.search_batch(q, 10, over_query_factor=4.0), ref.search_batch(q, 10, over_query_factor=4.0),
              f"{kind} two-pass m={metric}")
        ref.close()
        got.close()


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_ivf_graph_bin_opens_the_same_index(oracle, metric):
    db = oracle.gen_mixture(20000, 128, 32, 0.3, SEED_C, SEED_DB, False)
    q = oracle.gen_mixture(60, 128, 32, 0.3, SEED_C, SEED_Q, False)
    cent = oracle.kmeans_train(db[:5000], 24, 10, 42)
    assign = oracle.kmeans_assign(db, cent)
    off, ords = oracle.build_ivf_lists(assign, 24)
    resid = db - cent[assign]
    cb = oracle.pq_train(resid, 16, 256)
    codes = oracle.pq_encode_all(resid, 16, 256, cb)
    blob = F.ivf_graph_bin(cent, off, ords, metric, pq=dict(m=16, ks=256, codebooks=cb, codes=codes))
    got = vx.IvfPqAdapter(nprobe=6)
    got.load_graph_bin(blob, vectors=_vectors_bin_view(db))  # metric taken from the file
    assert got.metric == vx.SimilarityFunction(metric) and got.size() == 20000
    ids, sc, cnt = oracle.ivfpq_search(cent, off, ords, 16, 256, cb, codes, q, metric, 10, 6)
    res = got.ivf_search(q, 10, 6)
    for i, o in enumerate(res):
        assert list(o.ordinals) == list(ids[i, : cnt[i]]), f"ivf graph.bin m={metric} query {i}"
        assert np.array_equal(o.scores, sc[i, : cnt[i]]), f"ivf graph.bin m={metric} query {i} scores"
    ref = vx.IvfPqAdapter(nprobe=6)
    ref.build_prebuilt(cent, off, ords, cb, codes, 16, 256, vx.SimilarityFunction(metric), vectors=db)
    _same(got.ivf_search(q, 10, 6, rescore_factor=3), ref.ivf_search(q, 10, 6, rescore_factor=3),
          f"ivf graph.bin rescore m={metric}")
    with pytest.raises(vx.UnsupportedOperationException, match="routes by"):
        vx.IvfPqAdapter().load_graph_bin(blob, metric=(metric + 1) % 3)
    got.close()
    ref.close()


@pytest.mark.parametrize("metric", [0, 2])
def test_ivf_flat_graph_bin_opens_the_same_index(oracle, metric):
    dim = 100
    db = oracle.gen_mixture(8000, dim, 16, 0.3, SEED_C, SEED_DB, metric == 2)
    q = oracle.gen_mixture(50, dim, 16, 0.3, SEED_C, SEED_Q, metric == 2)
    cent = oracle.kmeans_train(db[:3000], 20, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), 20)
    # the buoy's radii as BuoyIndex.computeRadii leaves them (the EUCLIDEAN early exit reads them)
    radii = oracle.ivf_radii(cent, off, ords, db)
    blob = F.ivf_graph_bin(cent, off, ords, metric, pq=None, key_dims=[[1, 2]] + [None] * 19, radii=radii)
    got = vx.IvfFlatAdapter(nprobe=5)
    got.load_graph_bin(blob, vectors=_vectors_bin_view(db))
    assert got.size() == 8000
    ref = vx.IvfFlatAdapter(nprobe=5)
    ref.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction(metric))
    ref.set_key_dims([[1, 2]] + [None] * 19)
    _same(got.ivf_search(q, 10, 5), ref.ivf_search(q, 10, 5), f"ivf-flat graph.bin m={metric}")
    # list 0 carries HARMONY key dimensions: the file's index scans it with squareDistance once
    # a query's heap is full, the array-built one (no key dimensions) does not
    ids, sc, cnt = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, metric, 10, 5,
                                              key_dims=[[1, 2]] + [None] * 19)
    for i, o in enumerate(got.search_batch(q, 10)):
        assert list(o.ordinals) == list(ids[i, : cnt[i]]), f"ivf-flat graph.bin m={metric} query {i}"
    got.close()
    ref.close()
