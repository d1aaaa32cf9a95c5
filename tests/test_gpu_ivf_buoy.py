"""GPU parity for the parts of IvfIndex.search that depend on the BuoyIndex state:

* the EUCLIDEAN early exit of the IVF-flat search (IvfIndex.java:190-205): clusters visited in
  route order, and the walk ends at the first cluster whose bound
  (max(0, (float) sqrt(centroid distance) - radius))^2 reaches the heap's worst distance --
  including the worked 2-D case where the break loses the nearest row, and clusters of mixed
  spreads where it changes most results;
* SOAR spill routing at search time (gamma > 0, CentroidIndex.routeWithSpillDistances,
  CentroidIndex.java:155-187) for IVF-PQ (both ADC kernels) and IVF-flat;
* the radii and spill targets a prebuilt BuoyIndex carries (vx_ivf_set_buoy) and a graph.bin
  stores (BuoyIndex.decode).

Against the oracle's restatement of the same Java code (oracle.ivfflat_search_full,
oracle.ivfpq_search_spill): bit-exact ordinals and scores, within 1e-4 for fp32 re-scores.
"""
import numpy as np
import pytest

import vectors_b200 as vx
from oracle import formats as F

pytestmark = pytest.mark.gpu

SEED_C, SEED_DB, SEED_Q = 0xC0FFEE03, 0xC0FFEE01, 0xC0FFEE02


def _same(got, ids, sc, cnt, tag, exact=True):
    for i, o in enumerate(got):
        c = cnt[i]
        assert list(o.ordinals) == list(ids[i, :c]), f"{tag}: query {i} ids {list(o.ordinals)[:6]} vs {list(ids[i, :6])}"
        if exact:
            assert np.array_equal(o.scores, sc[i, :c]), f"{tag}: query {i} scores"
        else:
            np.testing.assert_allclose(o.scores, sc[i, :c], rtol=1e-4, atol=0, err_msg=f"{tag}: query {i}")


def _spill_targets(nlist):
    # a far cluster per cluster (so the spill addition is rarely a primary already), some none
    spill = ((np.arange(nlist) * 7 + nlist // 2 + 1) % nlist).astype(np.int32)
    spill[::5] = -1
    return spill


# ------------------------------------------------------------------ early exit
def test_early_exit_two_dims_loses_the_nearest_row(oracle):
    # route order for q = 0: cluster 0 (d^2 4), 1 (6.25), 2 (9); with k = 1 the heap holds d^2 4
    # after cluster 0 and cluster 1's bound 2.5^2 >= 4 ends the walk, so the row at d^2 1.21 in
    # the wider cluster 2 is never seen -- the reference returns row 0, and so must the GPU
    cent = np.array([[2, 0], [-2.5, 0], [0, 3]], np.float32)
    db = np.array([[2, 0], [-2.5, 0], [0, 3], [0, 1.1]], np.float32)
    off = np.array([0, 1, 2, 4], np.int64)
    ords = np.array([0, 1, 2, 3], np.int32)
    q = np.zeros((1, 2), np.float32)
    a = vx.IvfFlatAdapter(nprobe=3)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction.EUCLIDEAN)
    got = a.ivf_search(q, 1, 3)
    assert list(got[0].ordinals) == [0] and got[0].scores[0] == np.float32(-4.0)
    radii = oracle.ivf_radii(cent, off, ords, db)
    _same(got, *oracle.ivfflat_search_full(cent, off, ords, db, radii, q, oracle.EUCLIDEAN, 1, 3), "2-D")
    # k = 2: the heap is not full after cluster 0, so cluster 1 is scanned; then the bound of
    # cluster 2 ((3 - 1.9)^2 = 1.21) is below the worst (6.25) and the closer row is found
    got = a.ivf_search(q, 2, 3)
    assert list(got[0].ordinals) == [3, 0]
    a.close()


def test_early_exit_changes_most_results_on_mixed_spreads(oracle):
    # 2-D clusters of very different spreads, rows kept in the cluster that generated them:
    # wide clusters late in route order hold rows the break skips
    rng = np.random.default_rng(0)
    cent = (10.0 * rng.standard_normal((8, 2))).astype(np.float32)
    sig = np.array([0.2, 0.2, 0.3, 0.3, 0.5, 4.0, 6.0, 8.0], np.float32)
    assign = rng.integers(0, 8, 2000)
    db = (cent[assign] + sig[assign, None] * rng.standard_normal((2000, 2))).astype(np.float32)
    off, ords = oracle.build_ivf_lists(assign.astype(np.int32), 8)
    q = (10.0 * rng.standard_normal((60, 2))).astype(np.float32)
    a = vx.IvfFlatAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction.EUCLIDEAN)
    got = a.ivf_search(q, 5, 8)
    radii = oracle.ivf_radii(cent, off, ords, db)
    want = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, oracle.EUCLIDEAN, 5, 8)
    every = oracle.ivfflat_search(cent, off, ords, db, q, oracle.EUCLIDEAN, 5, 8)
    assert sum(not np.array_equal(every[0][j], want[0][j]) for j in range(len(q))) > len(q) // 4
    _same(got, *want, "mixed spreads")
    a.close()


@pytest.mark.parametrize("scale", [0.0, 0.5, 1.5])
def test_early_exit_with_a_buoys_own_radii(oracle, scale):
    # radii handed over from a prebuilt BuoyIndex (vx_ivf_set_buoy) replace the computed ones:
    # smaller radii end the walk sooner, larger ones later; min_score is applied before the heap
    n, dim, nlist = 9000, 64, 16
    db = oracle.gen_mixture(n, dim, 12, 0.3, SEED_C, SEED_DB, False)
    q = oracle.gen_mixture(200, dim, 12, 0.3, SEED_C, SEED_Q, False)
    cent = oracle.kmeans_train(db[:3000], nlist, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), nlist)
    radii = (oracle.ivf_radii(cent, off, ords, db) * np.float32(scale)).astype(np.float32)
    a = vx.IvfFlatAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction.EUCLIDEAN)
    a.set_buoy(radii=radii)
    for k in (1, 10, 40):
        got = a.ivf_search(q, k, 8)
        _same(got, *oracle.ivfflat_search_full(cent, off, ords, db, radii, q, oracle.EUCLIDEAN, k, 8),
              f"radii x{scale} k={k}")
    a.close()


# ------------------------------------------------------------------ SOAR spill
def _ivfpq(oracle, dim, m, nlist=32, n=20000):
    db = oracle.gen_mixture(n, dim, 32, 0.3, SEED_C, SEED_DB, False)
    q = oracle.gen_mixture(64, dim, 32, 0.3, SEED_C, SEED_Q, False)
    cent = oracle.kmeans_train(db[:5000], nlist, 10, 42)
    assign = oracle.kmeans_assign(db, cent)
    off, ords = oracle.build_ivf_lists(assign, nlist)
    resid = db - cent[assign]
    cb = oracle.pq_train(resid, m, 256)
    codes = oracle.pq_encode_all(resid, m, 256, cb)
    return db, q, cent, off, ords, cb, codes


@pytest.mark.parametrize("metric", [0, 1, 2, 3])
@pytest.mark.parametrize("dim,m", [(128, 16), (96, 8)])
def test_ivfpq_spill_routing(oracle, metric, dim, m):
    # (128, 16): grouped ADC kernel; (96, 8): general ADC kernel (12-dim subspaces)
    db, q, cent, off, ords, cb, codes = _ivfpq(oracle, dim, m)
    spill = _spill_targets(len(cent))
    gamma = 0.6 if metric == 0 else 0.3
    a = vx.IvfPqAdapter(nprobe=4, gamma=gamma)
    a.build_prebuilt(cent, off, ords, cb, codes, m, 256, vx.SimilarityFunction(metric), vectors=db)
    a.set_buoy(spill_targets=spill)
    routes = oracle.route_spill(cent, q, metric, 4, gamma, spill)
    assert sum(len(r[0]) > 4 for r in routes) > len(q) // 4, "the case must exercise spill targets"
    got = a.ivf_search(q, 10, 4)
    _same(got, *oracle.ivfpq_search_spill(cent, off, ords, m, 256, cb, codes, q, metric, 10, 4, gamma, spill),
          f"ivfpq spill m={metric}")
    got = a.ivf_search(q, 10, 4, rescore_factor=4)
    _same(got, *oracle.ivfpq_search_spill(cent, off, ords, m, 256, cb, codes, q, metric, 10, 4, gamma, spill, 4, db),
          f"ivfpq spill rescore m={metric}", exact=False)
    # searchBatch follows the adapter's gamma as well
    _same(a.search_batch(q, 10), *oracle.ivfpq_search_spill(cent, off, ords, m, 256, cb, codes, q, metric, 10, 4,
                                                             gamma, spill), f"ivfpq spill searchBatch m={metric}")
    a.close()


@pytest.mark.parametrize("metric", [0, 1, 2, 3])
def test_ivfflat_spill_routing_with_early_exit(oracle, metric):
    n, dim, nlist = 9000, 96, 16
    db = oracle.gen_mixture(n, dim, 12, 0.3, SEED_C, SEED_DB, metric == 2)
    q = oracle.gen_mixture(120, dim, 12, 0.3, SEED_C, SEED_Q, metric == 2)
    cent = oracle.kmeans_train(db[:3000], nlist, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), nlist)
    spill = _spill_targets(len(cent))
    gamma = 0.6 if metric == 0 else 0.3
    a = vx.IvfFlatAdapter(nprobe=4, gamma=gamma)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction(metric))
    a.set_buoy(spill_targets=spill)
    radii = oracle.ivf_radii(cent, off, ords, db)
    for k in (5, 20):
        got = a.ivf_search(q, k, 4)
        want = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, metric, k, 4, gamma, spill)
        if metric == 2:
            _same(got, want[0], want[1], want[2], f"ivfflat spill m={metric} k={k}", exact=False)
        else:
            _same(got, *want, f"ivfflat spill m={metric} k={k}")
    a.close()


def test_graph_bin_carries_radii_and_spill_targets(oracle):
    # a graph.bin's buoy holds the spill targets and radii (BuoyIndex.encode); the index opened
    # from it searches with them, as IvfIndex.decode's index does
    n, dim, nlist = 9000, 96, 16
    db = oracle.gen_mixture(n, dim, 12, 0.3, SEED_C, SEED_DB, False)
    q = oracle.gen_mixture(80, dim, 12, 0.3, SEED_C, SEED_Q, False)
    cent = oracle.kmeans_train(db[:3000], nlist, 8, 42)
    assign = oracle.kmeans_assign(db, cent)
    off, ords = oracle.build_ivf_lists(assign, nlist)
    spill = _spill_targets(len(cent))
    radii = (oracle.ivf_radii(cent, off, ords, db) * np.float32(0.7)).astype(np.float32)
    blob = F.ivf_graph_bin(cent, off, ords, 0, pq=None, radii=radii, spill=spill)
    a = vx.IvfFlatAdapter(nprobe=4, gamma=0.6)
    a.load_graph_bin(blob, vectors=db)
    got = a.ivf_search(q, 10, 4)
    _same(got, *oracle.ivfflat_search_full(cent, off, ords, db, radii, q, 0, 10, 4, 0.6, spill), "graph.bin flat")
    a.close()
    resid = db - cent[assign]
    cb = oracle.pq_train(resid, 12, 256)
    codes = oracle.pq_encode_all(resid, 12, 256, cb)
    blob = F.ivf_graph_bin(cent, off, ords, 0, pq=dict(m=12, ks=256, codebooks=cb, codes=codes), radii=radii,
                           spill=spill)
    p = vx.IvfPqAdapter(nprobe=4, gamma=0.6)
    p.load_graph_bin(blob)
    got = p.ivf_search(q, 10, 4)
    _same(got, *oracle.ivfpq_search_spill(cent, off, ords, 12, 256, cb, codes, q, 0, 10, 4, 0.6, spill),
          "graph.bin pq spill")
    p.close()


def test_negative_gamma_is_rejected():
    with pytest.raises(vx.IllegalArgumentException, match="gamma"):
        vx.IvfPqAdapter(nprobe=4, gamma=-0.1)


@pytest.mark.parametrize("metric", [0, 1])
def test_ivfflat_large_k_with_early_exit(oracle, metric):
    # k up to 256 per (query, list) on the list scan's widest candidate buffers
    n, dim, nlist = 12000, 64, 16
    db = oracle.gen_mixture(n, dim, 12, 0.3, SEED_C, SEED_DB, False)
    q = oracle.gen_mixture(100, dim, 12, 0.3, SEED_C, SEED_Q, False)
    cent = oracle.kmeans_train(db[:3000], nlist, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), nlist)
    radii = (oracle.ivf_radii(cent, off, ords, db) * np.float32(0.6)).astype(np.float32)
    a = vx.IvfFlatAdapter(nprobe=6)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction(metric))
    a.set_buoy(radii=radii)
    for k in (150, 256):
        _same(a.ivf_search(q, k, 6), *oracle.ivfflat_search_full(cent, off, ords, db, radii, q, metric, k, 6),
              f"ivfflat k={k} m={metric}")
    with pytest.raises(vx.UnsupportedOperationException):
        a.ivf_search(q, 257, 6)
    a.close()


@pytest.mark.parametrize("k", [8, 40])
def test_harmony_partitions_scanned_with_square_distance(oracle, k):
    # partitions with key dimensions (IvfIndex.build's harmonyKeyDims): once a query's heap is
    # full, the reference scores their rows with squareDistance instead of the batched order
    n, dim, nlist = 9000, 100, 16
    db = oracle.gen_mixture(n, dim, 12, 0.3, SEED_C, SEED_DB, False)
    q = oracle.gen_mixture(120, dim, 12, 0.3, SEED_C, SEED_Q, False)
    cent = oracle.kmeans_train(db[:3000], nlist, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), nlist)
    rng = np.random.default_rng(11)
    key_dims = [list(rng.choice(dim, 6, replace=False)) if l % 3 != 1 else None for l in range(nlist)]
    radii = oracle.ivf_radii(cent, off, ords, db)
    a = vx.IvfFlatAdapter(nprobe=6)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction.EUCLIDEAN)
    a.set_key_dims(key_dims)
    got = a.ivf_search(q, k, 6)
    want = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, 0, k, 6, key_dims=key_dims)
    plain = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, 0, k, 6)
    assert sum(not np.array_equal(want[1][j], plain[1][j]) for j in range(len(q))) > 0
    _same(got, *want, f"harmony k={k}")
    a.set_key_dims(None)  # cleared: the batched scan everywhere again
    _same(a.ivf_search(q, k, 6), *plain, f"harmony cleared k={k}")
    a.close()


@pytest.mark.parametrize("world", [1, 2, 3])
def test_ivfflat_pair_split_equals_unsplit_with_early_exit(oracle, world):
    # vectors_b200.sharded.ivfflat_search_pair_split, the ranks emulated on one GPU: each rank
    # scans its share of every list's pairs into per-slot results, the slots are added up and
    # merged in route order with the early exit -- on clusters where the break changes most
    # results, the same ordinals and scores as the unsplit search and the oracle
    import torch

    from vectors_b200.sharded import deal_pairs

    rng = np.random.default_rng(1)
    cent = (10.0 * rng.standard_normal((16, 3))).astype(np.float32)
    sig = np.array([0.2, 0.3, 0.5, 4.0, 6.0, 8.0, 0.4, 2.0] * 2, np.float32)
    assign = rng.integers(0, 16, 6000)
    db = (cent[assign] + sig[assign, None] * rng.standard_normal((6000, 3))).astype(np.float32)
    off, ords = oracle.build_ivf_lists(assign.astype(np.int32), 16)
    q = (10.0 * rng.standard_normal((700, 3))).astype(np.float32)
    a = vx.IvfFlatAdapter(nprobe=8)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction.EUCLIDEAN)
    qd = torch.from_numpy(q).cuda()
    ref = a.ivf_search_device(qd, 5, 8)
    lists, dist = a.route_dist_device(qd, 8)
    assert torch.equal(lists, a.route_device(qd, 8))
    keys = cnt = None
    for r in range(world):
        kr, cr = a.scan_pairs_device(qd, 5, 8, deal_pairs(lists, r, world, 64))
        keys = kr if keys is None else keys + kr
        cnt = cr if cnt is None else cnt + cr
    mi, ms, mc = a.merge_pairs_device(5, 8, lists, dist, keys, cnt)
    torch.cuda.synchronize()
    assert torch.equal(mi, ref[0]) and torch.equal(ms, ref[1]) and torch.equal(mc, ref[2])
    radii = oracle.ivf_radii(cent, off, ords, db)
    ids, sc, n = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, oracle.EUCLIDEAN, 5, 8)
    every = oracle.ivfflat_search(cent, off, ords, db, q, oracle.EUCLIDEAN, 5, 8)
    assert sum(not np.array_equal(every[0][j], ids[j]) for j in range(len(q))) > len(q) // 10  # the break fires
    assert np.array_equal(mc.cpu().numpy(), n)
    for i in range(len(q)):
        assert list(mi[i, : n[i]].cpu().numpy()) == list(ids[i, : n[i]]), f"query {i}"
        assert np.array_equal(ms[i, : n[i]].cpu().numpy(), sc[i, : n[i]]), f"query {i} scores"
    a.close()


def test_ivfflat_pair_split_refuses_harmony_partitions(oracle):
    import torch

    rng = np.random.default_rng(2)
    db = rng.standard_normal((500, 8)).astype(np.float32)
    cent = db[:4].copy()
    assign = np.argmin(((db[:, None, :] - cent[None]) ** 2).sum(2), 1).astype(np.int32)
    off, ords = oracle.build_ivf_lists(assign, 4)
    a = vx.IvfFlatAdapter(nprobe=4)
    a.build_prebuilt(cent, off, ords, db, vx.SimilarityFunction.EUCLIDEAN)
    a.set_key_dims([2, None, None, 3])
    qd = torch.from_numpy(db[:10]).cuda()
    lists, _ = a.route_dist_device(qd, 4)
    with pytest.raises(vx.UnsupportedOperationException):
        a.scan_pairs_device(qd, 5, 4, lists)
    a.close()
