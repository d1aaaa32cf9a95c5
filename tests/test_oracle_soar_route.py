"""SOAR spill routing (CentroidIndex.routeWithSpillDistances with gamma > 0,
vectors-core/.../cluster/CentroidIndex.java:89-187, spillBoundary :213-220), restated by the
oracle for IVF collections configured with a spill ratio.  CPU only; worked by hand."""
import numpy as np

CENT = np.array([[0.0], [1.0], [2.5], [10.0]], np.float32)
SPILL = np.array([2, 3, 1, 0], np.int32)


def test_gamma_zero_is_plain_routing(oracle):
    q = np.array([[0.4]], np.float32)
    (ids, d), = oracle.route_spill(CENT, q, oracle.EUCLIDEAN, 2, 0.0, SPILL)
    r_ids, r_d = oracle.route(CENT, q, oracle.EUCLIDEAN, 2)
    assert list(ids) == list(r_ids[0]) == [0, 1] and np.array_equal(d, r_d[0])


def test_euclidean_boundary_is_nearest_times_one_plus_gamma(oracle):
    # squared distances from 0.4: 0.16, 0.36, 4.41, 92.16; primaries 0, 1
    q = np.array([[0.4]], np.float32)
    # gamma 0.5: boundary 0.24 admits primary 0 only -> its spill target 2, at its own distance
    (ids, d), = oracle.route_spill(CENT, q, oracle.EUCLIDEAN, 2, 0.5, SPILL)
    assert list(ids) == [0, 1, 2] and d[2] == np.float32(np.float32(2.1) * np.float32(2.1))
    # gamma 3: boundary 0.64 admits both -> targets 2 and 3 in primary order
    (ids, _), = oracle.route_spill(CENT, q, oracle.EUCLIDEAN, 2, 3.0, SPILL)
    assert list(ids) == [0, 1, 2, 3]


def test_targets_already_routed_or_invalid_are_skipped(oracle):
    q = np.array([[0.4]], np.float32)
    # primary 0 spills to 1 (already a primary), primary 1 to -1 (none)
    (ids, _), = oracle.route_spill(CENT, q, oracle.EUCLIDEAN, 2, 3.0, np.array([1, -1, 0, 0], np.int32))
    assert list(ids) == [0, 1]


def test_dot_boundary_scales_the_best_score(oracle):
    # DOT_PRODUCT: distances are negated dots, q = 1 -> -0, -1, -2.5, -10; primaries 3, 2.
    # nearest score 10; gamma 0.3 -> threshold 10 - 3 = 7: primary 3 (10) admits its spill
    # target 0, primary 2 (2.5) is below the threshold and stops the walk
    q = np.array([[1.0]], np.float32)
    (ids, d), = oracle.route_spill(CENT, q, oracle.DOT_PRODUCT, 2, 0.3, SPILL)
    assert list(ids) == [3, 2, 0] and d[2] == np.float32(-0.0)
    (ids, _), = oracle.route_spill(CENT, q, oracle.DOT_PRODUCT, 2, 0.8, SPILL)
    assert list(ids) == [3, 2, 0, 1]


def _lists(oracle, n=3000, dim=16, nlist=12, seed=3):
    rng = np.random.default_rng(seed)
    cent = (3.0 * rng.standard_normal((nlist, dim))).astype(np.float32)
    assign = rng.integers(0, nlist, n).astype(np.int32)
    db = (cent[assign] + rng.standard_normal((n, dim))).astype(np.float32)
    off, ords = oracle.build_ivf_lists(assign, nlist)
    q = (3.0 * rng.standard_normal((25, dim))).astype(np.float32)
    spill = np.roll(np.arange(nlist, dtype=np.int32), 5)
    spill[::4] = -1
    return cent, off, ords, db, q, spill


def _canonical(pairs, k):
    pairs = sorted(pairs, key=lambda t: (-t[0], t[1]))[:k]
    return [i for _, i in pairs], [s for s, _ in pairs]


def test_ivfpq_spill_search_scans_the_spill_routed_lists(oracle):
    # IvfIndex.pqSearch over routeWithSpillDistances' clusters: every listed cluster's rows scored
    # with its ADC table (sequential fp32 sum), canonical top-k -- composed here from the route and
    # the table builder, one list at a time
    cent, off, ords, db, q, spill = _lists(oracle)
    m, ks = 4, 16
    assign = np.zeros(len(db), np.int32)
    for l in range(len(cent)):
        assign[ords[off[l]:off[l + 1]]] = l
    resid = db - cent[assign]
    cb = oracle.pq_train(resid, m, ks)
    codes = oracle.pq_encode_all(resid, m, ks, cb)
    for metric in (oracle.EUCLIDEAN, oracle.DOT_PRODUCT):
        got = oracle.ivfpq_search_spill(cent, off, ords, m, ks, cb, codes, q, metric, 10, 3, 0.6, spill)
        plain = oracle.ivfpq_search(cent, off, ords, m, ks, cb, codes, q, metric, 10, 3)
        zero = oracle.ivfpq_search_spill(cent, off, ords, m, ks, cb, codes, q, metric, 10, 3, 0.0, spill)
        assert all(np.array_equal(a, b) for a, b in zip(plain, zero))
        routes = oracle.route_spill(cent, q, metric, 3, 0.6, spill)
        assert any(len(r[0]) > 3 for r in routes)
        for j, (lids, _) in enumerate(routes):
            pairs = []
            for cid in lids:
                if metric == oracle.EUCLIDEAN:
                    t = oracle.pq_adc_table(q[j] - cent[cid], m, ks, cb)
                    base = np.float32(0)
                else:
                    t = oracle.pq_adc_table(q[j], m, ks, cb, use_dot=True)
                    base = np.float32(oracle.dot(q[j], cent[cid]))
                for o in ords[off[cid]:off[cid + 1]]:
                    s = np.float32(0)
                    for sub in range(m):
                        s = np.float32(s + t[sub, codes[o, sub]])
                    pairs.append((np.float32(-s) if metric == oracle.EUCLIDEAN else np.float32(base + s), int(o)))
            ids, sc = _canonical(pairs, 10)
            assert list(got[0][j, :got[2][j]]) == ids, (metric, j)
            assert list(got[1][j, :got[2][j]]) == sc, (metric, j)


def test_ivfflat_full_search_merges_spill_lists_with_the_early_exit(oracle):
    # IvfIndex.search without PQ: the spill-routed clusters in route order, each scored alone in
    # the batched order, merged into the heap with the EUCLIDEAN bound checked before each cluster
    cent, off, ords, db, q, spill = _lists(oracle)
    radii = oracle.ivf_radii(cent, off, ords, db)
    for metric in (oracle.EUCLIDEAN, oracle.DOT_PRODUCT):
        k = 8
        got = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, metric, k, 3, 0.6, spill)
        routes = oracle.route_spill(cent, q, metric, 3, 0.6, spill)
        for j, (lids, dists) in enumerate(routes):
            kept = []
            for cid, dd in zip(lids, dists):
                if metric == oracle.EUCLIDEAN and len(kept) == k:
                    lb = np.float32(np.float32(np.sqrt(np.float64(dd))) - radii[cid])
                    if lb > 0 and np.float32(lb * lb) >= -kept[-1][0]:
                        break
                b, e = int(off[cid]), int(off[cid + 1])
                if e == b:
                    continue
                one = np.array([0, e - b], np.int64)
                ids, sc, cnt = oracle.ivfflat_search(cent[cid:cid + 1], one, ords[b:e], db, q[j:j + 1], metric, k, 1)
                kept = sorted(kept + [(sc[0, i], int(ids[0, i])) for i in range(cnt[0])], key=lambda t: (-t[0], t[1]))[:k]
            assert list(got[0][j, :got[2][j]]) == [i for _, i in kept], (metric, j)
            assert list(got[1][j, :got[2][j]]) == [s for s, _ in kept], (metric, j)
