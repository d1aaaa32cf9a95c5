"""IvfIndex.search's EUCLIDEAN early exit (IvfIndex.java:190-200) against per-cluster radii
(BuoyIndex.computeRadii, BuoyIndex.java:175-183), restated by the oracle.  The GPU scans every
probed list; these CPU tests pin (1) that the reference's break can skip a closer row held by a
later, wider cluster, and (2) that on the inputs of the IVF-flat GPU parity tests the break
changes no result, so parity with the scan-all oracle there is parity with the reference."""
import numpy as np
import pytest

SEED_C, SEED_DB, SEED_Q = 0xC0FFEE03, 0xC0FFEE01, 0xC0FFEE02


def test_radii_are_the_largest_member_distance(oracle):
    cent = np.array([[2, 0], [-2.5, 0], [0, 3]], np.float32)
    rows = np.array([[2, 0], [-2.5, 0], [0, 3], [0, 1.1]], np.float32)
    off = np.array([0, 1, 2, 4], np.int64)
    ords = np.array([0, 1, 2, 3], np.int32)
    assert oracle.ivf_radii(cent, off, ords, rows).tolist() == [0.0, 0.0, np.float32(1.9)]


def test_break_skips_a_closer_row_in_a_wider_later_cluster(oracle):
    # route order for q = 0: cluster 0 (d^2 4), 1 (6.25), 2 (9).  After cluster 0 the heap (k = 1)
    # holds d^2 = 4; cluster 1's bound 2.5^2 >= 4 ends the scan, so cluster 2's row at d^2 1.21
    # (bound (3 - 1.9)^2 = 1.21 < 4) is never seen
    cent = np.array([[2, 0], [-2.5, 0], [0, 3]], np.float32)
    rows = np.array([[2, 0], [-2.5, 0], [0, 3], [0, 1.1]], np.float32)
    off = np.array([0, 1, 2, 4], np.int64)
    ords = np.array([0, 1, 2, 3], np.int32)
    q = np.zeros((1, 2), np.float32)
    radii = oracle.ivf_radii(cent, off, ords, rows)
    ids, sc, _ = oracle.ivfflat_search_early_exit(cent, off, ords, rows, radii, q, oracle.EUCLIDEAN, 1, 3)
    assert ids[0, 0] == 0 and sc[0, 0] == -4.0
    ids, sc, _ = oracle.ivfflat_search(cent, off, ords, rows, q, oracle.EUCLIDEAN, 1, 3)
    assert ids[0, 0] == 3 and sc[0, 0] == np.float32(-1.21)


@pytest.mark.parametrize("dim,nq,k", [(128, 400, 10), (96, 50, 50), (100, 40, 10), (7, 30, 5)])
def test_break_changes_nothing_on_the_gpu_parity_inputs(oracle, dim, nq, k):
    # the inputs of test_ivfflat_matches_oracle (EUCLIDEAN): 9,000 rows, 16 lists, 8 probes
    n, nlist = 9000, 16
    db = oracle.gen_mixture(n, dim, 12, 0.3, SEED_C, SEED_DB, False)
    q = oracle.gen_mixture(nq, dim, 12, 0.3, SEED_C, SEED_Q, False)
    cent = oracle.kmeans_train(db[:3000], nlist, 8, 42)
    off, ords = oracle.build_ivf_lists(oracle.kmeans_assign(db, cent), nlist)
    radii = oracle.ivf_radii(cent, off, ords, db)
    a = oracle.ivfflat_search(cent, off, ords, db, q, oracle.EUCLIDEAN, k, 8)
    b = oracle.ivfflat_search_early_exit(cent, off, ords, db, radii, q, oracle.EUCLIDEAN, k, 8)
    for j in range(nq):
        assert list(a[0][j, : a[2][j]]) == list(b[0][j, : b[2][j]]), j
        assert np.array_equal(a[1][j, : a[2][j]], b[1][j, : b[2][j]]), j


def _ordered_merge(oracle, cent, off, ords, db, radii, q, k, nprobe):
    """The early exit from per-list results: each probed list's own top-k (scored alone, in the
    same batch order), merged in route order with the bound checked before each list -- the heap
    after i lists is the k best of those lists' top-k."""
    lids, dists = oracle.route(cent, q, oracle.EUCLIDEAN, nprobe)
    out = []
    for j in range(len(q)):
        kept = []  # (score, id)
        for p in range(nprobe):
            cid = int(lids[j, p])
            if len(kept) == k:
                worst = kept[-1][0]
                lb = np.float32(np.float32(np.sqrt(np.float64(dists[j, p]))) - radii[cid])
                if lb > 0 and np.float32(lb * lb) >= -worst:
                    break
            b, e = int(off[cid]), int(off[cid + 1])
            if e == b:
                continue
            one = np.array([0, e - b], np.int64)
            ids, sc, cnt = oracle.ivfflat_search(cent[cid:cid + 1], one, ords[b:e], db, q[j:j + 1],
                                                 oracle.EUCLIDEAN, k, 1)
            kept += [(sc[0, i], int(ids[0, i])) for i in range(cnt[0])]
            kept = sorted(kept, key=lambda t: (-t[0], t[1]))[:k]
        out.append(kept)
    return out


@pytest.mark.parametrize("case", ["two_dims", "wide_late_clusters"])
def test_ordered_merge_of_list_top_k_reproduces_the_break(oracle, case):
    if case == "two_dims":
        cent = np.array([[2, 0], [-2.5, 0], [0, 3]], np.float32)
        db = np.array([[2, 0], [-2.5, 0], [0, 3], [0, 1.1]], np.float32)
        off = np.array([0, 1, 2, 4], np.int64)
        ords = np.array([0, 1, 2, 3], np.int32)
        q = np.zeros((1, 2), np.float32)
        k, nprobe = 1, 3
    else:
        # 2-D clusters of very different spreads, rows kept in the cluster that generated them:
        # wide clusters late in route order hold rows the break skips (most queries change)
        rng = np.random.default_rng(0)
        cent = (10.0 * rng.standard_normal((8, 2))).astype(np.float32)
        sig = np.array([0.2, 0.2, 0.3, 0.3, 0.5, 4.0, 6.0, 8.0], np.float32)
        assign = rng.integers(0, 8, 2000)
        db = (cent[assign] + sig[assign, None] * rng.standard_normal((2000, 2))).astype(np.float32)
        off, ords = oracle.build_ivf_lists(assign.astype(np.int32), 8)
        q = (10.0 * rng.standard_normal((60, 2))).astype(np.float32)
        k, nprobe = 5, 8
    radii = oracle.ivf_radii(cent, off, ords, db)
    want = oracle.ivfflat_search_early_exit(cent, off, ords, db, radii, q, oracle.EUCLIDEAN, k, nprobe)
    if case == "wide_late_clusters":
        every = oracle.ivfflat_search(cent, off, ords, db, q, oracle.EUCLIDEAN, k, nprobe)
        assert sum(not np.array_equal(every[0][j], want[0][j]) for j in range(len(q))) > len(q) // 4
    got = _ordered_merge(oracle, cent, off, ords, db, radii, q, k, nprobe)
    for j in range(len(q)):
        assert [i for _, i in got[j]] == list(want[0][j, : want[2][j]]), j
        assert [s for s, _ in got[j]] == list(want[1][j, : want[2][j]]), j


def _harmony_model(oracle, cent, off, ords, db, radii, q, k, nprobe, key_dims, skip=True):
    """IvfIndex.search (EUCLIDEAN) restated here: clusters in route order with the early exit; a
    cluster with key dimensions met with a full heap takes scanPartitionWithHarmony -- rows whose
    partial distance over the key dimensions reaches the worst are skipped (skip=False scores
    them anyway), the rest are scored -squareDistance; other clusters the batched scan."""
    lids, dists = oracle.route(cent, q, oracle.EUCLIDEAN, nprobe)
    out = []
    for j in range(len(q)):
        kept = []
        for p_ in range(nprobe):
            cid = int(lids[j, p_])
            if len(kept) == k:
                lb = np.float32(np.float32(np.sqrt(np.float64(dists[j, p_]))) - radii[cid])
                if lb > 0 and np.float32(lb * lb) >= -kept[-1][0]:
                    break
            b, e = int(off[cid]), int(off[cid + 1])
            if key_dims[cid] is not None and len(kept) == k:
                for o in ords[b:e]:
                    partial = np.float32(0)
                    for d in key_dims[cid]:
                        df = np.float32(q[j, d] - db[o, d])
                        partial = np.float32(partial + np.float32(df * df))
                    if skip and partial >= -kept[-1][0]:
                        continue
                    s = np.float32(-oracle.square_distance(q[j], db[o]))
                    kept = sorted(kept + [(s, int(o))], key=lambda t: (-t[0], t[1]))[:k]
                continue
            if e == b:
                continue
            one = np.array([0, e - b], np.int64)
            ids, sc, cnt = oracle.ivfflat_search(cent[cid:cid + 1], one, ords[b:e], db, q[j:j + 1], oracle.EUCLIDEAN, k, 1)
            kept = sorted(kept + [(sc[0, i], int(ids[0, i])) for i in range(cnt[0])], key=lambda t: (-t[0], t[1]))[:k]
        out.append(kept)
    return out


def test_harmony_scan_of_partitions_with_key_dimensions(oracle):
    # partitions with key dimensions met with a full heap are scanned row by row with
    # squareDistance after the partial-distance skip; the skip drops only rows that could not
    # enter the heap here, so scoring them anyway gives the same results
    rng = np.random.default_rng(4)
    dim, nlist = 100, 10  # 100 dims: squareDistance and the batched order round differently
    cent = (2.0 * rng.standard_normal((nlist, dim))).astype(np.float32)
    assign = rng.integers(0, nlist, 3000).astype(np.int32)
    db = (cent[assign] + rng.standard_normal((3000, dim))).astype(np.float32)
    off, ords = oracle.build_ivf_lists(assign, nlist)
    q = (2.0 * rng.standard_normal((25, dim))).astype(np.float32)
    radii = oracle.ivf_radii(cent, off, ords, db)
    key_dims = [list(rng.choice(dim, 4, replace=False)) if l % 2 == 0 else None for l in range(nlist)]
    k, nprobe = 8, 6
    got = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, oracle.EUCLIDEAN, k, nprobe, key_dims=key_dims)
    want = _harmony_model(oracle, cent, off, ords, db, radii, q, k, nprobe, key_dims)
    noskip = _harmony_model(oracle, cent, off, ords, db, radii, q, k, nprobe, key_dims, skip=False)
    plain = oracle.ivfflat_search_full(cent, off, ords, db, radii, q, oracle.EUCLIDEAN, k, nprobe)
    changed = 0
    for j in range(len(q)):
        assert list(got[0][j, :got[2][j]]) == [i for _, i in want[j]], j
        assert list(got[1][j, :got[2][j]]) == [s for s, _ in want[j]], j
        assert want[j] == noskip[j], j
        changed += not np.array_equal(got[1][j], plain[1][j])
    assert changed > 0  # squareDistance scores differ from the batched order's somewhere
