"""Row-sharded search over two CPU ranks (gloo): every rank scans its IndexShards range with the
oracle, vectors_b200.sharded.gather_and_merge all-gathers the per-rank top-k lists and merges
them with global ordinals; the result must equal the unsharded search on every rank."""
import os
import socket
import tempfile

import numpy as np
import pytest

SEEDS = (0xC0FFEE03, 0xC0FFEE01, 0xC0FFEE02)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import oracle as O
        from vectors_b200.index_spi import shard_offsets
        from vectors_b200.sharded import gather_and_merge, shard_range

        db = O.gen_mixture(n, 64, 8, 0.3, SEEDS[0], SEEDS[1], True)
        q = O.gen_mixture(9, 64, 8, 0.3, SEEDS[0], SEEDS[2], True)
        lo, hi = shard_range(n, rank, world)
        ids, sc, cnt = O.flat_search(db[lo:hi], q, O.COSINE, 10)

        def merge(gi, gs, gc, off, k):
            r = O.merge_shards(off.numpy(), gi.numpy(), gs.numpy(), gc.numpy(), k)
            return tuple(torch.from_numpy(np.ascontiguousarray(x)) for x in r)

        mi, ms, mc = gather_and_merge(torch.from_numpy(ids), torch.from_numpy(sc), torch.from_numpy(cnt),
                                      shard_offsets(n, world), 10, merge=merge)
        ref_ids, ref_sc, ref_cnt = O.flat_search(db, q, O.COSINE, 10)
        ok = (np.array_equal(mi.numpy(), ref_ids) and np.array_equal(mc.numpy(), ref_cnt)
              and np.allclose(ms.numpy(), ref_sc, rtol=1e-6, atol=0))
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [3000, 3001])
def test_two_rank_gloo_sharded_search_matches_unsharded(n):
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), n, d), nprocs=2, join=True, start_method="spawn")
        for r in range(2):
            with open(os.path.join(d, f"rank{r}")) as f:
                assert f.read() == "ok", f"rank {r}"


def _rows_worker(rank, world, port, total, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from vectors_b200.sharded import gather_rows, shard_range

        full = torch.arange(total * 3, dtype=torch.int32).reshape(total, 3)
        lo, hi = shard_range(total, rank, world)
        got = gather_rows(full[lo:hi].clone(), total)
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if torch.equal(got, full) else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [7, 8])
def test_two_rank_gloo_gather_rows(total):
    # the routed-list exchange of ivf_search_sharded: uneven query slices padded for the collective
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rows_worker, args=(2, _free_port(), total, d), nprocs=2, join=True, start_method="spawn")
        for r in range(2):
            with open(os.path.join(d, f"rank{r}")) as f:
                assert f.read() == "ok", f"rank {r}"


def _qshard_worker(rank, world, port, nq, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import oracle as O
        from vectors_b200.sharded import search_query_sharded

        db = O.gen_mixture(2000, 48, 8, 0.3, SEEDS[0], SEEDS[1], True)
        q = O.gen_mixture(nq, 48, 8, 0.3, SEEDS[0], SEEDS[2], True)

        def search(qs):
            if qs.shape[0] == 0:
                raise ValueError("queries must not be empty")  # as the library refuses them
            ids, sc, cnt = O.flat_search(db, qs.numpy(), O.DOT_PRODUCT, 7)
            return torch.from_numpy(ids), torch.from_numpy(sc), torch.from_numpy(cnt)

        mi, ms, mc = search_query_sharded(search, torch.from_numpy(q))
        ref = O.flat_search(db, q, O.DOT_PRODUCT, 7)
        ok = (np.array_equal(mi.numpy(), ref[0]) and np.array_equal(ms.numpy(), ref[1])
              and np.array_equal(mc.numpy(), ref[2]))
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("nq", [9, 10, 1])
def test_two_rank_gloo_query_sharded_search(nq):
    # the replicated-index mode of the IVF-PQ benchmark: queries split, results all-gathered
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_qshard_worker, args=(2, _free_port(), nq, d), nprocs=2, join=True, start_method="spawn")
        for r in range(2):
            with open(os.path.join(d, f"rank{r}")) as f:
                assert f.read() == "ok", f"rank {r}"


@pytest.mark.parametrize("world", [2, 3, 8])
def test_assign_lists_deals_every_list_once_and_balances(world):
    import torch

    from vectors_b200.sharded import assign_lists

    g = torch.Generator().manual_seed(world)
    pairs = torch.randint(0, 300, (4096,), generator=g)
    rows = torch.randint(10, 20000, (4096,), generator=g)
    owner = assign_lists(pairs, rows, world)
    assert owner.shape == (4096,) and int(owner.min()) >= 0 and int(owner.max()) < world
    assert torch.equal(owner, assign_lists(pairs.clone(), rows.clone(), world))  # deterministic
    work = pairs.double() * (rows.double() + 600)
    loads = torch.zeros(world, dtype=torch.float64).index_add_(0, owner, work)
    # within one list's work of the mean
    assert float(loads.max() - loads.mean()) <= float(work.max())


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_deal_pairs_gives_each_pair_to_one_rank_and_splits_every_list(world):
    # the pair deal of ivf_search_pair_split: a hub list probed by every query is split evenly
    import torch

    from vectors_b200.sharded import deal_pairs

    g = torch.Generator().manual_seed(7 + world)
    lists = torch.randint(-1, 50, (997, 8), generator=g, dtype=torch.int32)
    lists[:, 0] = 5  # probed by every query
    parts = [deal_pairs(lists, r, world) for r in range(world)]
    owned = torch.stack([(p >= 0).int() for p in parts]).sum(0)
    assert torch.equal(owned, (lists >= 0).int())  # every pair exactly once, none invented
    for r, p in enumerate(parts):
        assert p.dtype == lists.dtype and torch.equal(torch.where(p >= 0, p, lists), lists)
        assert torch.equal(p, deal_pairs(lists.clone(), r, world))  # deterministic
    for lst in range(50):
        c = [int((p == lst).sum()) for p in parts]
        assert max(c) - min(c) <= 4, (lst, c)  # within one four-pair table group


class _ListScanFake:
    """Stands in for IvfPqAdapter on the CPU: routing to the nprobe nearest centroids, and a
    routed search that scores every row of a query's given lists (-|q - x|^2 in float32) and
    keeps the k best by (score desc, ordinal asc)."""

    def __init__(self, db, cent, assign):
        self.db, self.cent, self.assign = db, cent, assign

    def route_device(self, qs, nprobe):
        import torch

        if qs.shape[0] == 0:
            raise ValueError("queries must not be empty")  # as the library refuses them
        q = qs.numpy()
        d = ((q[:, None, :] - self.cent[None, :, :]) ** 2).sum(2)
        return torch.from_numpy(np.argsort(d, axis=1, kind="stable")[:, :nprobe].astype(np.int32))

    def ivf_search_routed_device(self, qs, k, nprobe, lists, rescore_factor):
        import torch

        q, L = qs.numpy(), lists.numpy()
        ids = np.full((q.shape[0], k), -1, np.int32)
        sc = np.zeros((q.shape[0], k), np.float32)
        cnt = np.zeros(q.shape[0], np.int32)
        for i in range(q.shape[0]):
            rows = np.nonzero(np.isin(self.assign, L[i][L[i] >= 0]))[0]
            s = -((self.db[rows] - q[i]) ** 2).sum(1).astype(np.float32)
            o = np.lexsort((rows, -s))[:k]
            ids[i, : len(o)], sc[i, : len(o)], cnt[i] = rows[o], s[o], len(o)
        return torch.from_numpy(ids), torch.from_numpy(sc), torch.from_numpy(cnt)


def _pair_split_worker(rank, world, port, out_dir, nq=41):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import vectors_b200.sharded as S
        from oracle import oracle as O

        db = O.gen_mixture(1500, 16, 6, 0.4, SEEDS[0], SEEDS[1], False)
        q = O.gen_mixture(nq, 16, 6, 0.4, SEEDS[0], SEEDS[2], False)
        cent = db[:12].copy()
        assign = np.argmin(((db[:, None, :] - cent[None]) ** 2).sum(2), 1)
        fake = _ListScanFake(db, cent, assign)

        def merge(gi, gs, gc, off, k):
            r = O.merge_shards(off.numpy(), gi.numpy(), gs.numpy(), gc.numpy(), k)
            return tuple(torch.from_numpy(np.ascontiguousarray(x)) for x in r)

        real = S.gather_and_merge
        S.gather_and_merge = lambda *a, **kw: real(*a, merge=merge, **kw)
        try:
            mi, ms, mc = S.ivf_search_pair_split(fake, torch.from_numpy(q), 9, 4)
        finally:
            S.gather_and_merge = real
        ref = fake.ivf_search_routed_device(torch.from_numpy(q), 9, 4, fake.route_device(torch.from_numpy(q), 4), 1)
        ok = all(np.array_equal(a.numpy(), b.numpy()) for a, b in zip((mi, ms, mc), ref))
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("nq", [41, 1])
def test_two_rank_gloo_pair_split_search_matches_unsplit(nq):
    # ivf_search_pair_split: queries routed per rank, lists all-gathered, pairs dealt, per-rank
    # top-k merged; equals the search over every routed pair on one rank (one query: a rank
    # with an empty slice still takes part in the collectives)
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_pair_split_worker, args=(2, _free_port(), d, nq), nprocs=2, join=True,
                           start_method="spawn")
        for r in range(2):
            with open(os.path.join(d, f"rank{r}")) as f:
                assert f.read() == "ok", f"rank {r}"


class _SlotFake:
    """Stands in for IvfFlatAdapter's pair steps on the CPU: per-slot results are the rows of the
    slot's list scored -|q - x|^2 as int64 keys (score bits above 0xFFFFFFFF - ordinal), and the
    merge keeps the k best keys of all slots."""

    def __init__(self, db, cent, assign):
        self.db, self.cent, self.assign = db, cent, assign

    def route_dist_device(self, qs, nprobe):
        import torch

        if qs.shape[0] == 0:
            raise ValueError("queries must not be empty")  # as the library refuses them
        d = ((qs.numpy()[:, None, :] - self.cent[None]) ** 2).sum(2).astype(np.float32)
        o = np.argsort(d, axis=1, kind="stable")[:, :nprobe]
        return torch.from_numpy(o.astype(np.int32)), torch.from_numpy(np.take_along_axis(d, o, 1))

    @staticmethod
    def _key(score, ordinal):
        b = np.float32(score).view(np.uint32).astype(np.uint64)
        b = np.where(b >> np.uint64(31), ~b & np.uint64(0xFFFFFFFF), b | np.uint64(0x80000000))
        return ((b << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.uint64(ordinal))).astype(np.uint64)

    def scan_pairs_device(self, qs, k, nprobe, lists):
        import torch

        q, L = qs.numpy(), lists.numpy()
        keys = np.zeros((L.shape[1], q.shape[0], k), np.uint64)
        cnt = np.zeros((L.shape[1], q.shape[0]), np.int32)
        for i in range(q.shape[0]):
            for s in range(L.shape[1]):
                if L[i, s] < 0:
                    continue
                rows = np.nonzero(self.assign == L[i, s])[0]
                kk = np.sort(self._key(-((self.db[rows] - q[i]) ** 2).sum(1), rows))[::-1][:k]
                keys[s, i, : len(kk)], cnt[s, i] = kk, len(kk)
        return torch.from_numpy(keys.view(np.int64)), torch.from_numpy(cnt)

    def merge_pairs_device(self, k, nprobe, lists, dist, keys, counts):
        import torch

        ky, ct = keys.numpy().view(np.uint64), counts.numpy()
        best = np.zeros((ky.shape[1], k), np.uint64)
        for i in range(ky.shape[1]):
            allk = np.concatenate([ky[s, i, : ct[s, i]] for s in range(ky.shape[0])])
            top = np.sort(allk)[::-1][:k]
            best[i, : len(top)] = top
        return torch.from_numpy(best.view(np.int64))


def _flat_split_worker(rank, world, port, out_dir, nq=37):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import oracle as O
        from vectors_b200.sharded import ivfflat_search_pair_split

        db = O.gen_mixture(900, 12, 5, 0.4, SEEDS[0], SEEDS[1], False)
        q = O.gen_mixture(nq, 12, 5, 0.4, SEEDS[0], SEEDS[2], False)
        cent = db[:9].copy()
        assign = np.argmin(((db[:, None, :] - cent[None]) ** 2).sum(2), 1)
        fake = _SlotFake(db, cent, assign)
        got = ivfflat_search_pair_split(fake, torch.from_numpy(q), 6, 4)
        lists, dd = fake.route_dist_device(torch.from_numpy(q), 4)
        ref = fake.merge_pairs_device(6, 4, lists, dd, *fake.scan_pairs_device(torch.from_numpy(q), 6, 4, lists))
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if torch.equal(got, ref) else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("nq", [37, 1])
def test_two_rank_gloo_ivfflat_pair_split_matches_unsplit(nq):
    # ivfflat_search_pair_split: routed lists and distances all-gathered, pairs dealt in runs of
    # 64, disjoint per-slot results combined by a sum all-reduce, merged on every rank
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_flat_split_worker, args=(2, _free_port(), d, nq), nprocs=2, join=True,
                           start_method="spawn")
        for r in range(2):
            with open(os.path.join(d, f"rank{r}")) as f:
                assert f.read() == "ok", f"rank {r}"
