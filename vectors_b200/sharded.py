"""Row-sharded search across ranks (one process per GPU).

The database is split into contiguous ordinal ranges exactly as IndexShards.build does
(vectors-db/.../index/IndexShards.java:64-81); every rank scans its range for the whole query
batch and returns its local top-k with shard-local ordinals.  The only exchange is those
per-rank lists: they are all-gathered over the process group (NCCL on GPUs) and merged on
every rank into the global top-k, ordinals offset by each shard's start, as
IndexShards.mergeWithOffsets does (IndexShards.java:168-211) but in the canonical
(score desc, ordinal asc) order.
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence

from .index_spi import merge_shards_device, shard_offsets

__all__ = ["shard_range", "gather_and_merge", "gather_rows", "ivf_search_sharded", "search_query_sharded",
           "assign_lists", "ivf_search_balanced", "deal_pairs", "ivf_search_pair_split",
           "ivfflat_search_pair_split"]


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Ordinal range [lo, hi) of `rank`'s shard."""
    offs = shard_offsets(n, world)
    return offs[rank], offs[rank + 1]


def _slice_call(fn, queries, lo: int, hi: int):
    """fn(queries[lo:hi]); a rank whose slice is empty (fewer queries than ranks) calls fn on one
    query and keeps none of its rows -- the library refuses empty batches, and every rank must
    still reach the collectives that follow with tensors of the right trailing shape."""
    if hi > lo:
        return fn(queries[lo:hi])
    out = fn(queries[:1])
    return tuple(t[:0] for t in out) if isinstance(out, tuple) else out[:0]


def gather_and_merge(local_ids, local_scores, local_counts, offsets: Sequence[int], k: int,
                     group=None, merge: Optional[Callable] = None):
    """All-gathers every rank's (ids [nq][kin], scores [nq][kin], counts [nq]) tensors and
    merges them into the global top-k.  `offsets` holds each shard's first ordinal (a sequence,
    or an int64 tensor on the device, which spares a host-to-device copy per call); `merge`
    defaults to the device merge (vx_merge_shards_device) and is called as
    merge(ids [S][nq][kin], scores [S][nq][kin], counts [S][nq], offsets tensor, k).
    Every rank takes the same collective steps and returns the same merged result."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    nq, kin = local_ids.shape
    dev = local_ids.device
    # one collective: ids, score bits and the count of each query packed into an int32 row
    packed = torch.cat([local_ids.to(torch.int32), local_scores.contiguous().view(torch.int32),
                        local_counts.to(torch.int32).reshape(nq, 1)], 1)
    g = torch.empty((world, nq, 2 * kin + 1), dtype=torch.int32, device=dev)
    if dev.type == "cuda":
        dist.all_gather_into_tensor(g, packed, group=group)
    else:  # gloo has no all_gather_into_tensor on every build: gather into per-rank views
        dist.all_gather(list(g.unbind(0)), packed, group=group)
    gi = g[:, :, :kin].contiguous()
    gs = g[:, :, kin:2 * kin].contiguous().view(torch.float32)
    gc = g[:, :, 2 * kin].contiguous()
    if isinstance(offsets, torch.Tensor):  # a device tensor prepared once: no host copy per call
        off = offsets[:world].to(device=dev, dtype=torch.int64)
    else:
        off = torch.tensor(list(offsets)[:world], dtype=torch.int64, device=dev)
    return (merge or merge_shards_device)(gi, gs, gc, off, k)


def gather_rows(local, total: int, group=None):
    """All-gathers a row slice: rank r holds rows [total*r/W, total*(r+1)/W) of a
    [total][...] tensor; every rank returns the whole tensor (slices padded to equal size
    for the collective)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    offs = shard_offsets(total, world)
    width = max(offs[i + 1] - offs[i] for i in range(world))
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    out = torch.empty((world, width) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    if local.device.type == "cuda":
        dist.all_gather_into_tensor(out, pad, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), pad, group=group)
    return torch.cat([out[i, : offs[i + 1] - offs[i]] for i in range(world)], 0)


def ivf_search_sharded(adapter, queries, k: int, nprobe: int, offsets: Sequence[int], group=None,
                       rescore_factor: int = 1):
    """IVF-PQ search over row-sharded indexes that share the centroids: each rank routes its
    slice of the queries, the routed lists are all-gathered, every rank scans its own rows for
    the whole batch, and the per-rank top-k lists are merged (gather_and_merge)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    lo, hi = shard_range(queries.shape[0], rank, world)
    lists = gather_rows(_slice_call(lambda qs: adapter.route_device(qs, nprobe), queries, lo, hi),
                        queries.shape[0], group)
    ids, sc, cnt = adapter.ivf_search_routed_device(queries, k, nprobe, lists, rescore_factor)
    return gather_and_merge(ids, sc, cnt, offsets, k, group)


def search_query_sharded(search, queries, group=None):
    """Query-parallel search over an index replicated on every rank (the IVF-PQ index of 10M
    rows is about 1 GB): rank r answers queries [nq*r/W, nq*(r+1)/W) with search(slice) ->
    (ids, scores, counts) and the slices are all-gathered, so every rank returns the whole
    batch.  No table build or list scan is duplicated and the load is balanced by the queries."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    nq = queries.shape[0]
    lo, hi = shard_range(nq, rank, world)
    ids, sc, cnt = _slice_call(search, queries, lo, hi)
    return gather_rows(ids, nq, group), gather_rows(sc, nq, group), gather_rows(cnt, nq, group)


def assign_lists(pairs_per_list, list_rows, world: int, table_rows: int = 600):
    """Deals lists to ranks for one routed batch: work(l) = pairs(l) * (rows(l) + table_rows)
    (the table build of a pair costs about as much as scanning `table_rows` rows); lists sorted
    by work (ties by id) are dealt in snake order 0..W-1, W-1..0, ... -- a longest-first deal
    that keeps the ranks within about one list's work of each other.  Deterministic, so every
    rank computes the same owners from the same inputs.  Returns owner[l] (int64)."""
    import torch

    work = pairs_per_list.to(torch.float64) * (list_rows.to(torch.float64) + table_rows)
    nl = work.shape[0]
    # sort by (work desc, id asc): stable sort on -work keeps ids ascending within ties
    order = torch.sort(-work, stable=True).indices
    pos = torch.arange(nl, device=work.device)
    rnd, r = pos // world, pos % world
    snake = torch.where(rnd % 2 == 0, r, world - 1 - r)
    owner = torch.empty(nl, dtype=torch.int64, device=work.device)
    owner[order] = snake
    return owner


def ivf_search_balanced(adapter, queries, k: int, nprobe: int, list_rows, group=None, rescore_factor: int = 1):
    """IVF-PQ search over an index replicated on every rank, balanced by list: each rank routes
    its slice of the queries, the routed lists are all-gathered, lists are dealt to ranks by
    their work in this batch (assign_lists), and each rank scans every query's pairs on its own
    lists -- full four-query table groups, no table built twice -- before the per-rank top-k
    lists are merged.  `list_rows` is a device tensor of the lists' row counts.  A list is never
    split, so a batch whose work concentrates in a few lists (centroids near every query, as
    in high-dimensional Gaussian mixtures) stays unbalanced; ivf_search_pair_split splits them.
    With rescore_factor > 1 each rank re-scores its own k * rescore_factor best, which can keep
    a row that is not among the k * rescore_factor best of the whole index (IvfIndex.pqSearch
    re-scores those only); search_query_sharded keeps the reference's results there."""
    import torch
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    nq = queries.shape[0]
    lo, hi = shard_range(nq, rank, world)
    lists = gather_rows(_slice_call(lambda qs: adapter.route_device(qs, nprobe), queries, lo, hi), nq, group)
    flat = lists.reshape(-1).long()
    pairs = torch.bincount(flat[flat >= 0], minlength=list_rows.shape[0])
    owner = assign_lists(pairs, list_rows, world)
    mine = torch.where((lists >= 0) & (owner[lists.clamp_min(0).long()] == rank), lists, torch.full_like(lists, -1))
    ids, sc, cnt = adapter.ivf_search_routed_device(queries, k, nprobe, mine, rescore_factor)
    return gather_and_merge(ids, sc, cnt, [0] * (world + 1), k, group)


def deal_pairs(lists, rank: int, world: int, group_size: int = 4):
    """Deals one routed batch's (query, list) pairs to ranks: lists [nq][nprobe] (int32, -1 for
    none) -> the same shape with the pairs of other ranks set to -1.  The pairs of each list, in
    query order, are cut into runs of `group_size` (the ADC scan's table group: one table build
    serves a run) and the runs are dealt round-robin, starting at rank (list id mod world), so
    every list -- the hub lists near every query included -- is split evenly over the ranks and
    every rank scans full groups.  Deterministic: all ranks derive the same deal from the same
    all-gathered lists, and every pair goes to exactly one rank."""
    import torch

    flat = lists.reshape(-1).long()
    valid = flat >= 0
    big = torch.iinfo(torch.int64).max
    key = torch.where(valid, flat, torch.full_like(flat, big))
    order = torch.sort(key, stable=True).indices  # by list, then by pair index (query order)
    sk = key[order]
    pos = torch.arange(sk.shape[0], device=sk.device) - torch.searchsorted(sk, sk)  # rank within its list
    owner_sorted = torch.remainder(pos // group_size + torch.where(sk == big, 0, sk), world)
    owner = torch.empty_like(owner_sorted)
    owner[order] = owner_sorted
    mine = torch.where(valid & (owner == rank), flat, torch.full_like(flat, -1))
    return mine.to(lists.dtype).reshape(lists.shape)


def ivf_search_pair_split(adapter, queries, k: int, nprobe: int, group=None):
    """IVF-PQ search over an index replicated on every rank, split by (query, list) pair: each
    rank routes its slice of the queries, the routed lists are all-gathered, deal_pairs gives
    every rank an even share of every list's pairs in whole four-query table groups, each rank
    scans its pairs for the whole batch, and the per-rank top-k lists are merged.  Every pair is
    scanned once, so the merged top-k is the single-GPU result (IvfIndex.pqSearch keeps the k
    best of all probed lists).  rescore_factor 1 only: with a re-score, a rank's own
    k * rescore_factor best need not be among the whole index's (use search_query_sharded)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    nq = queries.shape[0]
    lo, hi = shard_range(nq, rank, world)
    lists = gather_rows(_slice_call(lambda qs: adapter.route_device(qs, nprobe), queries, lo, hi), nq, group)
    mine = deal_pairs(lists, rank, world)
    ids, sc, cnt = adapter.ivf_search_routed_device(queries, k, nprobe, mine, 1)
    return gather_and_merge(ids, sc, cnt, [0] * (world + 1), k, group)


def ivfflat_search_pair_split(adapter, queries, k: int, nprobe: int, group=None):
    """IVF-flat search (IvfIndex.search, IvfIndex.java:170-226) over an index replicated on
    every rank, split by (query, list) pair: each rank routes its slice of the queries (lists and
    their distances), both are all-gathered, deal_pairs gives every rank an even share of every
    list's pairs in runs of 64 (the list scan's query group), each rank scans its pairs into
    per-slot results, a sum all-reduce combines them (each slot's keys come from one rank, the
    others hold zeros), and every rank merges all slots per query in route order with the
    EUCLIDEAN early exit -- the single-GPU result for the same routing.  Not for partitions with
    HARMONY key dimensions (the library refuses them)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    nq = queries.shape[0]
    lo, hi = shard_range(nq, rank, world)
    l_loc, d_loc = _slice_call(lambda qs: adapter.route_dist_device(qs, nprobe), queries, lo, hi)
    lists = gather_rows(l_loc, nq, group)
    ldist = gather_rows(d_loc, nq, group)
    keys, cnt = adapter.scan_pairs_device(queries, k, nprobe, deal_pairs(lists, rank, world, 64))
    dist.all_reduce(keys, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(cnt, op=dist.ReduceOp.SUM, group=group)
    return adapter.merge_pairs_device(k, nprobe, lists, ldist, keys, cnt)
