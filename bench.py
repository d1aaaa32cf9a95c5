"""Benchmark: queries/sec of the 10M x 768 FLAT (COSINE, fp32, top-10) batch scan, with the
10M x 768 IVF-PQ (nlist 4096, M=96, nprobe 32, top-10) scan reported beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

One process per GPU (torchrun for N > 1).  The database is split into contiguous ordinal
ranges (IndexShards.build); every rank scans its range for the whole query batch, the
per-rank top-10 lists are all-gathered over NCCL and merged on the device (IndexShards.
mergeWithOffsets).  `value` = queries of the batch / step time (max over ranks, CUDA events,
inputs resident in HBM); `e2e` = the same through the host-buffer C ABI call (queries copied
in, results copied out inside the timed region).  `--impl reference` times the CPU
restatement of the reference's Java path (the oracle) on the host cores instead.

Synthetic data: seeded Gaussian mixtures with the reference benchmark's shapes (no dataset is
needed); both arms draw from the same generator.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FLAT = dict(n=10_000_000, dim=768, comps=64, sigma=0.3, nq=10_000, k=10, metric=2)
IVF = dict(n=10_000_000, dim=768, comps=1024, sigma=0.3, nq=10_000, k=10, nlist=4096, m=96, ks=256,
           nprobe=32, train=500_000, pq_train=25_000)
SEED_DB, SEED_Q, SEED_C = 0xC0FFEE01, 0xC0FFEE02, 0xC0FFEE03
FLAT_TRAFFIC_FIXED, FLAT_TRAFFIC_PER_ROW = 2.03e9, 3024.0  # bytes per scan launch (measured, 10k queries)
METRIC = "queries/sec, 10M x 768 FLAT COSINE top-10"
CHUNK = 65536


# ------------------------------------------------------------------ synthetic data
def centres(comps, dim, seed):
    return np.random.Generator(np.random.PCG64([seed, 0xCE])).standard_normal((comps, dim), dtype=np.float32)


def gen_chunk(c, dim, cent, sigma, seed, normalize):
    rng = np.random.Generator(np.random.PCG64([seed, c]))
    comp = rng.integers(0, cent.shape[0], size=CHUNK)
    x = cent[comp]
    x += sigma * rng.standard_normal((CHUNK, dim), dtype=np.float32)
    if normalize:
        x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x


def gen_rows(first, count, dim, cent, sigma, seed, normalize, sink=None, threads=None):
    """Rows [first, first+count) of the seeded mixture; chunk-seeded, so any slice of the
    global dataset is identical however it is split.  sink(offset, array) receives pieces."""
    out = None if sink else np.empty((count, dim), np.float32)
    c0, c1 = first // CHUNK, (first + count + CHUNK - 1) // CHUNK
    threads = threads or min(32, os.cpu_count() or 4)

    def work(c):
        x = gen_chunk(c, dim, cent, sigma, seed, normalize)
        lo, hi = max(first, c * CHUNK), min(first + count, (c + 1) * CHUNK)
        return lo - first, x[lo - c * CHUNK: hi - c * CHUNK]

    with cf.ThreadPoolExecutor(threads) as ex:
        for off, piece in ex.map(work, range(c0, c1)):
            if sink:
                sink(off, piece)
            else:
                out[off: off + len(piece)] = piece
    return out


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clocks, power and throttle reasons of this rank's GPU sampled during the timed region.

    Reads NVML in a background thread of this process (50 ms period; the same counters
    nvidia-smi's clocks / clocks_event_reasons fields report); an external nvidia-smi poller is
    the fallback when NVML is missing.  Only one rank samples: several pollers on one box stall
    kernel launches measurably."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, local_rank, enabled=True):
        cvd = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [s.strip() for s in cvd.split(",") if s.strip()]
        self.gpu = ids[local_rank] if local_rank < len(ids) else str(local_rank)
        self.enabled = enabled
        self.samples = []
        self.max_mhz = None
        self.thread = None
        self.proc = None
        self.stop_evt = None

    def start(self):
        if not self.enabled:
            return
        try:
            import threading

            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(int(self.gpu))
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            masks = [(name, getattr(nv, attr)) for name, attr in self.REASONS]
            self.stop_evt = threading.Event()

            def run():
                while not self.stop_evt.is_set():
                    try:
                        mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((mhz, [nm for nm, m in masks if bits & m]))
                    except Exception:
                        pass
                    self.stop_evt.wait(0.05)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
        except Exception:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", "-i", self.gpu, "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                     "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                     "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                self.proc = None

    def stop(self):
        if not self.enabled:
            return None
        if self.thread is not None:
            self.stop_evt.set()
            self.thread.join(timeout=2)
        elif self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            names = [nm for nm, _ in self.REASONS]
            for line in out.strip().splitlines():
                f = [x.strip() for x in line.split(",")]
                try:
                    self.max_mhz = float(f[1])
                    self.samples.append((float(f[0]), [nm for nm, v in zip(names, f[2:6]) if v.lower() == "active"]))
                except (ValueError, IndexError):
                    continue
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no NVML / nvidia-smi"]}
        sm = [m for m, _ in self.samples]
        reasons = sorted({r for _, rs in self.samples for r in rs})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sm), "source": "NVML (rank 0's GPU)" if self.thread else "nvidia-smi"}


# ------------------------------------------------------------------ helpers
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def cpu_flat_baseline(db_sample, q_sample, total_rows, metric):
    """The oracle (CPU restatement of FlatScanAdapter.searchBatch) on a bounded sample."""
    from oracle import oracle as O

    th = os.cpu_count() or 1
    t = time.perf_counter()
    O.flat_search(db_sample, q_sample, metric, FLAT["k"], O.REFERENCE_HEAP, th)
    dt = time.perf_counter() - t
    qps = len(q_sample) / dt * (len(db_sample) / total_rows)
    return qps, th, dt


def parity(got, ref, exact, rows):
    """Compares a GPU result (ids [q][k], scores [q][k], counts [q]) with the oracle's on the same
    queries and rows: ids must be identical, scores bit-exact (integer / code paths) or within
    1e-4 relative (fp32 / fp16 paths)."""
    gi, gs, gc = (np.asarray(a) for a in got)
    ri, rs, rc = ref
    ids_equal, bit, max_rel = True, True, 0.0
    for i in range(len(rc)):
        c = int(rc[i])
        if int(gc[i]) != c or not np.array_equal(gi[i, :c], ri[i, :c]):
            ids_equal = False
            continue
        if not np.array_equal(gs[i, :c], rs[i, :c]):
            bit = False
        if c:
            a, b = gs[i, :c].astype(np.float64), rs[i, :c].astype(np.float64)
            max_rel = max(max_rel, float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-30))))
    return {"queries": int(len(rc)), "rows": int(rows), "against": "oracle (CPU restatement of the reference path)",
            "bar": "ids equal, scores bit-exact" if exact else "ids equal, scores within 1e-4 relative",
            "ids_equal": ids_equal, "scores_bit_exact": bit, "max_rel_score_diff": max_rel,
            "ok": bool(ids_equal and (bit if exact else max_rel <= 1e-4))}


def timed_oracle(fn):
    """Runs one oracle call on all host threads; returns (result, seconds, threads)."""
    th = os.cpu_count() or 1
    t = time.perf_counter()
    r = fn(th)
    return r, time.perf_counter() - t, th


def pinned(x):
    """A page-locked copy of a host array (the end-to-end calls copy their queries from it)."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).pin_memory().numpy()


def e2e_host(args, call, nq, h2d, d2h):
    """End to end through a host-buffer C ABI call (queries copied in from page-locked memory,
    results copied out inside the timed region), one GPU: K blocking calls after one warm-up
    call, host wall clock."""
    call()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        call()
    dt = (time.perf_counter() - t0) / args.steps
    return {"value": nq / dt, "unit": "queries/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "timing": "host wall clock around the blocking host-buffer call (one GPU)"}


# ------------------------------------------------------------------ reference arm
def run_reference(args, rank):
    if rank != 0:
        return 0
    from oracle import oracle as O

    O.lib()
    rows = args.ref_rows
    cent = centres(FLAT["comps"], FLAT["dim"], SEED_C)
    db = gen_rows(0, rows, FLAT["dim"], cent, FLAT["sigma"], SEED_DB, True)
    q = gen_rows(0, args.ref_queries, FLAT["dim"], cent, FLAT["sigma"], SEED_Q, True)
    th = os.cpu_count() or 1
    for _ in range(args.warmup):
        O.flat_search(db, q[:4], FLAT["metric"], FLAT["k"], O.REFERENCE_HEAP, th)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        O.flat_search(db, q, FLAT["metric"], FLAT["k"], O.REFERENCE_HEAP, th)
        times.append(time.perf_counter() - t)
    step = sum(times) / len(times)
    qps = args.ref_queries / step * (rows / FLAT["n"])
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": qps,
        "unit": "queries/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "FLAT COSINE fp32, n=10,000,000, dim=768, k=10", "n": FLAT["n"], "dim": FLAT["dim"],
                   "k": FLAT["k"], "metric": "COSINE"},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": th, "kind": "port",
                         "sample": f"{args.ref_queries} queries x {rows:,} rows per step (first rows of the "
                                   f"10M dataset); QPS scaled by rows/10,000,000"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n", "--flat-n", dest="n", type=int, default=FLAT["n"],
                    help="FLAT rows (--flat-n under torchrun, whose own options take --n)")
    ap.add_argument("--nq", type=int, default=FLAT["nq"])
    ap.add_argument("--no-ivf", action="store_true")
    ap.add_argument("--no-quant", action="store_true", help="skip the SQ8, BQ and FP16 scan legs")
    ap.add_argument("--no-ivfflat", action="store_true", help="skip the IVF-flat leg")
    ap.add_argument("--ivfflat-n", type=int, default=IVFFLAT["n"])
    ap.add_argument("--sq8-n", type=int, default=SQ8["n"], help="smaller cases for profiling")
    ap.add_argument("--bq-n", type=int, default=BQ["n"])
    ap.add_argument("--bbq-n", type=int, default=1_000_000, help="rows per GPU of the BBQ scan")
    ap.add_argument("--fp16-n", type=int, default=FP16["n_per_gpu"], help="rows per GPU")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--ivf-n", type=int, default=IVF["n"])
    ap.add_argument("--ivf-nlist", type=int, default=IVF["nlist"], help="smaller cases for profiling keep n/nlist")
    ap.add_argument("--ivf-nq", type=int, default=IVF["nq"])
    ap.add_argument("--ivfflat-split", default="auto", choices=["auto", "pair", "query"],
                    help="IVF-flat at N > 1: deal (query, list) pairs, split the queries, or auto (queries "
                         "at 2 ranks, pairs from 4)")
    ap.add_argument("--ivf-split", default="auto", choices=["auto", "pair", "query"],
                    help="IVF-PQ at N > 1: deal (query, list) pairs, split the queries, or auto (queries at "
                         "2 ranks, pairs from 4)")
    ap.add_argument("--ref-rows", type=int, default=1_000_000)
    ap.add_argument("--ref-queries", type=int, default=256)
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch
    import torch.distributed as dist

    import vectors_b200 as vx
    from vectors_b200 import _native as N
    from vectors_b200.sharded import gather_and_merge

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    hbm_peak, tc_burst, tc_sustained, peak_kind = peaks()
    n_total = args.n
    offs = vx.shard_offsets(n_total, world)
    lo, hi = offs[rank], offs[rank + 1]
    dim, k, nq = FLAT["dim"], FLAT["k"], args.nq

    # ---- FLAT data (this rank's ordinal range), generated straight into HBM
    cent = centres(FLAT["comps"], dim, SEED_C)
    rows = torch.empty((hi - lo, dim), dtype=torch.float32, device=dev)

    def sink(off, piece):
        rows[off: off + len(piece)].copy_(torch.from_numpy(np.ascontiguousarray(piece)), non_blocking=False)

    gen_rows(lo, hi - lo, dim, cent, FLAT["sigma"], SEED_DB, True, sink=sink)
    q_host = gen_rows(0, nq, dim, cent, FLAT["sigma"], SEED_Q, True)
    q_pinned = torch.from_numpy(q_host).pin_memory()
    q_dev = q_pinned.to(dev)

    flat = vx.FlatScanAdapter(device=local)
    flat.build(rows, vx.SimilarityFunction.COSINE)  # device rows: copied device-to-device
    cpu_sample = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu_sample = rows[: args.ref_rows].cpu().numpy()
    del rows
    torch.cuda.empty_cache()


    gm_events = []  # (start, end) around each step's all-gather + shard merge (N > 1)
    offs_dev = torch.tensor(offs[:world], dtype=torch.int64, device=dev)

    def flat_step():
        ids, sc, cnt = flat.search_batch_device(q_dev, k)
        if world == 1:
            return ids, sc, cnt
        e_a, e_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_a.record()
        out = gather_and_merge(ids, sc, cnt, offs_dev, k)
        e_b.record()
        gm_events.append((e_a, e_b))
        return out

    for _ in range(args.warmup):
        flat_step()
    torch.cuda.synchronize()
    gm_events.clear()
    barrier()
    launches0 = vx.kernel_launches()
    N.profile_reset()
    N.profile_enable(True)
    clocks = ClockSampler(local, enabled=(rank == 0))
    clocks.start()
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        out = flat_step()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    N.profile_enable(False)
    prof = N.profile_read()
    launches = vx.kernel_launches() - launches0
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms_local)
    qps = nq / (ms / 1e3)
    per_rank = None
    if world > 1:  # each rank's step time and its parts: load balance and the fixed per-rank work
        slots = ["gemm_scan", "pilot", "merge", "rescore", "fallback"]
        gm_ms = sum(a_.elapsed_time(b_) for a_, b_ in gm_events) / args.steps
        vals = [ms_local] + [prof.get(sl, (0.0, 0))[0] / args.steps for sl in slots] + [gm_ms]
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        g_ = torch.empty((world, len(vals)), dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(g_, t)
        per_rank = {"step_ms": g_[:, 0].tolist()}
        for j, sl in enumerate(slots):
            per_rank[sl + "_ms"] = g_[:, 1 + j].tolist()
        per_rank["allgather_and_shard_merge_ms"] = g_[:, -1].tolist()

    # roofline of the dominant kernel: the tcgen05 scan (algorithmic flops 2 * nq * rows * dim)
    g_ms, g_n = prof["gemm_scan"]
    flops_step = 2.0 * nq * (hi - lo) * dim
    gemm_ms_step = g_ms / args.steps
    achieved = flops_step / (gemm_ms_step / 1e3) / 1e12 if gemm_ms_step > 0 else None
    roofline = {
        "bound": "tensor",
        "achieved": achieved,
        "peak": tc_sustained,
        "unit": "TFLOP/s",
        "frac": (achieved / tc_sustained) if achieved else None,
        "traffic": None,
        "kernel": "gemm_scan_kernel (tcgen05 kind::f16, fused top-K)",
        "peak_source": f"{peak_kind} dense bf16/fp16 sustained",
        "kernel_ms_per_step": gemm_ms_step,
        "launches_per_step": g_n / args.steps,
        "breakdown_ms_per_step": {kk: v[0] / args.steps for kk, v in prof.items() if v[1]},
        "per_rank": per_rank,
    }
    # DRAM bytes of one scan launch: ncu's dram__bytes_read.sum + dram__bytes_write.sum at 600k and
    # 2.4M rows (10k queries) fit 2.03 GB + 3,024 B per row; scaled to this rank's rows
    roofline["traffic"] = FLAT_TRAFFIC_FIXED + FLAT_TRAFFIC_PER_ROW * (hi - lo)
    roofline["traffic_source"] = ("ncu DRAM bytes of the scan at 600k and 2.4M rows, linear fit scaled to "
                                  "this rank's rows")
    roofline["algorithmic_bytes"] = 2.0 * (hi - lo) * dim + 2.0 * nq * dim

    # ---- end to end through the host-buffer C ABI (queries in, results out every step)
    q_np = q_pinned.numpy()

    def e2e_step():
        # the host-buffer C ABI call: H2D queries, scan, D2H results (blocking)
        res = flat.search_batch_arrays(q_np, k)
        if world == 1:
            return res
        # shard results meet through the same NCCL all-gather + device merge, then D2H
        li, ls, lc = (torch.from_numpy(a).to(dev) for a in res)
        mi, ms_, mc = gather_and_merge(li, ls, lc, offs, k)
        return mi.cpu(), ms_.cpu(), mc.cpu()

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps)
    h2d = nq * dim * 4 + (nq * k * 8 + nq * 4 if world > 1 else 0)
    d2h = (nq * k * 8 + nq * 4) * (2 if world > 1 else 1)
    e2e = {"value": nq / e2e_s, "unit": "queries/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "timing": "host wall clock around the blocking host-buffer call, max over ranks"}

    # ---- parity (rank 0, N=1): the same path on an index of the dataset's first rows, 64 queries
    #      checked against the oracle (the 10M-row index itself is too large for the CPU check)
    flat_parity = None
    if cpu_sample is not None:
        from oracle import oracle as O

        sub = vx.FlatScanAdapter(device=local)
        sub.build(cpu_sample, vx.SimilarityFunction.COSINE)
        got = sub.search_batch_arrays(q_host[:64], k)
        sub.close()
        ref, _, _ = timed_oracle(lambda th: O.flat_search(cpu_sample, q_host[:64], FLAT["metric"], k, O.CANONICAL, th))
        flat_parity = parity(got, ref, False, len(cpu_sample))

    # ---- CPU baseline (rank 0, N=1): the oracle on a bounded sample
    cpu = None
    if cpu_sample is not None:
        qs = q_host[: args.ref_queries]
        cqps, cores, dt = cpu_flat_baseline(cpu_sample, qs, n_total, FLAT["metric"])
        cpu = {"value": cqps, "unit": "queries/s", "cores": cores, "kind": "port",
               "sample": f"{len(qs)} queries x {len(cpu_sample):,} rows ({dt:.1f} s); QPS scaled by rows/{n_total:,}"}
    flat.close()
    torch.cuda.empty_cache()

    def leg(fn, *a):
        # One GPU: a failed secondary leg is reported in its slot and the line still prints.
        # Several ranks: the exception propagates (a rank that skipped a leg's collectives
        # would leave the others waiting in them).
        if world > 1:
            return fn(*a)
        try:
            return fn(*a)
        except Exception as e:
            return {"error": f"{type(e).__name__}: {e}"[:500]}

    # ---- IVF-PQ sub-result
    ivf = None
    if not args.no_ivf:
        ivf = leg(run_ivf, args, rank, world, local, dev, barrier, max_over_ranks, hbm_peak, peak_kind)

    ivfflat = None
    if not args.no_ivf and not args.no_ivfflat:
        ivfflat = leg(run_ivfflat, args, rank, world, local, dev, barrier, max_over_ranks, peak_kind)

    # ---- SQ8 and BQ candidate scans (selectApproximateCandidates, k = 100)
    sq8 = bq = fp16 = None
    if not args.no_quant:
        sq8 = leg(run_sq8, args, rank, world, local, dev, barrier, max_over_ranks, tc_sustained, peak_kind)
        bq = leg(run_bq, args, rank, world, local, dev, barrier, max_over_ranks, tc_sustained, peak_kind)
        fp16 = leg(run_fp16, args, rank, world, local, dev, barrier, max_over_ranks, tc_sustained, peak_kind)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": qps,
            "unit": "queries/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16-mma+f32-rescore",
            "data": "synthetic",
            "config": {"workload": f"FLAT COSINE fp32, n={n_total:,}, dim={dim}, queries={nq:,}, k={k}",
                       "n": n_total, "dim": dim, "queries_per_step": nq, "k": k, "metric": "COSINE",
                       "parallelism": f"row-sharded x{world}, NCCL all-gather + merge",
                       "l2": "inputs larger than L2 (fp16 scan operand 15.4 GB)"},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "parity": flat_parity,
            "gpu_launches": launches,
            "clocks": clk,
            "ivf_flat": ivfflat,
            "sq8": sq8,
            "bq": bq,
            "fp16": fp16,
            "ivf_pq": ivf,  # last, so that a tail of the line keeps the second headline
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def run_ivf(args, rank, world, local, dev, barrier, max_over_ranks, hbm_peak, peak_kind):
    import torch
    import torch.distributed as dist

    import vectors_b200 as vx
    from vectors_b200 import _native as N
    from vectors_b200.sharded import gather_rows, ivf_search_pair_split, search_query_sharded

    P = IVF
    n, dim, nlist, m, ks = args.ivf_n, P["dim"], args.ivf_nlist, P["m"], P["ks"]
    offs = vx.shard_offsets(n, world)
    lo, hi = offs[rank], offs[rank + 1]
    offs_dev = torch.tensor(offs[:world], dtype=torch.int64, device=dev)
    cent_mix = centres(P["comps"], dim, SEED_C ^ 0x1F)
    g = torch.Generator(device=dev)
    g.manual_seed(42)
    # coarse centroids: k-means (10 Lloyd iterations) on a 500k-row sample, trained on rank 0
    cent = torch.empty((nlist, dim), dtype=torch.float32, device=dev)
    if rank == 0:
        sample = torch.from_numpy(gen_rows(0, min(P["train"], n), dim, cent_mix, P["sigma"], SEED_DB ^ 0x1F, False)).to(dev)
        cent.copy_(sample[torch.randperm(len(sample), generator=g, device=dev)[:nlist]])
        for _ in range(10):
            a = nearest(sample, cent)
            s = torch.zeros_like(cent).index_add_(0, a, sample)
            c = torch.bincount(a, minlength=nlist).clamp_min(1).unsqueeze(1).float()
            cent = torch.where(torch.bincount(a, minlength=nlist).unsqueeze(1) > 0, s / c, cent)
        del sample
    if world > 1:
        dist.broadcast(cent, 0)
    # this rank's rows, their lists, residuals; PQ codebooks trained on rank 0's residuals
    rows = torch.from_numpy(gen_rows(lo, hi - lo, dim, cent_mix, P["sigma"], SEED_DB ^ 0x1F, False)).to(dev)
    assign = nearest(rows, cent)
    books = torch.empty((m, ks, dim // m), dtype=torch.float32, device=dev)
    if rank == 0:
        pick = torch.randperm(len(rows), generator=g, device=dev)[: P["pq_train"]]
        resid = (rows[pick] - cent[assign[pick]]).view(-1, m, dim // m).transpose(0, 1).contiguous()
        books.copy_(pq_kmeans(resid, ks, g))
    if world > 1:
        dist.broadcast(books, 0)
    codes = torch.empty((len(rows), m), dtype=torch.uint8, device=dev)
    for s in range(0, len(rows), 32768):
        r = (rows[s: s + 32768] - cent[assign[s: s + 32768]]).view(-1, m, dim // m).transpose(0, 1)
        d = torch.cdist(r, books)  # [m, b, ks]
        codes[s: s + 32768] = d.argmin(2).transpose(0, 1).to(torch.uint8)
    del rows
    torch.cuda.empty_cache()
    counts = torch.bincount(assign, minlength=nlist)
    if world > 1:
        # The 10M-row IVF-PQ index (~1 GB) is replicated: every rank gathers all ranks' codes
        # and assignments and builds the whole index; queries are then split across ranks.
        dist.all_reduce(counts)
        codes = gather_rows(codes.contiguous(), n)
        assign = gather_rows(assign.contiguous(), n)
    order = torch.argsort(assign, stable=True).to(torch.int32)
    codes_h = codes.cpu().numpy()
    own = torch.bincount(assign, minlength=nlist)
    loff = torch.zeros(nlist + 1, dtype=torch.int64, device=dev)
    loff[1:] = torch.cumsum(own, 0)
    a = vx.IvfPqAdapter(nprobe=P["nprobe"], device=local)
    a.build_prebuilt(cent.cpu().numpy(), loff.cpu().numpy(), order.cpu().numpy(), books.cpu().numpy().reshape(-1),
                     codes_h, m, ks, vx.SimilarityFunction.EUCLIDEAN)
    nq, k = args.ivf_nq, P["k"]
    qh = gen_rows(0, nq, dim, cent_mix, P["sigma"], SEED_Q ^ 0x1F, False)
    q = torch.from_numpy(qh).to(dev)
    # algorithmic bytes: codes + ordinals of every probed list row, per query
    dq = torch.cdist(q, cent)
    probed = dq.topk(P["nprobe"], largest=False).indices
    bytes_step = float(counts[probed].sum().item()) * (m + 4)

    # auto: the split that measured faster at this rank count (one-GPU emulation of the ranks'
    # own work at 2 / 4 / 8 ranks, and 2 B200s): queries at 2 ranks, pairs from 4 up, where the
    # query slices leave most four-query table groups part-filled
    split = args.ivf_split if args.ivf_split != "auto" else ("query" if world <= 2 else "pair")

    def step():
        if world == 1:
            return a.ivf_search_device(q, k, P["nprobe"])[0]
        if split == "query":
            # replicated index: each rank answers its slice of the queries; results all-gathered
            return search_query_sharded(lambda qs: a.ivf_search_device(qs, k, P["nprobe"]), q)[0]
        # replicated index, (query, list) pairs dealt to ranks in four-pair table groups: every
        # list (the hub lists near every query included) split evenly, full groups on every rank
        return ivf_search_pair_split(a, q, k, P["nprobe"])[0]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    N.profile_reset()
    N.profile_enable(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    N.profile_enable(False)
    prof = N.profile_read()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    adc_local = prof["adc_scan"][0] / args.steps
    adc_ms = max_over_ranks(adc_local)
    per_rank = None
    if world > 1:  # load balance of the query split: each rank's scan time
        t = torch.tensor([adc_local], dtype=torch.float64, device=dev)
        g_ = torch.empty((world, 1), dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(g_, t)
        per_rank = {"adc_ms": g_[:, 0].tolist()}
    # per GPU: this job's algorithmic bytes split over the ranks, over the slowest rank's scan
    achieved = bytes_step / world / (adc_ms / 1e3) / 1e9 if adc_ms > 0 else None
    # shared-memory gather roof of the grouped ADC scan: each (four-query group, row, subspace)
    # reads one 16-byte interleaved table entry, and a warp's 32 such reads take at least four
    # 128-byte wavefronts; at 128 bytes per clock per SM that is this many seconds per step
    pair_rows = bytes_step / (m + 4)
    gather_bytes = pair_rows / 4.0 * m * 16.0 / world
    smem_peak = 148 * 128 * 1.965e9  # bytes/s: 148 SMs x 128 B/clk x max SM clock (nominal)
    smem_frac = (gather_bytes / smem_peak) / (adc_ms / 1e3) if adc_ms > 0 else None
    # with codes drawn at random, a quarter-warp's eight 16-byte reads land on 2.54 of the
    # eight 16-byte bank groups' worth of wavefronts on average (the expected largest number
    # of distinct codes sharing a bank group), not 1: the gather roof the data allows
    random_frac = smem_frac * 2.5408 if smem_frac else None
    par = cpu = e2e = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle as O

        cent_h, loff_h, ord_h, books_h = (cent.cpu().numpy(), loff.cpu().numpy(), order.cpu().numpy(),
                                          books.cpu().numpy().reshape(-1))
        qs = qh[:256]
        ref, dt, th = timed_oracle(lambda t: O.ivfpq_search(cent_h, loff_h, ord_h, m, ks, books_h, codes_h, qs, 0, k,
                                                            P["nprobe"], 1, None, O.CANONICAL, t))
        par = parity(a.ivf_search_arrays(qs, k, P["nprobe"]), ref, True, n)
        cpu = {"value": len(qs) / dt, "unit": "queries/s", "cores": th, "kind": "port",
               "sample": f"{len(qs)} queries over the same 10M-row index ({dt:.1f} s)"}
        qp = pinned(qh)
        e2e = e2e_host(args, lambda: a.ivf_search_arrays(qp, k, P["nprobe"]), nq, nq * dim * 4, nq * (k * 8 + 4))
    a.close()
    return {
        "value": nq / (ms / 1e3),
        "unit": "queries/s",
        "ms_per_step": ms,
        "config": {"workload": f"IVF-PQ EUCLIDEAN n={n:,} dim={dim} nlist={nlist} M={m} ks={ks} nprobe={P['nprobe']} "
                               f"rescore=1 queries={nq:,} k={k}", "train": "torch k-means (10 iters, 500k sample), "
                               "PQ k-means on 25k residuals"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": (achieved / hbm_peak) if achieved else None, "traffic": None,
                     "kernel": "adc_group_kernel (grouped ADC list scan)", "peak_source": f"{peak_kind} HBM copy",
                     "algorithmic_bytes_per_step": bytes_step, "per": "GPU",
                     "sharding": ("single GPU" if world == 1 else "index replicated, queries split across ranks"
                                  if split == "query" else
                                  "index replicated, (query, list) pairs dealt across ranks in four-pair groups"),
                     "breakdown_ms_per_step": {kk: v[0] / args.steps for kk, v in prof.items() if v[1]},
                     "per_rank": per_rank,
                     "smem_gather_roof": {"frac": smem_frac, "gather_bytes_per_step": gather_bytes,
                                          "peak_bytes_per_s": smem_peak,
                                          "peak_source": "nominal: 148 SMs x 128 B/clk x 1.965 GHz",
                                          "note": "conflict-free minimum of the 16-byte four-query table reads",
                                          "random_code_frac": random_frac,
                                          "random_code_note": "the same roof with the expected bank conflicts of "
                                                              "uniformly random codes (2.54 wavefronts per "
                                                              "quarter-warp read instead of 1)"}},
        "parity": par,
        "cpu_baseline": cpu,
        "e2e": e2e,
    }


SQ8 = dict(n=1_000_000, dim=768, comps=64, sigma=0.3, nq=10_000, k=100)
IVFFLAT = dict(n=1_000_000, dim=768, comps=256, sigma=0.3, nq=10_000, k=10, nlist=1024, nprobe=32, train=200_000)
BQ = dict(n=10_000_000, dim=1024, comps=256, sigma=0.5, nq=10_000, k=100)
FP16 = dict(n_per_gpu=12_500_000, dim=768, comps=4096, sigma=0.3, nq=4096, k=100)


def _timed_scan(args, world, dev, barrier, max_over_ranks, step, slot):
    """Warm-up, then K timed steps (CUDA events on the current stream, max over ranks) and the
    library's per-kernel time of `slot` per step."""
    import torch

    from vectors_b200 import _native as N

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    N.profile_reset()
    N.profile_enable(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    N.profile_enable(False)
    prof = N.profile_read()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    kms = max_over_ranks(prof[slot][0] / args.steps)
    return ms, kms, {kk: v[0] / args.steps for kk, v in prof.items() if v[1]}


def run_ivfflat(args, rank, world, local, dev, barrier, max_over_ranks, peak_kind):
    """IVF-flat (IvfIndex.search without PQ), 1M x 768 EUCLIDEAN, nlist 1024, nprobe 32, 10k
    queries, top-10: routing, then the exact list scan in the reference's batched fp32 order
    (CUDA cores: the scores must be the reference's to the bit).  The index is replicated; the
    queries (2 ranks) or the (query, list) pairs (4 and more) are split across ranks."""
    import torch

    import vectors_b200 as vx
    from vectors_b200.sharded import ivfflat_search_pair_split, search_query_sharded

    P = IVFFLAT
    n, dim, nlist, nq, k = args.ivfflat_n, P["dim"], P["nlist"], P["nq"], P["k"]
    cent_mix = centres(P["comps"], dim, SEED_C ^ 0x2E)
    rows = torch.from_numpy(gen_rows(0, n, dim, cent_mix, P["sigma"], SEED_DB ^ 0x2E, False)).to(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    sample = rows[torch.randperm(n, generator=g, device=dev)[: P["train"]]]
    cent = sample[:nlist].clone()
    for _ in range(10):
        a_ = nearest(sample, cent)
        s_ = torch.zeros_like(cent).index_add_(0, a_, sample)
        c_ = torch.bincount(a_, minlength=nlist)
        cent = torch.where(c_.unsqueeze(1) > 0, s_ / c_.clamp_min(1).unsqueeze(1).float(), cent)
    del sample
    assign = nearest(rows, cent)
    counts = torch.bincount(assign, minlength=nlist)
    order = torch.argsort(assign, stable=True).to(torch.int32)
    loff = torch.zeros(nlist + 1, dtype=torch.int64, device=dev)
    loff[1:] = torch.cumsum(counts, 0)
    a = vx.IvfFlatAdapter(nprobe=P["nprobe"], device=local)
    a.build_prebuilt(cent.cpu().numpy(), loff.cpu().numpy(), order.cpu().numpy(), rows, vx.SimilarityFunction.EUCLIDEAN)
    qh = gen_rows(0, nq, dim, cent_mix, P["sigma"], SEED_Q ^ 0x2E, False)
    q = torch.from_numpy(qh).to(dev)
    probed = torch.cdist(q, cent).topk(P["nprobe"], largest=False).indices
    pair_rows = float(counts[probed].sum().item())

    # auto: the split that measured faster at this rank count (one-GPU emulation of each rank's
    # own work at 2 / 4 / 8 ranks, and 2 B200s): queries at 2 ranks (1.66M against 1.64M queries/s
    # on 2 GPUs), from 4 the (query, list) pair split -- every rank scans an even share of every
    # list's pairs in full 64-query groups, the per-slot results meet in one sum all-reduce
    split = args.ivfflat_split if args.ivfflat_split != "auto" else ("query" if world <= 2 else "pair")

    def step():
        if world == 1:
            return a.ivf_search_device(q, k, P["nprobe"])[0]
        if split == "query":
            return search_query_sharded(lambda qs: a.ivf_search_device(qs, k, P["nprobe"]), q)[0]
        return ivfflat_search_pair_split(a, q, k, P["nprobe"])[0]

    ms, kms, br = _timed_scan(args, world, dev, barrier, max_over_ranks, step, "adc_scan")
    ops = 2.0 * pair_rows * dim / world  # subtract + fused multiply-add per (query, row, dim)
    achieved = ops / (kms / 1e3) / 1e12 if kms > 0 else None
    peak = 148 * 128 * 1.965e9 / 1e12  # fp32 lanes x max SM clock, as instructions
    cpu = par = e2e = None
    if rank == 0 and world == 1 and not args.no_cpu:  # the CPU baseline is a 1-GPU figure
        from oracle import oracle as O

        qs = qh[:64]
        cent_h, loff_h, ord_h, rows_h = cent.cpu().numpy(), loff.cpu().numpy(), order.cpu().numpy(), rows.cpu().numpy()
        radii = O.ivf_radii(cent_h, loff_h, ord_h, rows_h)  # BuoyIndex.computeRadii, as the index holds them
        ref, dt, th = timed_oracle(lambda t: O.ivfflat_search_full(cent_h, loff_h, ord_h, rows_h, radii, qs, 0, k,
                                                                   P["nprobe"], nthreads=t))
        par = parity(a.ivf_search_arrays(qs, k, P["nprobe"]), ref, True, n)
        cpu = {"value": len(qs) / dt, "unit": "queries/s", "cores": th, "kind": "port",
               "sample": f"{len(qs)} queries over the same index ({dt:.1f} s)"}
        qp = pinned(qh)
        e2e = e2e_host(args, lambda: a.ivf_search_arrays(qp, k, P["nprobe"]), nq, nq * dim * 4, nq * (k * 8 + 4))
    a.close()
    del rows
    torch.cuda.empty_cache()
    return {
        "value": nq / (ms / 1e3), "unit": "queries/s", "ms_per_step": ms,
        "config": {"workload": f"IVF-flat EUCLIDEAN n={n:,} dim={dim} nlist={nlist} nprobe={P['nprobe']} "
                               f"queries={nq:,} k={k}", "train": "torch k-means (10 iters, 200k sample)"},
        "roofline": {"bound": "fp32 CUDA cores (exact batched order)", "achieved": achieved, "peak": peak,
                     "unit": "T fp32 ops/s", "frac": (achieved / peak) if achieved else None, "traffic": None,
                     "kernel": "flat_list_kernel (IVF-flat list scan)", "per": "GPU",
                     "peak_source": "nominal: 148 SMs x 128 fp32 lanes x 1.965 GHz",
                     "pair_rows_per_step": pair_rows, "breakdown_ms_per_step": br,
                     "sharding": ("single GPU" if world == 1 else "index replicated, queries split across ranks"
                                  if split == "query" else
                                  "index replicated, (query, list) pairs dealt across ranks in 64-pair groups, "
                                  "per-slot results summed (NCCL all-reduce) and merged in route order")},
        "parity": par,
        "cpu_baseline": cpu,
        "e2e": e2e,
    }


def run_sq8(args, rank, world, local, dev, barrier, max_over_ranks, tc_sustained, peak_kind):
    """SQ8 DOT candidate scan, 1M x 768, 10k queries, k = 100: the int8 tcgen05 scan (exact
    int32 dot + the reference's score epilogue) over this rank's rows."""
    import torch

    import vectors_b200 as vx
    from vectors_b200.sharded import gather_and_merge

    P = SQ8
    n, dim, nq, k = args.sq8_n, P["dim"], P["nq"], P["k"]
    offs = vx.shard_offsets(n, world)
    lo, hi = offs[rank], offs[rank + 1]
    offs_dev = torch.tensor(offs[:world], dtype=torch.int64, device=dev)
    cent = centres(P["comps"], dim, SEED_C ^ 0x5A)
    x = torch.from_numpy(gen_rows(lo, hi - lo, dim, cent, P["sigma"], SEED_DB ^ 0x5A, True)).to(dev)
    # ScalarQuantizer encoding (global quantile pair, codes 0..127, per-row correction), as data
    # preparation on the device; the quantile pair comes from rank 0's first 25k rows
    qs = torch.quantile(x[:25_000].flatten()[:16_000_000], torch.tensor([0.005, 0.995], device=dev))
    if world > 1:
        import torch.distributed as dist

        dist.broadcast(qs, 0)
    mn, mx = float(qs[0]), float(qs[1])
    scale, alpha = 127.0 / (mx - mn), (mx - mn) / 127.0
    qc = torch.clamp(torch.round(scale * (torch.clamp(x, mn, mx) - mn)), 0, 127)
    corr = (mn * (x - mn / 2) + ((x - mn) - qc * alpha) * (qc * alpha)).sum(1)
    codes = qc.to(torch.int8).cpu().numpy()
    del x, qc
    torch.cuda.empty_cache()
    a = vx.QuantizedFlatScanAdapter(device=local)
    a.build_sq8(codes, corr.cpu().numpy(), mn, mx, vx.SimilarityFunction.DOT_PRODUCT)
    q = torch.from_numpy(gen_rows(0, nq, dim, cent, P["sigma"], SEED_Q ^ 0x5A, True)).to(dev)

    def step():
        ids, sc, cnt = a.scan_candidates_device(q, k)
        return ids if world == 1 else gather_and_merge(ids, sc, cnt, offs_dev, k)[0]

    ms, kms, br = _timed_scan(args, world, dev, barrier, max_over_ranks, step, "gemm_scan")
    par = cpu = e2e = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import oracle as O

        qh = q.cpu().numpy()
        corr_h = corr.cpu().numpy()
        ref, dt, th = timed_oracle(lambda t: O.sq8_search(codes, corr_h, mn, mx, qh[:64], O.DOT_PRODUCT, k,
                                                          O.CANONICAL, t))
        par = parity(a.scan_candidates_arrays(qh[:64], k), ref, True, n)
        cpu = {"value": 64 / dt, "unit": "queries/s", "cores": th, "kind": "port",
               "sample": f"64 queries over the same {n:,}-row index ({dt:.1f} s)"}
        qp = pinned(qh)
        e2e = e2e_host(args, lambda: a.scan_candidates_arrays(qp, k), nq, nq * dim * 4, nq * (k * 8 + 4))
    a.close()
    ops = 2.0 * nq * (hi - lo) * dim  # int8 multiply-adds x 2 on this rank
    achieved = ops / (kms / 1e3) / 1e12 if kms > 0 else None
    peak = 2.0 * tc_sustained
    return {
        "value": nq / (ms / 1e3), "unit": "queries/s", "ms_per_step": ms,
        "config": {"workload": f"SQ8 DOT candidate scan n={n:,} dim={dim} queries={nq:,} k={k}",
                   "encoding": "ScalarQuantizer global quantile pair, codes 0..127 (the reference's SQ8)"},
        "roofline": {"bound": "tensor (int8)", "achieved": achieved, "peak": peak, "unit": "TOP/s",
                     "frac": (achieved / peak) if achieved else None, "traffic": None,
                     "kernel": "gemm_scan_kernel (tcgen05 kind::i8, fused top-K)", "per": "GPU",
                     "peak_source": f"2 x {peak_kind} dense bf16 sustained (int8 MMA runs at twice the bf16 rate)",
                     "breakdown_ms_per_step": br},
        "parity": par,
        "cpu_baseline": cpu,
        "e2e": e2e,
    }


def run_bq(args, rank, world, local, dev, barrier, max_over_ranks, tc_sustained, peak_kind):
    """BQ (sign-bit) Hamming candidate scan, 10M x 1024 bits, 10k queries, k = 100."""
    import torch

    import vectors_b200 as vx
    from vectors_b200.sharded import gather_and_merge

    P = BQ
    n, dim, nq, k = args.bq_n, P["dim"], P["nq"], P["k"]
    offs = vx.shard_offsets(n, world)
    lo, hi = offs[rank], offs[rank + 1]
    offs_dev = torch.tensor(offs[:world], dtype=torch.int64, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0xB0 + 0)  # the same centres on every rank
    cent = torch.randn((P["comps"], dim), generator=g, device=dev)
    weights = (1 << torch.arange(64, device=dev, dtype=torch.int64))

    def pack(x):  # BinaryQuantizer.packBits + bytesToLongs: bit j of word w = x[64w + j] >= 0
        b = (x >= 0).view(x.shape[0], dim // 64, 64).to(torch.int64)
        return (b * weights).sum(2)

    words = torch.empty((hi - lo, dim // 64), dtype=torch.int64, device=dev)
    # BBQ on this rank's first rows: centroid-relative bits and (|v - c|^2, vl, width)
    nb = min(hi - lo, args.bbq_n)
    bbq_c = cent.mean(0)
    bbq_words = torch.empty((nb, dim // 64), dtype=torch.int64, device=dev)
    bbq_corr = torch.empty((nb, 3), dtype=torch.float32, device=dev)
    for s0 in range(lo, hi, 1 << 18):
        s1 = min(hi, s0 + (1 << 18))
        gc = torch.Generator(device=dev)
        gc.manual_seed(0xB1 * 1_000_003 + s0)  # chunk-seeded: identical however rows are split
        comp = torch.randint(0, P["comps"], (s1 - s0,), generator=gc, device=dev)
        x = cent[comp] + P["sigma"] * torch.randn((s1 - s0, dim), generator=gc, device=dev)
        words[s0 - lo: s1 - lo] = pack(x)
        if s0 - lo < nb:
            e = min(s1 - lo, nb) - (s0 - lo)
            xc = x[:e] - bbq_c
            bbq_words[s0 - lo: s0 - lo + e] = pack(xc)
            bbq_corr[s0 - lo: s0 - lo + e, 0] = (xc * xc).sum(1)
            bbq_corr[s0 - lo: s0 - lo + e, 1] = xc.min(1).values
            bbq_corr[s0 - lo: s0 - lo + e, 2] = xc.max(1).values - xc.min(1).values
    gq = torch.Generator(device=dev)
    gq.manual_seed(0xB2)
    comp = torch.randint(0, P["comps"], (nq,), generator=gq, device=dev)
    q = cent[comp] + P["sigma"] * torch.randn((nq, dim), generator=gq, device=dev)
    a = vx.QuantizedFlatScanAdapter(device=local)
    words_h = words.cpu().numpy().view(np.uint64)
    a.build_bq(words_h, dim, vx.SimilarityFunction.DOT_PRODUCT)
    del words
    torch.cuda.empty_cache()
    check = rank == 0 and world == 1 and not args.no_cpu
    qh = q.cpu().numpy()

    def step():
        ids, sc, cnt = a.scan_candidates_device(q, k)
        return ids if world == 1 else gather_and_merge(ids, sc, cnt, offs_dev, k)[0]

    ms, kms, br = _timed_scan(args, world, dev, barrier, max_over_ranks, step, "gemm_scan")
    par = cpu = e2e = None
    if check:
        from oracle import oracle as O

        ref, dt, th = timed_oracle(lambda t: O.bq_search(words_h, dim, qh[:64], O.DOT_PRODUCT, k, O.CANONICAL, t))
        par = parity(a.scan_candidates_arrays(qh[:64], k), ref, True, n)
        cpu = {"value": 64 / dt, "unit": "queries/s", "cores": th, "kind": "port",
               "sample": f"64 queries over the same {n:,}-row index ({dt:.1f} s)"}
        qp = pinned(qh)
        e2e = e2e_host(args, lambda: a.scan_candidates_arrays(qp, k), nq, nq * dim * 4, nq * (k * 8 + 4))
    a.close()
    # The same rows as an index above the int8 operand budget: packed bits alone on the device
    # (128 B per row instead of 1,152), the tensor scan over row windows whose +-1 operand is
    # expanded at search time (VX_BQ_WINDOW_BYTES, default 4 GiB: 4,194,304 rows per window).
    saved = os.environ.get("VX_BQ_TENSOR_BYTES")
    os.environ["VX_BQ_TENSOR_BYTES"] = "0"
    try:
        aw = vx.QuantizedFlatScanAdapter(device=local)
        aw.build_bq(words_h, dim, vx.SimilarityFunction.DOT_PRODUCT)
    finally:
        if saved is None:
            del os.environ["VX_BQ_TENSOR_BYTES"]
        else:
            os.environ["VX_BQ_TENSOR_BYTES"] = saved

    def wstep():
        ids, sc, cnt = aw.scan_candidates_device(q, k)
        return ids if world == 1 else gather_and_merge(ids, sc, cnt, offs_dev, k)[0]

    wms, wkms, wbr = _timed_scan(args, world, dev, barrier, max_over_ranks, wstep, "gemm_scan")
    wpar = parity(aw.scan_candidates_arrays(qh[:64], k), ref, True, n) if check else None
    aw.close()
    del words_h
    rows = hi - lo
    dp8w = (dim + 127) // 128 * 128
    wach = 2.0 * nq * rows * dp8w / (wkms / 1e3) / 1e12 if wkms > 0 else None
    windowed = {"value": nq / (wms / 1e3), "unit": "queries/s", "ms_per_step": wms,
                "config": {"index_bytes_per_row": dim // 8, "window_bytes": 4 << 30,
                           "note": "index above the int8 operand budget (VX_BQ_TENSOR_BYTES=0): bits only, "
                                   "+-1 operand expanded per row window at search time"},
                "roofline": {"bound": "tensor (int8)", "achieved": wach, "peak": 2.0 * tc_sustained, "unit": "TOP/s",
                             "frac": (wach / (2.0 * tc_sustained)) if wach else None,
                             "kernel": "gemm_scan_kernel per row window (+ the window's bit expansion)",
                             "breakdown_ms_per_step": wbr},
                "parity": wpar}
    if br.get("gemm_scan"):
        # tensor-core path: +-1 int8 operands, dot = D - 2h, exact int32 (2 ops per bit pair)
        dp8 = (dim + 127) // 128 * 128
        achieved = 2.0 * nq * rows * dp8 / (kms / 1e3) / 1e12 if kms > 0 else None
        peak = 2.0 * tc_sustained
        roof = {"bound": "tensor (int8)", "achieved": achieved, "peak": peak, "unit": "TOP/s",
                "frac": (achieved / peak) if achieved else None,
                "kernel": "gemm_scan_kernel (tcgen05 kind::i8 on +-1 expanded bits, Hamming epilogue)",
                "peak_source": f"2 x {peak_kind} dense bf16 sustained (int8 MMA runs at twice the bf16 rate)"}
    else:
        # popcount path (VX_BQ_TENSOR_BYTES below the operand size): XOR + popc + add per word
        bms = br.get("bq_scan", 0.0)
        achieved = nq * rows * (dim // 64) / (bms / 1e3) / 1e12 if bms > 0 else None
        roof = {"bound": "integer pipe (xor + popc)", "achieved": achieved, "unit": "T word-compares/s",
                "peak": None, "frac": None, "kernel": "bq_scan_kernel"}
    roof.update({"per": "GPU", "traffic": None, "breakdown_ms_per_step": br})
    # BBQ (BinaryMode.BBQ): 4-bit queries against the centroid-relative sign bits; rawAsymDot on
    # the int8 tensor cores (0/1 rows x 4-bit codes), or the popcount kernel without the operand
    b = vx.QuantizedFlatScanAdapter(device=local)
    bw_h, bc_h, bcent_h = bbq_words.cpu().numpy().view(np.uint64), bbq_corr.cpu().numpy(), bbq_c.cpu().numpy()
    b.build_bbq(bw_h, bc_h, bcent_h, dim, vx.SimilarityFunction.DOT_PRODUCT)
    del bbq_words, bbq_corr

    def bstep():
        ids, sc, cnt = b.scan_candidates_device(q, k)
        return ids if world == 1 else gather_and_merge(ids, sc, cnt, offs_dev, k)[0]

    bms_step, bkms, bbr = _timed_scan(args, world, dev, barrier, max_over_ranks, bstep, "gemm_scan")
    bpar = bcpu = be2e = None
    if check:
        from oracle import oracle as O

        ref, dt, th = timed_oracle(lambda t: O.bbq_search(bw_h, bc_h, bcent_h, dim, qh[:64], O.DOT_PRODUCT, k,
                                                          O.CANONICAL, t))
        bpar = parity(b.scan_candidates_arrays(qh[:64], k), ref, True, nb)
        bcpu = {"value": 64 / dt, "unit": "queries/s", "cores": th, "kind": "port",
                "sample": f"64 queries over the same {nb:,}-row index ({dt:.1f} s)"}
        qp = pinned(qh)
        be2e = e2e_host(args, lambda: b.scan_candidates_arrays(qp, k), nq, nq * dim * 4, nq * (k * 8 + 4))
    b.close()
    if bbr.get("gemm_scan"):
        dp8 = (dim + 127) // 128 * 128
        bach = 2.0 * nq * nb * dp8 / (bkms / 1e3) / 1e12 if bkms > 0 else None
        bpeak = 2.0 * tc_sustained
        broof = {"bound": "tensor (int8)", "achieved": bach, "peak": bpeak, "unit": "TOP/s",
                 "frac": (bach / bpeak) if bach else None,
                 "kernel": "gemm_scan_kernel (tcgen05 kind::i8 on 0/1 bits x 4-bit codes, BBQ epilogue)",
                 "peak_source": f"2 x {peak_kind} dense bf16 sustained (int8 MMA runs at twice the bf16 rate)"}
    else:
        bkms = bbr.get("bq_scan", 0.0)
        bwork = 4.0 * nq * nb * (dim // 64)  # AND + popcount of a 64-bit word per plane
        bach = bwork / (bkms / 1e3) / 1e12 if bkms > 0 else None
        broof = {"bound": "integer pipe (and + popc)", "achieved": bach, "unit": "T word-plane ops/s",
                 "peak": None, "frac": None, "kernel": "bbq_scan_kernel"}
    broof.update({"per": "GPU", "breakdown_ms_per_step": bbr})
    bbq = {"value": nq / (bms_step / 1e3), "unit": "queries/s", "ms_per_step": bms_step,
           "config": {"workload": f"BBQ candidate scan n={nb * world:,} x {dim} bits (4-bit queries) "
                                  f"queries={nq:,} k={k}"},
           "roofline": broof, "parity": bpar, "cpu_baseline": bcpu, "e2e": be2e}
    return {
        "value": nq / (ms / 1e3), "unit": "queries/s", "ms_per_step": ms,
        "config": {"workload": f"BQ sign-bit Hamming candidate scan n={n:,} x {dim} bits queries={nq:,} k={k}"},
        "roofline": roof,
        "parity": par,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "windowed": windowed,
        "bbq": bbq,
    }


def run_fp16(args, rank, world, local, dev, barrier, max_over_ranks, tc_sustained, peak_kind):
    """FP16 DOT candidate scan at the 100M x 768 configuration's per-GPU share: 12.5M stored
    binary16 rows per GPU (100M at 8 GPUs), 4,096 fp32 queries, k = 100; per-GPU top-k merged.
    Rows are generated on the device (4,096-component mixture, L2-normalised, rounded to fp16)."""
    import torch

    import vectors_b200 as vx
    from vectors_b200.sharded import gather_and_merge

    P = FP16
    per, dim, nq, k = args.fp16_n, P["dim"], P["nq"], P["k"]
    offs = [per * r for r in range(world + 1)]
    offs_dev = torch.tensor(offs[:world], dtype=torch.int64, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0xF16)  # the same centres on every rank
    cent = torch.randn((P["comps"], dim), generator=g, device=dev)
    rows = torch.empty((per, dim), dtype=torch.float16, device=dev)
    for s0 in range(0, per, 1 << 20):
        s1 = min(per, s0 + (1 << 20))
        gc = torch.Generator(device=dev)
        gc.manual_seed(0xF17 * 1_000_003 + offs[rank] + s0)
        comp = torch.randint(0, P["comps"], (s1 - s0,), generator=gc, device=dev)
        x = cent[comp] + P["sigma"] * torch.randn((s1 - s0, dim), generator=gc, device=dev)
        rows[s0:s1] = (x / x.norm(dim=1, keepdim=True)).half()
    gq = torch.Generator(device=dev)
    gq.manual_seed(0xF18)
    comp = torch.randint(0, P["comps"], (nq,), generator=gq, device=dev)
    q = cent[comp] + P["sigma"] * torch.randn((nq, dim), generator=gq, device=dev)
    q = q / q.norm(dim=1, keepdim=True)
    a = vx.QuantizedFlatScanAdapter(device=local)
    a.build_fp16(rows, vx.SimilarityFunction.DOT_PRODUCT)
    check = rank == 0 and world == 1 and not args.no_cpu
    sub_h = rows[: min(per, 1_000_000)].cpu().numpy().view(np.uint16) if check else None
    del rows, cent
    torch.cuda.empty_cache()

    def step():
        ids, sc, cnt = a.scan_candidates_device(q, k)
        return ids if world == 1 else gather_and_merge(ids, sc, cnt, offs_dev, k)[0]

    ms, kms, br = _timed_scan(args, world, dev, barrier, max_over_ranks, step, "gemm_scan")
    par = cpu = e2e = None
    if check:
        from oracle import oracle as O

        qh = q.cpu().numpy()
        qp = pinned(qh)
        e2e = e2e_host(args, lambda: a.scan_candidates_arrays(qp, k), nq, nq * dim * 4, nq * (k * 8 + 4))
        a.close()
        # parity on an index of this GPU's first 1M rows (the CPU check of 12.5M rows would take minutes)
        sub = vx.QuantizedFlatScanAdapter(device=local)
        sub.build_fp16(sub_h, vx.SimilarityFunction.DOT_PRODUCT)
        got = sub.scan_candidates_arrays(qh[:64], k)
        sub.close()
        ref, dt, th = timed_oracle(lambda t: O.fp16_search(sub_h, qh[:64], O.DOT_PRODUCT, k, O.CANONICAL, t))
        par = parity(got, ref, False, len(sub_h))
        cpu = {"value": 64 / dt * (len(sub_h) / per), "unit": "queries/s", "cores": th, "kind": "port",
               "sample": f"64 queries x {len(sub_h):,} rows ({dt:.1f} s); QPS scaled by rows/{per:,}"}
    else:
        a.close()
    flops = 2.0 * nq * per * dim
    achieved = flops / (kms / 1e3) / 1e12 if kms > 0 else None
    return {
        "value": nq / (ms / 1e3), "unit": "queries/s", "ms_per_step": ms, "scaling": "weak",
        "config": {"workload": f"FP16 DOT candidate scan, {per:,} x {dim} binary16 rows per GPU "
                               f"({per * world:,} in total), {nq:,} fp32 queries, k={k}",
                   "queries": "fp32, as Fp16QuantizedVectors scores them (fp16 operand pass + exact re-score)"},
        "roofline": {"bound": "tensor (fp16)", "achieved": achieved, "peak": tc_sustained, "unit": "TFLOP/s",
                     "frac": (achieved / tc_sustained) if achieved else None, "traffic": None, "per": "GPU",
                     "kernel": "gemm_scan_kernel (tcgen05 kind::f16, fused top-K)",
                     "peak_source": f"{peak_kind} dense bf16/fp16 sustained", "breakdown_ms_per_step": br},
        "parity": par,
        "cpu_baseline": cpu,
        "e2e": e2e,
    }


def nearest(x, c, chunk=131072):
    import torch

    out = torch.empty(len(x), dtype=torch.int64, device=x.device)
    cn = (c * c).sum(1)
    for s in range(0, len(x), chunk):
        xs = x[s: s + chunk]
        d = cn.unsqueeze(0) - 2.0 * (xs @ c.T)
        out[s: s + chunk] = d.argmin(1)
    return out


def pq_kmeans(resid, ks, g, iters=10):
    """Batched k-means over subspaces: resid [m, npts, sub] -> codebooks [m, ks, sub]."""
    import torch

    m, npts, sub = resid.shape
    books = resid[:, torch.randperm(npts, generator=g, device=resid.device)[:ks]].clone()
    for _ in range(iters):
        a = torch.cdist(resid, books).argmin(2)  # [m, npts]
        for j in range(m):
            s = torch.zeros_like(books[j]).index_add_(0, a[j], resid[j])
            cnt = torch.bincount(a[j], minlength=ks).unsqueeze(1)
            books[j] = torch.where(cnt > 0, s / cnt.clamp_min(1).float(), books[j])
    return books


if __name__ == "__main__":
    sys.exit(main())
