"""numpy front end of the CPU oracle (liboracle.so, vx_oracle.cpp).

TEST INFRASTRUCTURE ONLY: used by tests/, the smoke check and the CPU-baseline leg of
bench.py to check and time the CUDA path.  The product never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")

EUCLIDEAN, DOT_PRODUCT, COSINE, MAXIMUM_INNER_PRODUCT = 0, 1, 2, 3
REFERENCE_HEAP, CANONICAL = 0, 1

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        h = _lib
        f32, i32, i64, u64, p = C.c_float, C.c_int32, C.c_int64, C.c_uint64, C.c_void_p
        sig = {
            "vo_dot": (f32, [p, p, i32]),
            "vo_square_distance": (f32, [p, p, i32]),
            "vo_cosine": (f32, [p, p, i32]),
            "vo_compare": (f32, [i32, p, p, i32]),
            "vo_scale_mip": (f32, [f32]),
            "vo_l2normalize": (None, [p, i32]),
            "vo_byte_dot": (i32, [p, p, i32]),
            "vo_byte_square_distance": (i32, [p, p, i32]),
            "vo_hamming": (i32, [p, p, i32]),
            "vo_mat_vec_square_l2": (None, [p, p, i32, i32, p]),
            "vo_mat_vec_dot": (None, [p, p, i32, i32, p]),
            "vo_jrandom_init": (None, [p, i64]),
            "vo_jrandom_next_int": (i32, [p]),
            "vo_jrandom_next_int_bound": (i32, [p, i32]),
            "vo_jrandom_next_long": (i64, [p]),
            "vo_jrandom_next_float": (f32, [p]),
            "vo_jrandom_next_double": (C.c_double, [p]),
            "vo_jrandom_next_bytes": (None, [p, p, i32]),
            "vo_splitmix64_at": (u64, [u64, u64]),
            "vo_uniform_at": (C.c_double, [u64, u64]),
            "vo_normal_at": (C.c_double, [u64, u64]),
            "vo_gen_mixture": (None, [p, i64, i64, i32, i32, f32, u64, u64, i32, i32]),
            "vo_sq8_train": (None, [p, i64, i32, f32, p, p]),
            "vo_sq8_encode": (f32, [f32, f32, p, i32, p]),
            "vo_sq8_score": (f32, [i32, f32, f32, p, f32, p, f32, i32]),
            "vo_bq_encode": (None, [p, i32, p]),
            "vo_bq_score": (f32, [i32, i32, i32]),
            "vo_f32_to_f16": (C.c_uint16, [f32]),
            "vo_f16_to_f32": (f32, [C.c_uint16]),
            "vo_pq_subspaces": (None, [i32, i32, p]),
            "vo_pq_train": (None, [p, i64, i32, i32, i32, p]),
            "vo_pq_encode": (None, [p, i32, i32, i32, p, p]),
            "vo_pq_adc_table": (None, [p, i32, i32, i32, p, i32, p]),
            "vo_kmeans_train": (None, [p, i64, i32, i32, i32, i64, p, i32]),
            "vo_kmeans_assign": (None, [p, i64, i32, p, i32, p, i32]),
            "vo_sq8_encode_all": (None, [f32, f32, p, i64, i32, p, p, i32]),
            "vo_bq_encode_all": (None, [p, i64, i32, p, i32]),
            "vo_fp16_encode_all": (None, [p, i64, i32, p, i32]),
            "vo_pq_encode_all": (None, [p, i64, i32, i32, i32, p, p, i32]),
            "vo_flat_search": (None, [p, i64, i32, i32, p, i32, i32, i32, i32, p, p, p]),
            "vo_sq8_search": (None, [p, p, i64, i32, f32, f32, i32, p, i32, i32, i32, i32, p, p, p]),
            "vo_sq_search": (None, [p, p, i64, i32, f32, f32, i32, i32, p, i32, i32, i32, i32, p, p, p]),
            "vo_sq_encode_all": (None, [f32, f32, i32, p, i64, i32, p, p, i32]),
            "vo_bbq_encode_all": (None, [p, p, i64, i32, p, p, i32]),
            "vo_bbq_search": (None, [p, p, p, i64, i32, i32, p, i32, i32, i32, i32, p, p, p]),
            "vo_bq_search": (None, [p, i64, i32, i32, p, i32, i32, i32, i32, p, p, p]),
            "vo_fp16_search": (None, [p, i64, i32, i32, p, i32, i32, i32, i32, p, p, p]),
            "vo_quantized_two_pass_search": (None, [i32, p, p, f32, f32, p, i64, i32, i32, p, i32, i32, f32, i32, i32, p, p, p]),
            "vo_pq_flat_search": (None, [p, p, p, i64, i32, i32, i32, i32, p, i32, i32, i32, i32, p, p, p]),
            "vo_rescore_candidates": (None, [p, i32, i32, p, i32, p, i32, p, i32, i32, i32, p, p, p]),
            "vo_route": (None, [p, i32, i32, i32, p, i32, i32, i32, i32, p, p]),
            "vo_ivfpq_search": (None, [p, i32, i32, p, p, i32, i32, p, p, i64, i32, p, i32, i32, i32, i32, p, i32, i32, p, p, p]),
            "vo_ivfflat_search": (None, [p, i32, i32, p, p, p, i64, i32, p, i32, i32, i32, i32, i32, p, p, p]),
            "vo_ivfpq_search_spill": (None, [p, i32, i32, p, p, i32, i32, p, p, i64, i32, p, i32, i32, i32, f32, p, i32, p, i32, p, p, p]),
            "vo_ivfflat_search_spill": (None, [p, i32, i32, p, p, p, i32, p, p, i32, i32, i32, f32, p, p, p, i32, p, p, p]),
            "vo_ivfflat_search_early_exit": (None, [p, i32, i32, p, p, p, i64, i32, p, p, i32, i32, i32, i32, i32, p, p,
                                                    p]),
            "vo_ivf_radii": (None, [p, i32, i32, p, p, p, p]),
            "vo_route_spill": (None, [p, i32, i32, i32, p, i32, i32, f32, p, i32, p, p, p]),
            "vo_merge_shards": (None, [i32, p, p, p, p, i32, i32, i32, i32, p, p, p]),
            "vo_topk_select": (i32, [p, i32, i32, p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def P(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def threads() -> int:
    return max(1, os.cpu_count() or 1)


class JavaRandom:
    """java.util.Random (published LCG), for reproducing the reference tests' inputs."""

    class _S(C.Structure):
        _fields_ = [("seed", C.c_uint64), ("nng", C.c_double), ("have", C.c_int32)]

    def __init__(self, seed: int):
        self.s = JavaRandom._S()
        lib().vo_jrandom_init(C.byref(self.s), seed)

    def next_int(self, bound=None) -> int:
        if bound is None:
            return lib().vo_jrandom_next_int(C.byref(self.s))
        return lib().vo_jrandom_next_int_bound(C.byref(self.s), bound)

    def next_long(self) -> int:
        return lib().vo_jrandom_next_long(C.byref(self.s))

    def next_float(self) -> float:
        return lib().vo_jrandom_next_float(C.byref(self.s))

    def next_double(self) -> float:
        return lib().vo_jrandom_next_double(C.byref(self.s))

    def next_bytes(self, n: int) -> np.ndarray:
        out = np.zeros(n, np.int8)
        lib().vo_jrandom_next_bytes(C.byref(self.s), P(out), n)
        return out


# ------------------------------------------------------------------ data
def gen_mixture(n, dim, n_centres, sigma, seed_centres, seed_points, normalize, first_row=0, nthreads=None):
    out = np.empty((n, dim), np.float32)
    lib().vo_gen_mixture(P(out), first_row, n, dim, n_centres, sigma, seed_centres, seed_points,
                         1 if normalize else 0, nthreads or threads())
    return out


# ------------------------------------------------------------------ kernels
def dot(a, b):
    a, b = f32(a), f32(b)
    return lib().vo_dot(P(a), P(b), a.shape[0])


def square_distance(a, b):
    a, b = f32(a), f32(b)
    return lib().vo_square_distance(P(a), P(b), a.shape[0])


def cosine(a, b):
    a, b = f32(a), f32(b)
    return lib().vo_cosine(P(a), P(b), a.shape[0])


def compare(metric, a, b):
    a, b = f32(a), f32(b)
    return lib().vo_compare(metric, P(a), P(b), a.shape[0])


def l2normalize(v):
    v = f32(v).copy()
    lib().vo_l2normalize(P(v), v.shape[0])
    return v


def byte_dot(a, b):
    a, b = np.ascontiguousarray(a, np.int8), np.ascontiguousarray(b, np.int8)
    return lib().vo_byte_dot(P(a), P(b), a.shape[0])


def byte_square_distance(a, b):
    a, b = np.ascontiguousarray(a, np.int8), np.ascontiguousarray(b, np.int8)
    return lib().vo_byte_square_distance(P(a), P(b), a.shape[0])


def hamming(a, b):
    a, b = np.ascontiguousarray(a, np.uint64), np.ascontiguousarray(b, np.uint64)
    return lib().vo_hamming(P(a), P(b), a.shape[0])


# ------------------------------------------------------------------ quantizers
def sq8_train(data, ci=0.99):
    d = f32(data)
    lo, hi = C.c_float(), C.c_float()
    lib().vo_sq8_train(P(d), d.shape[0], d.shape[1], ci, C.byref(lo), C.byref(hi))
    return lo.value, hi.value


def sq8_encode_all(min_q, max_q, data):
    d = f32(data)
    codes = np.empty(d.shape, np.int8)
    corr = np.empty(d.shape[0], np.float32)
    lib().vo_sq8_encode_all(min_q, max_q, P(d), d.shape[0], d.shape[1], P(codes), P(corr), threads())
    return codes, corr


def bq_encode_all(data):
    d = f32(data)
    words = np.empty((d.shape[0], (d.shape[1] + 63) // 64), np.uint64)
    lib().vo_bq_encode_all(P(d), d.shape[0], d.shape[1], P(words), threads())
    return words


def bq_score(metric, h, dim):
    return lib().vo_bq_score(metric, h, dim)


def fp16_encode_all(data):
    d = f32(data)
    codes = np.empty(d.shape, np.uint16)
    lib().vo_fp16_encode_all(P(d), d.shape[0], d.shape[1], P(codes), threads())
    return codes


def pq_subspaces(dim, m):
    so = np.empty((m, 2), np.int32)
    lib().vo_pq_subspaces(dim, m, P(so))
    return so


def pq_codebook_size(dim, m, ks):
    return int(pq_subspaces(dim, m)[:, 0].sum()) * ks


def pq_train(data, m, ks):
    d = f32(data)
    cb = np.empty(pq_codebook_size(d.shape[1], m, ks), np.float32)
    lib().vo_pq_train(P(d), d.shape[0], d.shape[1], m, ks, P(cb))
    return cb


def pq_encode_all(data, m, ks, codebooks):
    d = f32(data)
    codes = np.empty((d.shape[0], m), np.uint8)
    lib().vo_pq_encode_all(P(d), d.shape[0], d.shape[1], m, ks, P(f32(codebooks)), P(codes), threads())
    return codes


def pq_adc_table(q, m, ks, codebooks, use_dot=False):
    q = f32(q)
    t = np.empty((m, ks), np.float32)
    lib().vo_pq_adc_table(P(q), q.shape[0], m, ks, P(f32(codebooks)), 1 if use_dot else 0, P(t))
    return t


def kmeans_train(data, k, max_iter, seed, nthreads=None):
    d = f32(data)
    cent = np.empty((k, d.shape[1]), np.float32)
    lib().vo_kmeans_train(P(d), d.shape[0], d.shape[1], k, max_iter, seed, P(cent), nthreads or threads())
    return cent


def kmeans_assign(data, cent, nthreads=None):
    d, c = f32(data), f32(cent)
    out = np.empty(d.shape[0], np.int32)
    lib().vo_kmeans_assign(P(d), d.shape[0], d.shape[1], P(c), c.shape[0], P(out), nthreads or threads())
    return out


# ------------------------------------------------------------------ searches
def _outs(nq, k):
    return np.full((nq, k), -1, np.int32), np.zeros((nq, k), np.float32), np.zeros(nq, np.int32)


def flat_search(db, queries, metric, k, policy=CANONICAL, nthreads=None):
    db, q = f32(db), f32(queries)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_flat_search(P(db), db.shape[0], q.shape[1], metric, P(q), q.shape[0], k, policy,
                         nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def sq4_encode_all(min_q, max_q, data):
    """ScalarQuantizer INT4 encode (ScalarQuantizer.java:285-301): packed [n][ceil(dim/2)] codes,
    low nibble = even dimension, and the per-row corrections."""
    d = f32(data)
    n, dim = d.shape
    codes = np.empty(d.shape, np.int8)
    corr = np.empty(n, np.float32)
    lib().vo_sq_encode_all(min_q, max_q, 15, P(d), n, dim, P(codes), P(corr), threads())
    return sq4_pack(codes), corr


def sq4_pack(codes):
    c = np.asarray(codes, np.uint8)
    n, dim = c.shape
    out = np.zeros((n, (dim + 1) // 2), np.uint8)
    out[:, :] = c[:, 0::2] & 0x0F
    out[:, : dim // 2] |= (c[:, 1::2] & 0x0F) << 4
    return out


def sq4_unpack(packed, dim):
    """unpackInt4 (ScalarQuantizer.java:330-336)."""
    p = np.asarray(packed, np.uint8)
    out = np.empty((p.shape[0], dim), np.int8)
    out[:, 0::2] = (p & 0x0F)[:, : (dim + 1) // 2]
    out[:, 1::2] = ((p >> 4) & 0x0F)[:, : dim // 2]
    return out


def sq4_search(packed, corr, dim, min_q, max_q, queries, metric, k, policy=CANONICAL, nthreads=None):
    codes = np.ascontiguousarray(sq4_unpack(packed, dim))
    corr = f32(corr)
    q = f32(queries)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_sq_search(P(codes), P(corr), codes.shape[0], dim, min_q, max_q, 15, metric, P(q), q.shape[0], k, policy,
                       nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def bbq_encode_all(data, centroid):
    """BinaryQuantizer BBQ encode given the centroid: words [n][ceil(dim/64)], corrections [n][3]."""
    d, c = f32(data), f32(centroid)
    n, dim = d.shape
    words = np.empty((n, (dim + 63) // 64), np.uint64)
    corr = np.empty((n, 3), np.float32)
    lib().vo_bbq_encode_all(P(d), P(c), n, dim, P(words), P(corr), threads())
    return words, corr


def bbq_search(words, corr, centroid, dim, queries, metric, k, policy=CANONICAL, nthreads=None):
    words = np.ascontiguousarray(words, np.uint64)
    corr, c, q = f32(corr), f32(centroid), f32(queries)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_bbq_search(P(words), P(corr), P(c), words.shape[0], dim, metric, P(q), q.shape[0], k, policy,
                        nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def sq8_search(codes, corr, min_q, max_q, queries, metric, k, policy=CANONICAL, nthreads=None):
    codes = np.ascontiguousarray(codes, np.int8)
    corr = f32(corr)
    q = f32(queries)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_sq8_search(P(codes), P(corr), codes.shape[0], codes.shape[1], min_q, max_q, metric, P(q), q.shape[0], k,
                        policy, nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def bq_search(words, dim, queries, metric, k, policy=CANONICAL, nthreads=None):
    words = np.ascontiguousarray(words, np.uint64)
    q = f32(queries)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_bq_search(P(words), words.shape[0], dim, metric, P(q), q.shape[0], k, policy, nthreads or threads(),
                       P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def fp16_search(codes, queries, metric, k, policy=CANONICAL, nthreads=None):
    codes = np.ascontiguousarray(codes, np.uint16)
    q = f32(queries)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_fp16_search(P(codes), codes.shape[0], codes.shape[1], metric, P(q), q.shape[0], k, policy,
                         nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def quantized_two_pass(kind, qdata, qcorr, min_q, max_q, db, queries, metric, k, oqf, policy=CANONICAL, nthreads=None):
    db, q = f32(db), f32(queries)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_quantized_two_pass_search(kind, P(qdata), P(None if qcorr is None else f32(qcorr)), min_q, max_q, P(db),
                                       db.shape[0], db.shape[1], metric, P(q), q.shape[0], k, oqf, policy,
                                       nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def pq_flat_search(codebooks, codes, dim, m, ks, queries, metric, k, global_centroid=None, policy=CANONICAL,
                   nthreads=None):
    """QuantizedFlatScanAdapter over PQVectors: the k best rows by PQVectors' ADC score."""
    q = f32(queries)
    codes = np.ascontiguousarray(codes, np.uint8)
    gc = None if global_centroid is None else f32(global_centroid)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_pq_flat_search(P(f32(codebooks)), P(gc), P(codes), codes.shape[0], dim, m, ks, metric, P(q), q.shape[0], k,
                            policy, nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def rescore_candidates(db, queries, metric, cand_ids, cand_counts, k, policy=CANONICAL, nthreads=None):
    """The two-pass search's exact second pass over given candidates (e.g. an SQ4 or BBQ scan's)."""
    db, q = f32(db), f32(queries)
    cid = np.ascontiguousarray(cand_ids, np.int32)
    cc = np.ascontiguousarray(cand_counts, np.int32)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_rescore_candidates(P(db), q.shape[1], metric, P(q), q.shape[0], P(cid), cid.shape[1], P(cc), k, policy,
                                nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def candidate_k(k, oqf):
    """QuantizedFlatScanAdapter's candidateK = max(k, ceil(k * overQueryFactor)) (float product)."""
    return max(k, int(np.ceil(np.float64(np.float32(k) * np.float32(oqf)))))


def route(centroids, queries, metric, nprobe, policy=CANONICAL, nthreads=None):
    c, q = f32(centroids), f32(queries)
    lids = np.empty((q.shape[0], nprobe), np.int32)
    dists = np.empty((q.shape[0], nprobe), np.float32)
    lib().vo_route(P(c), c.shape[0], c.shape[1], metric, P(q), q.shape[0], nprobe, policy, nthreads or threads(),
                   P(lids), P(dists))
    return lids, dists


def route_spill(centroids, queries, metric, nprobe, gamma, spill_targets, nthreads=None):
    """routeWithSpillDistances with SOAR spill: per query the lists (primaries ascending, then
    spill targets) and their distances, trimmed to each query's count."""
    c, q = f32(centroids), f32(queries)
    sp = np.ascontiguousarray(spill_targets, np.int32)
    lids = np.empty((q.shape[0], 2 * nprobe), np.int32)
    dists = np.empty((q.shape[0], 2 * nprobe), np.float32)
    cnt = np.empty(q.shape[0], np.int32)
    lib().vo_route_spill(P(c), c.shape[0], c.shape[1], metric, P(q), q.shape[0], nprobe, float(gamma), P(sp),
                         nthreads or threads(), P(lids), P(dists), P(cnt))
    return [(lids[i, : cnt[i]], dists[i, : cnt[i]]) for i in range(q.shape[0])]


def ivfpq_search(centroids, list_offsets, list_ordinals, m, ks, codebooks, codes, queries, metric, k, nprobe,
                 rescore=1, vectors=None, policy=CANONICAL, nthreads=None):
    c, q = f32(centroids), f32(queries)
    off = np.ascontiguousarray(list_offsets, np.int64)
    ords = np.ascontiguousarray(list_ordinals, np.int32)
    codes = np.ascontiguousarray(codes, np.uint8)
    v = None if vectors is None else f32(vectors)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_ivfpq_search(P(c), c.shape[0], c.shape[1], P(off), P(ords), m, ks, P(f32(codebooks)), P(codes),
                          codes.shape[0], metric, P(q), q.shape[0], k, nprobe, rescore, P(v), policy,
                          nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def ivfflat_search(centroids, list_offsets, list_ordinals, vectors, queries, metric, k, nprobe, policy=CANONICAL,
                   nthreads=None):
    c, q, v = f32(centroids), f32(queries), f32(vectors)
    off = np.ascontiguousarray(list_offsets, np.int64)
    ords = np.ascontiguousarray(list_ordinals, np.int32)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_ivfflat_search(P(c), c.shape[0], c.shape[1], P(off), P(ords), P(v), v.shape[0], metric, P(q), q.shape[0],
                            k, nprobe, policy, nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def ivfpq_search_spill(centroids, list_offsets, list_ordinals, m, ks, codebooks, codes, queries, metric, k, nprobe,
                       gamma, spill_targets, rescore=1, vectors=None, nthreads=None):
    """IvfIndex.pqSearch with SOAR spill routing (gamma > 0), canonical ranking."""
    c, q = f32(centroids), f32(queries)
    off = np.ascontiguousarray(list_offsets, np.int64)
    ords = np.ascontiguousarray(list_ordinals, np.int32)
    codes = np.ascontiguousarray(codes, np.uint8)
    sp = np.ascontiguousarray(spill_targets, np.int32)
    v = None if vectors is None else f32(vectors)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_ivfpq_search_spill(P(c), c.shape[0], c.shape[1], P(off), P(ords), m, ks, P(f32(codebooks)), P(codes),
                                codes.shape[0], metric, P(q), q.shape[0], k, nprobe, float(gamma), P(sp), rescore, P(v),
                                nthreads or threads(), P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def ivfflat_search_full(centroids, list_offsets, list_ordinals, vectors, radii, queries, metric, k, nprobe, gamma=0.0,
                        spill_targets=None, key_dims=None, nthreads=None):
    """IvfIndex.search without PQ as the reference runs it: SOAR spill routing (gamma > 0), for
    EUCLIDEAN the early exit against `radii` (None: every probed list scanned), and the HARMONY
    scan of partitions with key dimensions (`key_dims`: one list of dimensions, or None, per list)."""
    c, q, v = f32(centroids), f32(queries), f32(vectors)
    off = np.ascontiguousarray(list_offsets, np.int64)
    ords = np.ascontiguousarray(list_ordinals, np.int32)
    r = None if radii is None else f32(radii)
    sp = None if spill_targets is None else np.ascontiguousarray(spill_targets, np.int32)
    kd_off = kd = None
    if key_dims is not None:
        sizes = [0 if d is None else len(d) for d in key_dims]
        kd_off = np.zeros(len(key_dims) + 1, np.int64)
        kd_off[1:] = np.cumsum(sizes)
        kd = np.ascontiguousarray(np.concatenate([np.asarray(d, np.int32) for d in key_dims if d is not None]
                                                 or [np.zeros(0, np.int32)]), np.int32)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_ivfflat_search_spill(P(c), c.shape[0], c.shape[1], P(off), P(ords), P(v), metric, P(r), P(q), q.shape[0],
                                  k, nprobe, float(gamma), P(sp), P(kd_off), P(kd), nthreads or threads(), P(ids), P(sc),
                                  P(cnt))
    return ids, sc, cnt


def ivf_radii(centroids, list_offsets, list_ordinals, vectors):
    """BuoyIndex.computeRadii over CSR partitions: the largest member distance per cluster."""
    c, v = f32(centroids), f32(vectors)
    off = np.ascontiguousarray(list_offsets, np.int64)
    ords = np.ascontiguousarray(list_ordinals, np.int32)
    out = np.empty(c.shape[0], np.float32)
    lib().vo_ivf_radii(P(c), c.shape[0], c.shape[1], P(off), P(ords), P(v), P(out))
    return out


def ivfflat_search_early_exit(centroids, list_offsets, list_ordinals, vectors, radii, queries, metric, k, nprobe,
                              policy=CANONICAL, nthreads=None):
    """IvfIndex.search with the reference's EUCLIDEAN early exit against the given radii."""
    c, q, v, r = f32(centroids), f32(queries), f32(vectors), f32(radii)
    off = np.ascontiguousarray(list_offsets, np.int64)
    ords = np.ascontiguousarray(list_ordinals, np.int32)
    ids, sc, cnt = _outs(q.shape[0], k)
    lib().vo_ivfflat_search_early_exit(P(c), c.shape[0], c.shape[1], P(off), P(ords), P(v), v.shape[0], metric, P(r),
                                       P(q), q.shape[0], k, nprobe, policy, nthreads or threads(), P(ids), P(sc),
                                       P(cnt))
    return ids, sc, cnt


def merge_shards(offsets, shard_ids, shard_scores, shard_counts, k, policy=CANONICAL):
    sids = np.ascontiguousarray(shard_ids, np.int32)
    ssc = f32(shard_scores)
    scnt = np.ascontiguousarray(shard_counts, np.int32)
    S, nq, kin = sids.shape
    off = np.ascontiguousarray(offsets, np.int64)
    ids, sc, cnt = _outs(nq, k)
    lib().vo_merge_shards(S, P(off), P(sids), P(ssc), P(scnt), kin, nq, k, policy, P(ids), P(sc), P(cnt))
    return ids, sc, cnt


def topk_select(scores, k):
    s = f32(scores)
    out = np.empty(max(1, min(k, len(s))), np.int32)
    n = lib().vo_topk_select(P(s), len(s), k, P(out))
    if n < 0:
        raise ValueError("NaN score")
    return out[:n]


def build_ivf_lists(assign, nlist):
    """CSR partitions (IvfIndex.build posting lists, IvfIndex.java:110-113): ordinals ascending."""
    order = np.argsort(assign, kind="stable").astype(np.int32)
    counts = np.bincount(assign, minlength=nlist)
    off = np.zeros(nlist + 1, np.int64)
    off[1:] = np.cumsum(counts)
    return off, order
