"""Host-side mirror of the reference's index SPI over the libvx.so C ABI.

Names, argument meaning and error behaviour follow
``vectors-db/src/main/java/com/integrallis/vectors/db/index/IndexSpi.java`` and its scan
adapters, so a caller of ``FlatScanAdapter`` / ``QuantizedFlatScanAdapter`` / ``IvfPqAdapter``
/ ``IndexShards`` finds the same contract here, with the scans running on a B200:

* ``build(vectors, metric)``                         IndexSpi.java:43
* ``search(query, k, search_list_size, oqf)``        IndexSpi.java:62
* ``search_batch(queries, k, search_list_size, oqf)`` IndexSpi.java:127-152
* ``size()`` / ``close()``                            IndexSpi.java:155-159
* ``SearchOutcome(ordinals, scores)``                 IndexSpi.java:162-173

Exceptions: ``IllegalArgumentException`` (bad k, empty batch, dimension mismatch),
``NullPointerException`` (missing inputs), ``GpuUnavailableException`` (no usable GPU or a
native failure, as CuVsBruteForceAdapter.java:67-70,86-89), ``UnsupportedOperationException``.
Results are ordered by (score desc, ordinal asc).
"""
from __future__ import annotations

import ctypes as C
import enum
import os
import math
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _native as N


class IllegalArgumentException(ValueError):
    pass


class NullPointerException(TypeError):
    pass


class GpuUnavailableException(RuntimeError):
    pass


class UnsupportedOperationException(NotImplementedError):
    pass


class IOException(OSError):
    """java.io.IOException: a quantized.bin / graph.bin that does not decode."""


_EXC = {
    N.VX_ERR_INVALID_ARGUMENT: IllegalArgumentException,
    N.VX_ERR_NULL_POINTER: NullPointerException,
    N.VX_ERR_GPU_UNAVAILABLE: GpuUnavailableException,
    N.VX_ERR_CUDA: GpuUnavailableException,
    N.VX_ERR_OUT_OF_MEMORY: GpuUnavailableException,
    N.VX_ERR_UNSUPPORTED: UnsupportedOperationException,
    N.VX_ERR_DEVICE_TIMEOUT: GpuUnavailableException,
    N.VX_ERR_FORMAT: IOException,
}


def _check(status: int) -> None:
    if status != N.VX_OK:
        raise _EXC.get(status, GpuUnavailableException)(N.last_error())


class SimilarityFunction(enum.IntEnum):
    """vectors-core/.../SimilarityFunction.java:30-120 (ordinal order)."""

    EUCLIDEAN = 0
    DOT_PRODUCT = 1
    COSINE = 2
    MAXIMUM_INNER_PRODUCT = 3


@dataclass
class SearchOutcome:
    """IndexSpi.SearchOutcome: ordinals and scores, descending."""

    ordinals: np.ndarray
    scores: np.ndarray

    def __post_init__(self):
        if len(self.ordinals) != len(self.scores):
            raise IllegalArgumentException(
                f"ordinals.length ({len(self.ordinals)}) must match scores.length ({len(self.scores)})"
            )


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _as_matrix(vectors, name: str) -> np.ndarray:
    if vectors is None:
        raise NullPointerException(f"{name} must not be null")
    a = np.ascontiguousarray(np.asarray(vectors, dtype=np.float32))
    if a.ndim == 1 and a.size == 0:
        a = a.reshape(0, 0)
    if a.ndim != 2:
        raise IllegalArgumentException(f"{name} must be a 2-D array of rows")
    return a


def _expect_shape(a: np.ndarray, shape, name: str) -> None:
    """The C entry points read exactly this many elements; a Java array of another length
    would have thrown, so a mismatch is an IllegalArgumentException, never a short read."""
    if a.shape != tuple(shape):
        raise IllegalArgumentException(f"{name} must be {list(shape)}, got {list(a.shape)}")


def _expect_rows(v, n: int, dim: int) -> None:
    """Optional fp32 rows (two-pass rescore) must match the encoded index: [n][dim]."""
    if v is not None:
        _expect_shape(v, (n, dim), "vectors")


def _expect_partitions(off: np.ndarray, ords: np.ndarray, nlist: int) -> None:
    """CSR partitions: nlist + 1 offsets, as many ordinals as the last offset says."""
    _expect_shape(off, (nlist + 1,), "list_offsets")
    total = int(off[-1]) if off.size else 0
    if ords.ndim != 1 or ords.shape[0] != total:
        raise IllegalArgumentException(f"list_ordinals must hold list_offsets[nlist] = {total} ordinals, "
                                       f"got {list(ords.shape)}")


def _file_bytes(data) -> np.ndarray:
    """The bytes of a persistent file: a path, bytes-like, or a uint8 array (e.g. np.memmap)."""
    if isinstance(data, (str, os.PathLike)):
        return np.fromfile(data, dtype=np.uint8)
    if data is None:
        raise NullPointerException("bytes must not be null")
    if isinstance(data, np.ndarray):
        return np.ascontiguousarray(data.reshape(-1).view(np.uint8))
    return np.frombuffer(data, dtype=np.uint8)


def _strided_rows(vectors, dim: int):
    """(array, row stride in floats) for fp32 rows that may sit further apart than dim floats, as
    in a mapped vectors.bin viewed as np.memmap(path, np.float32).reshape(n, stride)[:, :dim]."""
    if vectors is None:
        return None, dim
    a = np.asarray(vectors, dtype=np.float32)
    if a.ndim != 2 or a.shape[1] != dim:
        raise IllegalArgumentException(f"vectors must be [n][{dim}] float32 rows")
    if a.strides[1] == 4 and a.strides[0] % 4 == 0 and a.strides[0] >= 4 * dim:
        return a, a.strides[0] // 4
    a = np.ascontiguousarray(a)
    return a, dim


def quantized_bin_info(data) -> tuple[int, int, int]:
    """(QuantizerKind ordinal, dimension, vectorCount) of a quantized.bin, validated the way
    QuantizedVectorsCodec.decode validates it (no GPU needed).  Raises IOException for malformed
    bytes and UnsupportedOperationException for kinds this library does not serve."""
    b = _file_bytes(data)
    kind, dim, cnt = C.c_int32(), C.c_int32(), C.c_int64()
    _check(N.lib().vx_quantized_bin_info(_ptr(b), b.size, C.byref(kind), C.byref(dim), C.byref(cnt)))
    return kind.value, dim.value, cnt.value


def ivf_graph_info(data) -> dict:
    """Shape of an IVF_PQ graph.bin (IvfIndex.encode) validated as IvfIndex.decode reads it."""
    b = _file_bytes(data)
    nlist, dim, cnt, m, metric = C.c_int32(), C.c_int32(), C.c_int64(), C.c_int32(), C.c_int32()
    _check(N.lib().vx_ivf_graph_info(_ptr(b), b.size, C.byref(nlist), C.byref(dim), C.byref(cnt), C.byref(m),
                                     C.byref(metric)))
    return {"nlist": nlist.value, "dim": dim.value, "count": cnt.value, "m": m.value,
            "metric": SimilarityFunction(metric.value)}


def _outcomes(ids: np.ndarray, scores: np.ndarray, counts: np.ndarray) -> list[SearchOutcome]:
    return [SearchOutcome(ids[i, : counts[i]].copy(), scores[i, : counts[i]].copy()) for i in range(len(counts))]


class _Handle:
    """Owns one vx_index*."""

    def __init__(self):
        self.ptr = C.c_void_p()

    def close(self):
        if self.ptr:
            N.lib().vx_index_free(self.ptr)
            self.ptr = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class IndexSpi:
    """Common search plumbing (IndexSpi.java:34-174)."""

    def __init__(self, device: int = 0):
        self.device = device
        self._h = _Handle()
        self._n = 0
        self._dim = 0

    # -- IndexSpi
    def size(self) -> int:
        return self._n

    def close(self) -> None:
        self._h.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def search(self, query, k: int, search_list_size: int = 0, over_query_factor: float = 1.0,
               search_multi_start: int = 1) -> SearchOutcome:
        """IndexSpi.search; the five-argument overload's searchMultiStart is ignored, as its
        default does for every brute-force and IVF backend (IndexSpi.java:82-86)."""
        if query is None:
            raise NullPointerException("query must not be null")
        if k <= 0:
            raise IllegalArgumentException(f"k must be positive: {k}")
        q = np.asarray(query, dtype=np.float32).reshape(1, -1)
        return self.search_batch(q, k, search_list_size, over_query_factor)[0]

    def search_with_predicate(self, query, k: int, search_list_size: int, over_query_factor: float,
                              predicate) -> SearchOutcome:
        """IndexSpi.searchWithPredicate (IndexSpi.java:103-107): the scan backends keep the default,
        which ignores the predicate and searches; the caller post-filters the outcome
        (VectorCollectionImpl.search widens k by filterExpansion for that)."""
        return self.search(query, k, search_list_size, over_query_factor)

    def search_batch(self, queries, k: int, search_list_size: int = 0, over_query_factor: float = 1.0) -> list[SearchOutcome]:
        q = self._queries(queries, k)
        if self._n == 0:
            return [SearchOutcome(np.zeros(0, np.int32), np.zeros(0, np.float32)) for _ in range(len(q))]
        ids, sc, cnt = self._alloc(len(q), k)
        _check(
            N.lib().vx_search_batch(
                self._h.ptr, _ptr(q), len(q), q.shape[1], k, search_list_size, float(over_query_factor),
                _ptr(ids), _ptr(sc), _ptr(cnt),
            )
        )
        return _outcomes(ids, sc, cnt)

    def search_batch_arrays(self, queries, k: int, search_list_size: int = 0, over_query_factor: float = 1.0):
        """searchBatch through the host-buffer C ABI call, returning the flat result arrays
        (ids [nq][k], scores [nq][k], counts [nq]) instead of one SearchOutcome per query."""
        q = self._queries(queries, k)
        ids, sc, cnt = self._alloc(len(q), k)
        if self._n == 0:
            ids.fill(-1)
            sc.fill(0)
            cnt.fill(0)
            return ids, sc, cnt
        _check(
            N.lib().vx_search_batch(
                self._h.ptr, _ptr(q), len(q), q.shape[1], k, search_list_size, float(over_query_factor),
                _ptr(ids), _ptr(sc), _ptr(cnt),
            )
        )
        return ids, sc, cnt

    def search_batch_device(self, queries, k: int, search_list_size: int = 0, over_query_factor: float = 1.0, stream=None):
        """searchBatch on device tensors (torch, cuda): returns (ids, scores, counts) tensors."""
        import torch

        q = queries.contiguous()
        nq = q.shape[0]
        ids = torch.empty((nq, k), dtype=torch.int32, device=q.device)
        sc = torch.empty((nq, k), dtype=torch.float32, device=q.device)
        cnt = torch.empty((nq,), dtype=torch.int32, device=q.device)
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        _check(
            N.lib().vx_search_batch_device(
                self._h.ptr, C.c_void_p(q.data_ptr()), nq, q.shape[1], k, search_list_size,
                float(over_query_factor), C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                C.c_void_p(cnt.data_ptr()), C.c_void_p(st),
            )
        )
        return ids, sc, cnt

    # -- helpers
    def _queries(self, queries, k: int) -> np.ndarray:
        if queries is None:
            raise NullPointerException("queries must not be null")
        if len(queries) == 0:
            raise IllegalArgumentException("queries must not be empty")
        if k <= 0:
            raise IllegalArgumentException(f"k must be positive: {k}")
        if self._n == 0:
            return np.zeros((len(queries), max(1, self._dim)), np.float32)
        if isinstance(queries, np.ndarray) and queries.ndim == 2 and queries.dtype == np.float32:
            # one contiguous [nq][dim] block (pinned or pageable): no per-row copies
            if queries.shape[1] != self._dim:
                raise IllegalArgumentException(
                    f"Query 0 dimension {queries.shape[1]} does not match index dimension {self._dim}"
                )
            return np.ascontiguousarray(queries)
        rows = []
        for i, qi in enumerate(queries):
            if qi is None:
                raise NullPointerException(f"queries[{i}] must not be null")
            a = np.asarray(qi, dtype=np.float32).reshape(-1)
            if a.shape[0] != self._dim:
                raise IllegalArgumentException(
                    f"Query {i} dimension {a.shape[0]} does not match index dimension {self._dim}"
                )
            rows.append(a)
        return np.ascontiguousarray(np.stack(rows))

    @staticmethod
    def _alloc(nq: int, k: int):
        return (np.empty((nq, k), np.int32), np.empty((nq, k), np.float32), np.empty((nq,), np.int32))


class FlatScanAdapter(IndexSpi):
    """FlatScanAdapter (FlatScanAdapter.java:35-233): exact scan, searchListSize and
    overQueryFactor ignored."""

    def build(self, vectors, metric: SimilarityFunction) -> None:
        """vectors: [n][dim] float32 rows (numpy / lists, or a CUDA tensor, copied on device)."""
        if metric is None:
            raise NullPointerException("metric must not be null")
        if vectors is None:
            raise NullPointerException("vectors must not be null")
        self._h.close()
        if getattr(vectors, "is_cuda", False):
            t = vectors.contiguous()
            n, dim = (t.shape[0], t.shape[1]) if t.numel() else (0, 0)
            _check(N.lib().vx_flat_build(self.device, C.c_void_p(t.data_ptr()), n, dim, dim, int(metric),
                                         C.byref(self._h.ptr)))
        else:
            v = _as_matrix(vectors, "vectors")
            n, dim = v.shape if v.size else (0, 0)
            _check(N.lib().vx_flat_build(self.device, _ptr(v), n, dim, dim, int(metric), C.byref(self._h.ptr)))
        self._n, self._dim, self.metric = n, dim, SimilarityFunction(metric)


class QuantizedFlatScanAdapter(IndexSpi):
    """QuantizedFlatScanAdapter (QuantizedFlatScanAdapter.java:27-177) over one of the
    reference encodings.  ``search_batch`` applies the adapter's contract (overQueryFactor <= 1
    -> exact scan; otherwise ceil(k * oqf) approximate candidates re-scored exactly), which needs
    the fp32 rows; ``scan_candidates`` is selectApproximateCandidates alone."""

    def __init__(self, device: int = 0):
        super().__init__(device)
        self.kind = None

    def build_sq8(self, codes, corrections, min_quantile: float, max_quantile: float, metric, vectors=None):
        codes = np.ascontiguousarray(np.asarray(codes, dtype=np.int8))
        corr = np.ascontiguousarray(np.asarray(corrections, dtype=np.float32))
        v = None if vectors is None else _as_matrix(vectors, "vectors")
        if codes.ndim != 2:
            raise IllegalArgumentException("codes must be [n][dim]")
        n, dim = codes.shape
        _expect_shape(corr, (n,), "corrections")
        _expect_rows(v, n, dim)
        self._h.close()
        _check(
            N.lib().vx_sq8_build(self.device, _ptr(codes), _ptr(corr), n, dim, float(min_quantile), float(max_quantile),
                                 int(metric), _ptr(v), dim, C.byref(self._h.ptr))
        )
        self._n, self._dim, self.metric, self.kind = n, dim, SimilarityFunction(metric), "SQ8"

    def build_sq4(self, packed, corrections, dim: int, min_quantile: float, max_quantile: float, metric, vectors=None):
        """ScalarQuantizedVectors INT4: packed [n][ceil(dim/2)] codes, low nibble = even dimension."""
        packed = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8))
        corr = np.ascontiguousarray(np.asarray(corrections, dtype=np.float32))
        v = None if vectors is None else _as_matrix(vectors, "vectors")
        n = packed.shape[0]
        if packed.ndim != 2 or packed.shape[1] != (dim + 1) // 2:
            raise IllegalArgumentException(f"packed codes must be [n][{(dim + 1) // 2}]")
        _expect_shape(corr, (n,), "corrections")
        _expect_rows(v, n, dim)
        self._h.close()
        _check(
            N.lib().vx_sq4_build(self.device, _ptr(packed), _ptr(corr), n, dim, float(min_quantile), float(max_quantile),
                                 int(metric), _ptr(v), dim, C.byref(self._h.ptr))
        )
        self._n, self._dim, self.metric, self.kind = n, dim, SimilarityFunction(metric), "SQ4"

    def build_bq(self, words, dim: int, metric, vectors=None):
        words = np.ascontiguousarray(np.asarray(words, dtype=np.uint64))
        v = None if vectors is None else _as_matrix(vectors, "vectors")
        n = words.shape[0]
        _expect_shape(words, (n, (dim + 63) // 64), "words")
        _expect_rows(v, n, dim)
        self._h.close()
        _check(N.lib().vx_bq_build(self.device, _ptr(words), n, dim, int(metric), _ptr(v), dim, C.byref(self._h.ptr)))
        self._n, self._dim, self.metric, self.kind = n, dim, SimilarityFunction(metric), "BQ"

    def build_bbq(self, words, corrections, centroid, dim: int, metric, vectors=None):
        """BinaryQuantizedVectors in BBQ mode: centroid-relative sign bits [n][ceil(dim/64)],
        corrections [n][3] = (|v - c|^2, vl, width), the quantizer's centroid."""
        words = np.ascontiguousarray(np.asarray(words, dtype=np.uint64))
        corr = np.ascontiguousarray(np.asarray(corrections, dtype=np.float32))
        cent = np.ascontiguousarray(np.asarray(centroid, dtype=np.float32))
        v = None if vectors is None else _as_matrix(vectors, "vectors")
        n = words.shape[0]
        if corr.shape != (n, 3) or cent.shape != (dim,):
            raise IllegalArgumentException("corrections must be [n][3] and the centroid [dim]")
        _expect_shape(words, (n, (dim + 63) // 64), "words")
        _expect_rows(v, n, dim)
        self._h.close()
        _check(N.lib().vx_bbq_build(self.device, _ptr(words), _ptr(corr), _ptr(cent), n, dim, int(metric), _ptr(v), dim,
                                    C.byref(self._h.ptr)))
        self._n, self._dim, self.metric, self.kind = n, dim, SimilarityFunction(metric), "BBQ"

    def build_pq(self, codes, codebooks, m: int, ks: int, metric, global_centroid=None, vectors=None):
        """PQVectors (PQVectors.java:40-191): codes [n][m] (uint8), codebooks concatenated per
        subspace (computeSubspaceSizesAndOffsets' sizes; ks * dim floats), the quantizer's global
        centroid or None."""
        codes = np.ascontiguousarray(np.asarray(codes, dtype=np.uint8))
        cb = np.ascontiguousarray(np.asarray(codebooks, dtype=np.float32)).reshape(-1)
        if codes.ndim != 2 or codes.shape[1] != m:
            raise IllegalArgumentException(f"codes must be [n][{m}]")
        if cb.size % ks:
            raise IllegalArgumentException("codebooks must hold ks * dim floats")
        n, dim = codes.shape[0], cb.size // ks
        gc = None if global_centroid is None else np.ascontiguousarray(np.asarray(global_centroid, dtype=np.float32))
        if gc is not None and gc.shape != (dim,):
            raise IllegalArgumentException(f"global_centroid must hold {dim} floats")
        v = None if vectors is None else _as_matrix(vectors, "vectors")
        _expect_rows(v, n, dim)
        self._h.close()
        _check(N.lib().vx_pq_build(self.device, _ptr(cb), _ptr(gc), _ptr(codes), n, dim, m, ks, int(metric), _ptr(v),
                                   dim, C.byref(self._h.ptr)))
        self._n, self._dim, self.metric, self.kind = n, dim, SimilarityFunction(metric), "PQ"

    def build_fp16(self, codes, metric, vectors=None):
        """codes: [n][dim] binary16 bit patterns (numpy uint16, or a CUDA float16 / int16 tensor,
        copied on the device)."""
        v = None if vectors is None else _as_matrix(vectors, "vectors")
        if getattr(codes, "is_cuda", False):
            t = codes.contiguous()
            if t.element_size() != 2:
                raise IllegalArgumentException("fp16 codes must be 2-byte elements")
            n, dim = t.shape
            ptr = C.c_void_p(t.data_ptr())
        else:
            arr = np.ascontiguousarray(np.asarray(codes, dtype=np.uint16))
            if arr.ndim != 2:
                raise IllegalArgumentException("codes must be [n][dim]")
            n, dim = arr.shape
            ptr = _ptr(arr)
        _expect_rows(v, n, dim)
        self._h.close()
        _check(N.lib().vx_fp16_build(self.device, ptr, n, dim, int(metric), _ptr(v), dim, C.byref(self._h.ptr)))
        self._n, self._dim, self.metric, self.kind = n, dim, SimilarityFunction(metric), "FP16"

    def load_quantized_bin(self, data, metric, vectors=None):
        """Opens a persistent quantized.bin (QuantizedVectorsCodec.decode) as this adapter's index:
        SQ8, SQ4, BQ (SIGN_BIT or BBQ), FP16 or PQ.  ``vectors`` are the fp32 rows for the two-pass rescore (a mapped
        vectors.bin view with its 64-byte row stride is taken as is)."""
        b = _file_bytes(data)
        kind, dim, n = quantized_bin_info(b)
        v, stride = _strided_rows(vectors, dim)
        self._h.close()
        _check(N.lib().vx_quantized_bin_build(self.device, _ptr(b), b.size, int(metric), _ptr(v), stride,
                                              C.byref(self._h.ptr)))
        self._n, self._dim, self.metric = n, dim, SimilarityFunction(metric)
        self.kind = {1: "SQ8", 2: "SQ4", 3: "PQ", 4: "BQ", 8: "FP16"}[kind]
        if kind == 4:  # SIGN_BIT or BBQ: the index knows
            built = C.c_int32()
            _check(N.lib().vx_index_info(self._h.ptr, C.byref(built), None, None, None))
            if built.value == N.VX_KIND_BBQ:
                self.kind = "BBQ"

    def build(self, vectors, metric):
        raise UnsupportedOperationException("QuantizedFlatScanAdapter wraps an already-built flat index")

    def scan_candidates(self, queries, k: int) -> list[SearchOutcome]:
        q = self._queries(queries, k)
        if self._n == 0:
            return [SearchOutcome(np.zeros(0, np.int32), np.zeros(0, np.float32)) for _ in range(len(q))]
        ids, sc, cnt = self._alloc(len(q), k)
        _check(N.lib().vx_scan_candidates(self._h.ptr, _ptr(q), len(q), q.shape[1], k, _ptr(ids), _ptr(sc), _ptr(cnt)))
        return _outcomes(ids, sc, cnt)

    def scan_candidates_arrays(self, queries, k: int):
        """selectApproximateCandidates through the host-buffer C ABI call, returning the flat
        result arrays (ids [nq][k], scores [nq][k], counts [nq])."""
        q = self._queries(queries, k)
        ids, sc, cnt = self._alloc(len(q), k)
        if self._n == 0:
            ids.fill(-1)
            sc.fill(0)
            cnt.fill(0)
            return ids, sc, cnt
        _check(N.lib().vx_scan_candidates(self._h.ptr, _ptr(q), len(q), q.shape[1], k, _ptr(ids), _ptr(sc), _ptr(cnt)))
        return ids, sc, cnt

    def scan_candidates_device(self, queries, k: int, stream=None):
        import torch

        q = queries.contiguous()
        nq = q.shape[0]
        ids = torch.empty((nq, k), dtype=torch.int32, device=q.device)
        sc = torch.empty((nq, k), dtype=torch.float32, device=q.device)
        cnt = torch.empty((nq,), dtype=torch.int32, device=q.device)
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        _check(
            N.lib().vx_scan_candidates_device(self._h.ptr, C.c_void_p(q.data_ptr()), nq, q.shape[1], k,
                                              C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                              C.c_void_p(cnt.data_ptr()), C.c_void_p(st))
        )
        return ids, sc, cnt


class IvfPqAdapter(IndexSpi):
    """IvfPqAdapter over a prebuilt IVF-PQ index (IvfIndex.fromPrebuilt, IvfIndex.java:343-351).
    ``search_batch`` follows IvfPqAdapter.search (IvfPqAdapter.java:124-158); ``ivf_search`` is
    IvfIndex.search(IvfSearchRequest) (IvfIndex.java:170-171,539-619)."""

    def __init__(self, nprobe: int = 32, rescore_factor: int = 1, device: int = 0, gamma: float = 0.0):
        super().__init__(device)
        if nprobe <= 0:
            raise IllegalArgumentException(f"nprobe must be positive: {nprobe}")
        if rescore_factor < 1:
            raise IllegalArgumentException(f"rescoreFactor must be >= 1: {rescore_factor}")
        if not gamma >= 0:
            raise IllegalArgumentException(f"gamma must be >= 0, got {gamma}")
        self.nprobe, self.rescore_factor, self.gamma = nprobe, rescore_factor, float(gamma)

    def _apply_gamma(self):
        if self.gamma != 0.0:
            _check(N.lib().vx_ivf_set_gamma(self._h.ptr, self.gamma))

    def set_buoy(self, radii=None, spill_targets=None):
        """The prebuilt BuoyIndex's own state (IvfIndex.fromPrebuilt takes a BuoyIndex): cluster
        radii (BuoyIndex.clusterRadii; the IVF-flat EUCLIDEAN early exit) and SOAR spill targets
        (BuoyIndex.spillTargets, -1 = none).  None leaves that part unchanged."""
        r = None if radii is None else np.ascontiguousarray(np.asarray(radii, dtype=np.float32))
        sp = None if spill_targets is None else np.ascontiguousarray(np.asarray(spill_targets, dtype=np.int32))
        for a, name in ((r, "radii"), (sp, "spill_targets")):
            if a is not None and a.shape != (self._nlist,):
                raise IllegalArgumentException(f"{name} must hold one entry per list ({self._nlist})")
        _check(N.lib().vx_ivf_set_buoy(self._h.ptr, _ptr(r), _ptr(sp)))

    def build(self, vectors, metric):
        raise UnsupportedOperationException("k-means / PQ training is an offline step; use build_prebuilt")

    def build_prebuilt(self, centroids, list_offsets, list_ordinals, codebooks, codes, m: int, ks: int, metric, vectors=None):
        cent = _as_matrix(centroids, "centroids")
        off = np.ascontiguousarray(np.asarray(list_offsets, dtype=np.int64))
        ords = np.ascontiguousarray(np.asarray(list_ordinals, dtype=np.int32))
        cb = np.ascontiguousarray(np.asarray(codebooks, dtype=np.float32))
        codes = np.ascontiguousarray(np.asarray(codes, dtype=np.uint8))
        v = None if vectors is None else _as_matrix(vectors, "vectors")
        nlist, dim = cent.shape
        _expect_partitions(off, ords, nlist)
        if codes.ndim != 2 or codes.shape[1] != m:
            raise IllegalArgumentException(f"codes must be [n][{m}]")
        n = codes.shape[0]
        if cb.size != ks * dim:
            raise IllegalArgumentException(f"codebooks must hold ks * dim = {ks * dim} floats, got {cb.size}")
        _expect_rows(v, n, dim)
        self._h.close()
        _check(
            N.lib().vx_ivfpq_build(self.device, _ptr(cent), nlist, dim, _ptr(off), _ptr(ords), m, ks, _ptr(cb), _ptr(codes),
                                   n, int(metric), _ptr(v), self.nprobe, self.rescore_factor, C.byref(self._h.ptr))
        )
        self._n, self._dim, self.metric = n, dim, SimilarityFunction(metric)
        self._nlist = nlist
        self._apply_gamma()

    def load_graph_bin(self, data, metric=None, vectors=None):
        """Opens an IVF_PQ generation's graph.bin (IvfIndex.decode, as
        VectorCollectionImpl.openIvfPqAdapter does): centroids, partitions, PQ codebooks and codes.
        ``metric`` None takes the routing metric recorded in the file; ``vectors`` (fp32 rows, e.g.
        a mapped vectors.bin view) enable rescore_factor > 1."""
        b = _file_bytes(data)
        info = ivf_graph_info(b)
        v, stride = _strided_rows(vectors, info["dim"])
        self._h.close()
        _check(N.lib().vx_ivf_graph_build(self.device, _ptr(b), b.size, -1 if metric is None else int(metric), _ptr(v),
                                          0 if v is None else v.shape[0], stride, self.nprobe, self.rescore_factor,
                                          C.byref(self._h.ptr)))
        self._n, self._dim = (info["count"] if v is None or info["m"] else v.shape[0]), info["dim"]
        self.metric = info["metric"] if metric is None else SimilarityFunction(metric)
        self._nlist = info["nlist"]
        self._apply_gamma()

    def ivf_search(self, queries, k: int, nprobe: int, rescore_factor: int = 1, min_score: float = -3.4028235e38):
        q = self._queries(queries, k)
        if self._n == 0:
            return [SearchOutcome(np.zeros(0, np.int32), np.zeros(0, np.float32)) for _ in range(len(q))]
        ids, sc, cnt = self._alloc(len(q), k)
        _check(
            N.lib().vx_ivfpq_search(self._h.ptr, _ptr(q), len(q), q.shape[1], k, nprobe, rescore_factor, float(min_score),
                                    _ptr(ids), _ptr(sc), _ptr(cnt))
        )
        return _outcomes(ids, sc, cnt)

    def ivf_search_arrays(self, queries, k: int, nprobe: int, rescore_factor: int = 1,
                          min_score: float = -3.4028235e38):
        """ivf_search through the host-buffer C ABI call, returning the flat result arrays."""
        q = self._queries(queries, k)
        ids, sc, cnt = self._alloc(len(q), k)
        if self._n == 0:
            ids.fill(-1)
            sc.fill(0)
            cnt.fill(0)
            return ids, sc, cnt
        _check(
            N.lib().vx_ivfpq_search(self._h.ptr, _ptr(q), len(q), q.shape[1], k, nprobe, rescore_factor, float(min_score),
                                    _ptr(ids), _ptr(sc), _ptr(cnt))
        )
        return ids, sc, cnt

    def ivf_search_device(self, queries, k: int, nprobe: int, rescore_factor: int = 1,
                          min_score: float = -3.4028235e38, stream=None):
        import torch

        q = queries.contiguous()
        nq = q.shape[0]
        ids = torch.empty((nq, k), dtype=torch.int32, device=q.device)
        sc = torch.empty((nq, k), dtype=torch.float32, device=q.device)
        cnt = torch.empty((nq,), dtype=torch.int32, device=q.device)
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        _check(
            N.lib().vx_ivfpq_search_device(self._h.ptr, C.c_void_p(q.data_ptr()), nq, q.shape[1], k, nprobe,
                                           rescore_factor, float(min_score), C.c_void_p(ids.data_ptr()),
                                           C.c_void_p(sc.data_ptr()), C.c_void_p(cnt.data_ptr()), C.c_void_p(st))
        )
        return ids, sc, cnt

    def route_device(self, queries, nprobe: int, stream=None):
        """The routing step of pqSearch alone (CentroidIndex.routeWithSpillDistances, gamma 0):
        an int32 [nq][min(nprobe, nlist)] tensor of list ids, nearest first."""
        import torch

        q = queries.contiguous()
        nq = q.shape[0]
        lists = torch.empty((nq, max(1, min(nprobe, self._nlist))), dtype=torch.int32, device=q.device)
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        _check(N.lib().vx_ivf_route_device(self._h.ptr, C.c_void_p(q.data_ptr()), nq, q.shape[1], nprobe,
                                           C.c_void_p(lists.data_ptr()), C.c_void_p(st)))
        return lists

    def ivf_search_routed_device(self, queries, k: int, nprobe: int, lists, rescore_factor: int = 1,
                                 min_score: float = -3.4028235e38, stream=None):
        """pqSearch over lists routed beforehand (route_device, on any GPU holding the same
        centroids): same results as ivf_search_device with the same lists."""
        import torch

        q = queries.contiguous()
        lst = lists.contiguous()
        nq = q.shape[0]
        if lst.dtype != torch.int32 or lst.shape[0] != nq or lst.shape[1] != min(nprobe, self._nlist):
            raise IllegalArgumentException("lists must be an int32 [nq][min(nprobe, nlist)] tensor")
        ids = torch.empty((nq, k), dtype=torch.int32, device=q.device)
        sc = torch.empty((nq, k), dtype=torch.float32, device=q.device)
        cnt = torch.empty((nq,), dtype=torch.int32, device=q.device)
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        _check(
            N.lib().vx_ivfpq_search_routed_device(self._h.ptr, C.c_void_p(q.data_ptr()), nq, q.shape[1], k, nprobe,
                                                  rescore_factor, float(min_score), C.c_void_p(lst.data_ptr()),
                                                  C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                  C.c_void_p(cnt.data_ptr()), C.c_void_p(st))
        )
        return ids, sc, cnt


class IvfFlatAdapter(IvfPqAdapter):
    """IvfFlatAdapter over a prebuilt IVF index without PQ (IvfIndex.fromPrebuilt /
    IvfIndex.decode, IvfIndex.java:330-351,408-442).  ``search_batch`` follows
    IvfFlatAdapter.search (IvfFlatAdapter.java:102-140); ``ivf_search`` is IvfIndex.search's flat
    list scan (IvfIndex.java:170-289); the routing helpers are those of the IVF-PQ adapter."""

    def __init__(self, nprobe: int = 32, device: int = 0, gamma: float = 0.0):
        super().__init__(nprobe=nprobe, rescore_factor=1, device=device, gamma=gamma)

    def build_prebuilt(self, centroids, list_offsets, list_ordinals, vectors, metric):
        cent = _as_matrix(centroids, "centroids")
        off = np.ascontiguousarray(np.asarray(list_offsets, dtype=np.int64))
        ords = np.ascontiguousarray(np.asarray(list_ordinals, dtype=np.int32))
        nlist, dim = cent.shape
        _expect_partitions(off, ords, nlist)
        if getattr(vectors, "is_cuda", False):
            t = vectors
            if t.dtype != __import__("torch").float32 or t.dim() != 2 or t.stride(1) != 1:
                raise IllegalArgumentException("vectors must be [n][dim] float32 rows")
            n, ptr, stride = t.shape[0], C.c_void_p(t.data_ptr()), t.stride(0)
        else:
            v, stride = _strided_rows(vectors, dim)
            n, ptr = v.shape[0], _ptr(v)
        self._h.close()
        _check(N.lib().vx_ivfflat_build(self.device, _ptr(cent), nlist, dim, _ptr(off), _ptr(ords), ptr, n, stride,
                                        int(metric), self.nprobe, C.byref(self._h.ptr)))
        self._n, self._dim, self.metric = n, dim, SimilarityFunction(metric)
        self._nlist = nlist
        self._apply_gamma()

    def route_dist_device(self, queries, nprobe: int, stream=None):
        """Routing with distances: (lists int32, distances float32) [nq][min(nprobe, nlist)],
        nearest first -- the first step of a search split by (query, list) pair across GPUs."""
        import torch

        q = queries.contiguous()
        nq = q.shape[0]
        w = max(1, min(nprobe, self._nlist))
        lists = torch.empty((nq, w), dtype=torch.int32, device=q.device)
        dist = torch.empty((nq, w), dtype=torch.float32, device=q.device)
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        _check(N.lib().vx_ivf_route_dist_device(self._h.ptr, C.c_void_p(q.data_ptr()), nq, q.shape[1], nprobe,
                                                C.c_void_p(lists.data_ptr()), C.c_void_p(dist.data_ptr()),
                                                C.c_void_p(st)))
        return lists, dist

    def scan_pairs_device(self, queries, k: int, nprobe: int, lists, stream=None):
        """The list scan of the slots of ``lists`` that hold a list id (-1: scanned elsewhere):
        per-slot keys (int64 view of the 64-bit keys) [w][nq][min(k, n)] and counts (int32)
        [w][nq], zero in the other slots, so buffers of disjoint slot sets add up."""
        import torch

        q = queries.contiguous()
        lst = lists.contiguous()
        nq = q.shape[0]
        w = max(1, min(nprobe, self._nlist))
        if lst.dtype != torch.int32 or tuple(lst.shape) != (nq, w):
            raise IllegalArgumentException("lists must be an int32 [nq][min(nprobe, nlist)] tensor")
        kk = max(1, min(k, self._n))
        keys = torch.empty((w, nq, kk), dtype=torch.int64, device=q.device)
        cnt = torch.empty((w, nq), dtype=torch.int32, device=q.device)
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        _check(N.lib().vx_ivfflat_scan_pairs_device(self._h.ptr, C.c_void_p(q.data_ptr()), nq, q.shape[1], k, nprobe,
                                                    C.c_void_p(lst.data_ptr()), C.c_void_p(keys.data_ptr()),
                                                    C.c_void_p(cnt.data_ptr()), C.c_void_p(st)))
        return keys, cnt

    def merge_pairs_device(self, k: int, nprobe: int, lists, dist, keys, counts, min_score: float = -3.4028235e38,
                           stream=None):
        """The per-slot results of every slot (combined over the GPUs that scanned them) merged
        per query in route order with IvfIndex.search's EUCLIDEAN early exit (radii held by the
        index), then minScore: (ids, scores, counts) as ivf_search_device returns them."""
        import torch

        lst, dst, ky, ct = lists.contiguous(), dist.contiguous(), keys.contiguous(), counts.contiguous()
        nq = lst.shape[0]
        ids = torch.empty((nq, k), dtype=torch.int32, device=lst.device)
        sc = torch.empty((nq, k), dtype=torch.float32, device=lst.device)
        cnt = torch.empty((nq,), dtype=torch.int32, device=lst.device)
        st = stream if stream is not None else torch.cuda.current_stream(lst.device).cuda_stream
        _check(N.lib().vx_ivfflat_merge_pairs_device(self._h.ptr, nq, k, nprobe, C.c_void_p(lst.data_ptr()),
                                                     C.c_void_p(dst.data_ptr()), C.c_void_p(ky.data_ptr()),
                                                     C.c_void_p(ct.data_ptr()), float(min_score),
                                                     C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                                     C.c_void_p(cnt.data_ptr()), C.c_void_p(st)))
        return ids, sc, cnt

    def set_key_dims(self, key_dims):
        """ClusterPartition.keyDimensions per list (HARMONY; None or an empty list = none): a
        EUCLIDEAN search reaching such a list with a full heap scores its rows with
        squareDistance (IvfIndex.scanPartitionWithHarmony)."""
        counts = None
        if key_dims is not None:
            counts = np.ascontiguousarray(
                [0 if d is None else (int(d) if np.isscalar(d) else len(d)) for d in key_dims], np.int32)
            if counts.shape != (self._nlist,):
                raise IllegalArgumentException(f"key_dims must hold one entry per list ({self._nlist})")
        _check(N.lib().vx_ivf_set_key_dims(self._h.ptr, _ptr(counts)))

    def load_graph_bin(self, data, metric=None, vectors=None):
        """Opens an IVF_FLAT generation's graph.bin (VectorCollectionImpl.openIvfFlatAdapter):
        centroids and partitions from the file, rows from ``vectors`` (required; e.g. a mapped
        vectors.bin view)."""
        if vectors is None:
            raise NullPointerException("an IVF-flat graph.bin needs the vectors")
        super().load_graph_bin(data, metric=metric, vectors=vectors)


def shard_offsets(n: int, shards: int) -> list[int]:
    """IndexShards.build ordinal ranges: offsets[i] = n*i/s (IndexShards.java:64-81)."""
    return [(n * i) // shards for i in range(shards + 1)]


def merge_shards_device(shard_ids, shard_scores, shard_counts, offsets, k: int, stream=None):
    """IndexShards.mergeWithOffsets on device tensors: shard_* are [S, nq, kin] / [S, nq]
    int32/float32 tensors, offsets an int64 tensor of S shard starts.  Returns (ids, scores,
    counts) for the k best by (score desc, ordinal asc)."""
    import torch

    S, nq, kin = shard_ids.shape
    dev = shard_ids.device
    ids = torch.empty((nq, k), dtype=torch.int32, device=dev)
    sc = torch.empty((nq, k), dtype=torch.float32, device=dev)
    cnt = torch.empty((nq,), dtype=torch.int32, device=dev)
    st = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    off = offsets.to(device=dev, dtype=torch.int64).contiguous()
    _check(
        N.lib().vx_merge_shards_device(dev.index or 0, S, C.c_void_p(off.data_ptr()), C.c_void_p(shard_ids.contiguous().data_ptr()),
                                       C.c_void_p(shard_scores.contiguous().data_ptr()),
                                       C.c_void_p(shard_counts.contiguous().data_ptr()), kin, nq, k,
                                       C.c_void_p(ids.data_ptr()), C.c_void_p(sc.data_ptr()),
                                       C.c_void_p(cnt.data_ptr()), C.c_void_p(st))
    )
    return ids, sc, cnt
