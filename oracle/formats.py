"""Writers of the reference's persistent index files, restated from its Java encoders.

TEST INFRASTRUCTURE ONLY: tests/ use these to produce files in the layout the reference writes,
which the library's readers (vx_quantized_bin_* / vx_ivf_graph_*) must load into the same index
the array builders make.  The product never imports this module.

  quantized_bin_*  QuantizedVectorsCodec.encode (vectors-db/.../storage/QuantizedVectorsCodec.java:
                   91-122): little-endian; writeCommonHeader (:1047-1054) = magic 'VQTZ'
                   (FileFormat.java:77), version 1 (FileFormat.java:112), QuantizerKind ordinal,
                   dimension, vectorCount; encodeSQ (:224-255), encodeBQ (:425-473), encodeFp16
                   (:194-209).
  ivf_graph_bin    IvfIndex.encode (vectors-ivf/.../IvfIndex.java:354-400) with the PQ trailer
                   (encodePqTrailer, :450-474) around BuoyIndex.encode (BuoyIndex.java:130-147):
                   java.nio.ByteBuffer.allocate (big-endian by default) and DataOutputStream
                   (big-endian, writeUTF = u16 length + modified UTF-8, ASCII for metric names).

No reference-written file exists to pin these (the reference cannot run here); the reference's own
codec tests pin the header offsets (version at byte 4, kind at 8, dimension at 12, 20-byte header,
12-byte SQ state: QuantizedVectorsCodecTest.java:510-586), which tests/test_formats.py re-checks.
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC_QUANTIZED = 0x5A545156
VERSION_QUANTIZED = 1
# QuantizerKind ordinals (vectors-db/.../QuantizerKind.java)
NONE, SQ8, SQ4, PQ, BQ, RABITQ, NVQ, TURBOQUANT, FP16, EXTENDED_RABITQ = range(10)
INT8, INT4 = 0, 1          # ScalarBits ordinals
SIGN_BIT, BBQ = 0, 1       # BinaryMode ordinals
METRIC_NAMES = ["EUCLIDEAN", "DOT_PRODUCT", "COSINE", "MAXIMUM_INNER_PRODUCT"]


def _header(kind: int, dim: int, count: int) -> bytes:
    return struct.pack("<iiiii", MAGIC_QUANTIZED, VERSION_QUANTIZED, kind, dim, count)


def quantized_bin_sq8(codes, corrections, min_quantile: float, max_quantile: float) -> bytes:
    """encodeSQ for ScalarBits.INT8: state (bits, minQuantile, maxQuantile), then per vector its
    dim code bytes followed by its float correction."""
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    corr = np.ascontiguousarray(corrections, dtype="<f4")
    n, dim = codes.shape
    rec = np.empty((n, dim + 4), np.uint8)
    rec[:, :dim] = codes.view(np.uint8)
    rec[:, dim:] = corr.reshape(n, 1).view(np.uint8)
    return _header(SQ8, dim, n) + struct.pack("<iff", INT8, min_quantile, max_quantile) + rec.tobytes()


def quantized_bin_sq4(packed, corrections, dim: int, min_quantile: float, max_quantile: float) -> bytes:
    """encodeSQ for ScalarBits.INT4: ceil(dim/2) packed bytes + correction per vector."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    corr = np.ascontiguousarray(corrections, dtype="<f4")
    n, nb = packed.shape
    rec = np.empty((n, nb + 4), np.uint8)
    rec[:, :nb] = packed
    rec[:, nb:] = corr.reshape(n, 1).view(np.uint8)
    return _header(SQ4, dim, n) + struct.pack("<iff", INT4, min_quantile, max_quantile) + rec.tobytes()


def quantized_bin_bq(words, dim: int, bbq_centroid=None, bbq_corrections=None) -> bytes:
    """encodeBQ: the BinaryMode ordinal (+ centroid for BBQ), then per vector ceil(dim/64)
    little-endian longs (+ 3 float corrections for BBQ)."""
    words = np.ascontiguousarray(words, dtype="<u8")
    n, nw = words.shape
    if bbq_centroid is None:
        return _header(BQ, dim, n) + struct.pack("<i", SIGN_BIT) + words.tobytes()
    corr = np.ascontiguousarray(bbq_corrections, dtype="<f4").reshape(n, 3)
    rec = np.empty((n, nw * 8 + 12), np.uint8)
    rec[:, : nw * 8] = words.view(np.uint8).reshape(n, nw * 8)
    rec[:, nw * 8:] = corr.view(np.uint8).reshape(n, 12)
    cent = np.ascontiguousarray(bbq_centroid, dtype="<f4")
    return _header(BQ, dim, n) + struct.pack("<i", BBQ) + cent.tobytes() + rec.tobytes()


def quantized_bin_pq(codes, codebooks, dim: int, m: int, ks: int, global_centroid=None, subs=None) -> bytes:
    """encodePQ: numSubspaces, numClusters, hasGlobalCentroid (+ the centroid), m (size, offset)
    pairs (default computeSubspaceSizesAndOffsets), the codebooks concatenated per subspace, then
    per vector its m code bytes."""
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    n = codes.shape[0]
    if subs is None:
        base, rem, o = dim // m, dim % m, 0
        subs = []
        for s_ in range(m):
            sz = base + (1 if s_ < rem else 0)
            subs.append((sz, o))
            o += sz
    out = _header(PQ, dim, n) + struct.pack("<iii", m, ks, 0 if global_centroid is None else 1)
    if global_centroid is not None:
        out += np.ascontiguousarray(global_centroid, dtype="<f4").tobytes()
    out += b"".join(struct.pack("<ii", sz, so) for sz, so in subs)
    return out + np.ascontiguousarray(codebooks, dtype="<f4").tobytes() + codes.tobytes()


def quantized_bin_fp16(codes) -> bytes:
    """encodeFp16: no quantizer state; dim little-endian binary16 values per vector."""
    codes = np.ascontiguousarray(codes, dtype="<u2")
    n, dim = codes.shape
    return _header(FP16, dim, n) + codes.tobytes()


def buoy_bytes(centroids, metric: int, spill=None, sizes=None, radii=None) -> bytes:
    """BuoyIndex.encode: k, dim, writeUTF(metric name), centroids row by row, spill targets,
    cluster sizes, cluster radii (DataOutputStream, big-endian)."""
    cent = np.ascontiguousarray(centroids, dtype=">f4")
    k, dim = cent.shape
    name = METRIC_NAMES[metric].encode("ascii")
    spill = np.full(k, -1, ">i4") if spill is None else np.asarray(spill, ">i4")
    sizes = np.zeros(k, ">i4") if sizes is None else np.asarray(sizes, ">i4")
    radii = np.zeros(k, ">f4") if radii is None else np.asarray(radii, ">f4")
    return (struct.pack(">iiH", k, dim, len(name)) + name + cent.tobytes() + spill.tobytes() + sizes.tobytes()
            + radii.tobytes())


def ivf_graph_bin(centroids, list_offsets, list_ordinals, metric: int, pq=None, key_dims=None,
                  sizes=None, radii=None, spill=None) -> bytes:
    """IvfIndex.encode: [buoyLen][buoy] [k] k x ([ordCount][ordinals][keyDimCount][keyDims])
    [pqFlag] [PQ trailer].  pq = dict(m, ks, codebooks (concatenated per subspace), codes
    [n][m] in ordinal order, anisotropic (float), global_centroid (optional), subs (optional
    [m][2] sizes/offsets; default computeSubspaceSizesAndOffsets)); None writes pqFlag 0."""
    buoy = buoy_bytes(centroids, metric, spill=spill, sizes=sizes, radii=radii)
    k, dim = np.asarray(centroids).shape
    off = np.asarray(list_offsets, np.int64)
    ords = np.asarray(list_ordinals, ">i4")
    parts = []
    for c in range(k):
        o = ords[off[c]:off[c + 1]]
        kd = np.asarray([] if key_dims is None or key_dims[c] is None else key_dims[c], ">i4")
        parts.append(struct.pack(">i", len(o)) + o.tobytes() + struct.pack(">i", len(kd)) + kd.tobytes())
    out = struct.pack(">i", len(buoy)) + buoy + struct.pack(">i", k) + b"".join(parts)
    if pq is None:
        return out + b"\x00"
    m, ks = pq["m"], pq["ks"]
    subs = pq.get("subs")
    if subs is None:  # computeSubspaceSizesAndOffsets (ProductQuantizer.java:686-700)
        base, rem, o = dim // m, dim % m, 0
        subs = []
        for s in range(m):
            sz = base + (1 if s < rem else 0)
            subs.append((sz, o))
            o += sz
    gc = pq.get("global_centroid")
    t = struct.pack(">iiif", dim, m, ks, pq.get("anisotropic", -1.0)) + (b"\x00" if gc is None else b"\x01")
    if gc is not None:
        t += np.asarray(gc, ">f4").tobytes()
    cb = np.asarray(pq["codebooks"], np.float32).reshape(-1)
    at = 0
    for sz, so in subs:
        t += struct.pack(">ii", sz, so) + cb[at:at + ks * sz].astype(">f4").tobytes()
        at += ks * sz
    codes = np.ascontiguousarray(pq["codes"], np.uint8)
    t += struct.pack(">i", codes.shape[0]) + codes.tobytes()
    return out + b"\x01" + t
