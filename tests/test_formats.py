"""Readers of the reference's persistent files (quantized.bin, IVF graph.bin), on the CPU.

The checks mirror the reference's codec tests (QuantizedVectorsCodecTest.java:480-586: header
offsets, magic / version / kind / dimension / truncation rejections with those words in the
message) through vx_quantized_bin_info / vx_ivf_graph_info and the build entry points, which
reject a malformed file before they touch a GPU.
"""
import ctypes as C
import struct

import numpy as np
import pytest

import vectors_b200 as vx
from vectors_b200 import _native as N
from oracle import formats as F


def _sq8(n=50, dim=24, seed=1):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 128, (n, dim)).astype(np.int8)
    corr = rng.standard_normal(n).astype(np.float32)
    return codes, corr, F.quantized_bin_sq8(codes, corr, -0.75, 0.5)


def _build_status(b: bytes) -> int:
    arr = np.frombuffer(b, np.uint8)
    out = C.c_void_p()
    return N.lib().vx_quantized_bin_build(0, arr.ctypes.data, arr.size, 0, None, 0, C.byref(out))


def test_quantized_header_layout_and_info():
    codes, corr, b = _sq8()
    # the offsets the reference's tests poke at: version at 4, kind at 8, dimension at 12
    magic, version, kind, dim, n = struct.unpack_from("<iiiii", b, 0)
    assert (magic, version, kind, dim, n) == (0x5A545156, 1, F.SQ8, 24, 50)
    assert b[:4] == b"VQTZ"
    assert len(b) == 20 + 12 + 50 * (24 + 4)
    assert vx.quantized_bin_info(b) == (F.SQ8, 24, 50)
    words = np.arange(30 * 2, dtype=np.uint64).reshape(30, 2)
    assert vx.quantized_bin_info(F.quantized_bin_bq(words, 100)) == (F.BQ, 100, 30)
    assert vx.quantized_bin_info(F.quantized_bin_fp16(np.zeros((7, 9), np.uint16))) == (F.FP16, 9, 7)
    assert vx.quantized_bin_info(F.quantized_bin_fp16(np.zeros((0, 9), np.uint16))) == (F.FP16, 9, 0)


@pytest.mark.parametrize(
    "mutate,word",
    [
        (lambda b: b[:10], "truncated"),                                         # shorter than the header
        (lambda b: bytes([b[0] ^ 0xFF]) + b[1:], "magic"),
        (lambda b: b[:4] + struct.pack("<i", 999) + b[8:], "version"),
        (lambda b: b[:8] + struct.pack("<i", 0) + b[12:], "NONE"),
        (lambda b: b[:8] + struct.pack("<i", 9999) + b[12:], "invalid quantizerKind"),
        (lambda b: b[: 20 + 12 + 10], "truncated"),                              # vector data cut short
        (lambda b: b[:12] + struct.pack("<i", -1) + b[16:], "dimension"),
        (lambda b: b[:16] + struct.pack("<i", -3) + b[20:], "vectorCount"),
        (lambda b: b[:20] + struct.pack("<i", 7) + b[24:], "ScalarBits"),
        (lambda b: b[:20] + struct.pack("<i", 1) + b[24:], "SQ8 kind but ScalarBits is INT4"),
    ],
)
def test_quantized_rejections_mirror_the_codec(mutate, word):
    _, _, b = _sq8()
    bad = mutate(b)
    with pytest.raises(vx.IOException, match=word):
        vx.quantized_bin_info(bad)
    assert _build_status(bad) == N.VX_ERR_FORMAT  # rejected before any device work
    assert word.split()[0] in N.last_error()


def test_quantized_kinds_not_served():
    packed = np.zeros((5, 6), np.uint8)
    assert vx.quantized_bin_info(F.quantized_bin_sq4(packed, np.zeros(5, np.float32), 12, 0.0, 1.0)) == (F.SQ4, 12, 5)
    with pytest.raises(vx.IOException, match="SQ vector data"):  # ceil(13/2) = 7 bytes a row expected
        vx.quantized_bin_info(F.quantized_bin_sq4(packed, np.zeros(5, np.float32), 13, 0.0, 1.0))
    words = np.zeros((4, 1), np.uint64)
    assert vx.quantized_bin_info(F.quantized_bin_bq(words, 64, np.zeros(64, np.float32),
                                                    np.zeros((4, 3), np.float32))) == (F.BQ, 64, 4)
    wide = np.zeros((2, 17), np.uint64)  # BBQ up to 2048 dimensions is served
    assert vx.quantized_bin_info(F.quantized_bin_bq(wide, 1050, np.zeros(1050, np.float32),
                                                    np.zeros((2, 3), np.float32))) == (F.BQ, 1050, 2)
    big = np.zeros((2, 33), np.uint64)  # beyond 2048 dimensions it is refused
    with pytest.raises(vx.UnsupportedOperationException, match="BBQ"):
        vx.quantized_bin_info(F.quantized_bin_bq(big, 2100, np.zeros(2100, np.float32), np.zeros((2, 3), np.float32)))
    # a PQ payload cut after the header: decodePQ's first ensureRemaining
    pq = struct.pack("<iiiii", F.MAGIC_QUANTIZED, 1, F.PQ, 16, 3)
    with pytest.raises(vx.IOException, match="PQ quantizer state header"):
        vx.quantized_bin_info(pq)
    # a truncated BBQ file is still a format error, as in decodeBQ
    with pytest.raises(vx.IOException, match="BQ centroid"):
        vx.quantized_bin_info(struct.pack("<iiiiii", F.MAGIC_QUANTIZED, 1, F.BQ, 64, 4, F.BBQ))


def test_quantized_pq_payload_decodes_as_decodePQ():
    # QuantizedVectorsCodec.decodePQ (:367-420): state, optional global centroid, subspaces,
    # codebooks, codes; its IOException reasons for each malformed part
    dim, m, ks, n = 16, 4, 8, 3
    cb = np.arange(ks * dim, dtype=np.float32)
    codes = np.zeros((n, m), np.uint8)
    assert vx.quantized_bin_info(F.quantized_bin_pq(codes, cb, dim, m, ks)) == (F.PQ, dim, n)
    assert vx.quantized_bin_info(F.quantized_bin_pq(codes, cb, dim, m, ks, np.ones(dim, np.float32))) == (F.PQ, dim, n)
    head = struct.pack("<iiiii", F.MAGIC_QUANTIZED, 1, F.PQ, dim, n)
    with pytest.raises(vx.IOException, match="numSubspaces must be positive: 0"):
        vx.quantized_bin_info(head + struct.pack("<iii", 0, ks, 0))
    with pytest.raises(vx.IOException, match=r"numClusters must be in \[1, 256\]: 300"):
        vx.quantized_bin_info(head + struct.pack("<iii", m, 300, 0))
    with pytest.raises(vx.IOException, match="hasGlobalCentroid must be 0 or 1: 2"):
        vx.quantized_bin_info(head + struct.pack("<iii", m, ks, 2))
    with pytest.raises(vx.IOException, match="PQ globalCentroid"):
        vx.quantized_bin_info(head + struct.pack("<iii", m, ks, 1))
    with pytest.raises(vx.IOException, match="PQ codebook 0"):
        vx.quantized_bin_info(head + struct.pack("<iii", m, ks, 0) + b"".join(struct.pack("<ii", 4, 4 * i) for i in range(m)))
    with pytest.raises(vx.IOException, match="PQ vector data"):
        vx.quantized_bin_info(F.quantized_bin_pq(codes, cb, dim, m, ks)[:-1])
    odd = F.quantized_bin_pq(codes, cb, dim, m, ks, subs=[(5, 0), (3, 5), (4, 8), (4, 12)])
    with pytest.raises(vx.UnsupportedOperationException, match="computeSubspaceSizesAndOffsets"):
        vx.quantized_bin_info(odd)


def test_quantized_accepts_paths_and_arrays(tmp_path):
    _, _, b = _sq8()
    p = tmp_path / "quantized.bin"
    p.write_bytes(b)
    assert vx.quantized_bin_info(str(p)) == (F.SQ8, 24, 50)
    assert vx.quantized_bin_info(np.memmap(p, dtype=np.uint8, mode="r")) == (F.SQ8, 24, 50)
    assert vx.quantized_bin_info(bytearray(b)) == (F.SQ8, 24, 50)


def _ivf(n=200, dim=32, nlist=6, m=8, ks=16, seed=3):
    rng = np.random.default_rng(seed)
    cent = rng.standard_normal((nlist, dim)).astype(np.float32)
    assign = rng.integers(0, nlist, n)
    ords = np.argsort(assign, kind="stable").astype(np.int32)
    off = np.concatenate([[0], np.cumsum(np.bincount(assign, minlength=nlist))]).astype(np.int64)
    cb = rng.standard_normal(ks * dim).astype(np.float32)  # m subspaces of dim/m floats, ks each
    codes = rng.integers(0, ks, (n, m)).astype(np.uint8)
    return cent, off, ords, cb, codes


def test_ivf_graph_info_roundtrip():
    cent, off, ords, cb, codes = _ivf()
    kd = [None, [0, 3, 5], None, [], None, [1]]
    b = F.ivf_graph_bin(cent, off, ords, vx.SimilarityFunction.EUCLIDEAN, key_dims=kd,
                        pq=dict(m=8, ks=16, codebooks=cb, codes=codes, anisotropic=0.2))
    info = vx.ivf_graph_info(b)
    assert info == {"nlist": 6, "dim": 32, "count": 200, "m": 8, "metric": vx.SimilarityFunction.EUCLIDEAN}
    b2 = F.ivf_graph_bin(cent, off, ords, vx.SimilarityFunction.COSINE, pq=dict(m=8, ks=16, codebooks=cb, codes=codes))
    assert vx.ivf_graph_info(b2)["metric"] == vx.SimilarityFunction.COSINE


def test_ivf_graph_rejections():
    cent, off, ords, cb, codes = _ivf()
    pq = dict(m=8, ks=16, codebooks=cb, codes=codes)
    good = F.ivf_graph_bin(cent, off, ords, 0, pq=pq)
    for cut in (3, 40, len(good) // 2, len(good) - 1):
        with pytest.raises(vx.IOException, match="truncated"):
            vx.ivf_graph_info(good[:cut])
    # IVF-flat (pqFlag 0, or the flag byte absent as in files older than IVF-PQ): m = 0
    flat = F.ivf_graph_bin(cent, off, ords, 0, pq=None)
    assert vx.ivf_graph_info(flat) == {"nlist": 6, "dim": 32, "count": 200, "m": 0,
                                       "metric": vx.SimilarityFunction.EUCLIDEAN}
    assert vx.ivf_graph_info(flat[:-1])["m"] == 0
    arr = np.frombuffer(flat, np.uint8)
    out = C.c_void_p()
    assert N.lib().vx_ivf_graph_build(0, arr.ctypes.data, arr.size, -1, None, 0, 0, 8, 1, C.byref(out)) == \
        N.VX_ERR_NULL_POINTER  # IVF-flat needs the vectors
    with pytest.raises(vx.NullPointerException):
        vx.IvfFlatAdapter().load_graph_bin(flat)
    # an unknown flag byte is IvfIndex.decode's IllegalArgumentException
    at = len(flat) - 1
    with pytest.raises(vx.IllegalArgumentException, match="pqFlag"):
        vx.ivf_graph_info(flat[:at] + b"\x02")
    with pytest.raises(vx.UnsupportedOperationException, match="global centroid"):
        vx.ivf_graph_info(F.ivf_graph_bin(cent, off, ords, 0, pq=dict(pq, global_centroid=np.zeros(32))))
    odd = [(4, 4 * i) for i in range(8)]
    odd[0], odd[1] = (5, 0), (3, 5)
    with pytest.raises(vx.UnsupportedOperationException, match="computeSubspaceSizesAndOffsets"):
        vx.ivf_graph_info(F.ivf_graph_bin(cent, off, ords, 0, pq=dict(pq, subs=odd)))
    bad_ords = ords.copy()
    bad_ords[7] = 200
    with pytest.raises(vx.IOException, match="ordinal"):
        vx.ivf_graph_info(F.ivf_graph_bin(cent, off, bad_ords, 0, pq=pq))
    # the partition count after the buoy must match its centroids
    buoy_len = struct.unpack_from(">i", good, 0)[0]
    at = 4 + buoy_len
    with pytest.raises(vx.IOException, match="partitions"):
        vx.ivf_graph_info(good[:at] + struct.pack(">i", 5) + good[at + 4:])
    out = C.c_void_p()
    arr = np.frombuffer(good[:40], np.uint8)
    assert N.lib().vx_ivf_graph_build(0, arr.ctypes.data, arr.size, -1, None, 0, 0, 8, 1, C.byref(out)) == N.VX_ERR_FORMAT


def test_strided_rows_view():
    from vectors_b200.index_spi import _strided_rows

    mm = np.zeros((10, 112), np.float32)  # a vectors.bin of dim 100: alignUp(400, 64) = 448 bytes per row
    v, stride = _strided_rows(mm[:, :100], 100)
    assert stride == 112 and v.ctypes.data == mm.ctypes.data
    v, stride = _strided_rows(np.ones((4, 8), np.float64), 8)
    assert stride == 8 and v.dtype == np.float32
    with pytest.raises(vx.IllegalArgumentException):
        _strided_rows(np.ones((4, 7), np.float32), 8)


def test_sq4_nibble_layout(oracle):
    # encodeInt4 / unpackInt4 (ScalarQuantizer.java:285-336): low nibble = even dimension
    codes = np.array([[1, 2, 3], [15, 0, 7]], np.int8)
    packed = oracle.sq4_pack(codes)
    assert packed.tolist() == [[0x21, 0x03], [0x0F, 0x07]]
    assert np.array_equal(oracle.sq4_unpack(packed, 3), codes)
    db = oracle.gen_mixture(300, 9, 4, 0.3, 5, 6, True)
    lo, hi = oracle.sq8_train(db)
    p4, c4 = oracle.sq4_encode_all(lo, hi, db)
    u = oracle.sq4_unpack(p4, 9)
    assert u.min() >= 0 and u.max() <= 15 and u.max() == 15
