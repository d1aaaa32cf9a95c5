"""C ABI checks that need no GPU: the library loads, exports exactly what include/vx.h declares,
and the SPI mirror reports the reference's errors (IndexSpi.java, FlatScanAdapter.java:51-175)."""
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "vx.h")).read()
    return sorted(set(re.findall(r"^VX_API\s+[\w\s\*]+?\b(vx_\w+)\(", src, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    import vectors_b200._native as N

    lib = N.lib()
    declared = _declared()
    assert len(declared) >= 19
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(line.split()[-1] for line in out.splitlines() if " T vx_" in line)
    assert exported == declared
    assert sorted(N.exported_symbols()) == declared


def test_abi_version():
    import vectors_b200._native as N

    assert N.lib().vx_abi_version() == 1


def test_no_gpu_reports_gpu_unavailable():
    import vectors_b200 as vx

    if vx.device_count() > 0:
        pytest.skip("a GPU is present")
    f = vx.FlatScanAdapter()
    with pytest.raises(vx.GpuUnavailableException):
        f.build(np.zeros((4, 3), np.float32), vx.SimilarityFunction.COSINE)


def test_injected_failure_maps_to_exception():
    import vectors_b200 as vx
    import vectors_b200._native as N

    N.lib().vx_debug_fail_next(N.VX_ERR_INVALID_ARGUMENT)
    with pytest.raises(vx.IllegalArgumentException, match="injected"):
        vx.FlatScanAdapter().build(np.zeros((4, 3), np.float32), vx.SimilarityFunction.COSINE)
    N.lib().vx_debug_fail_next(N.VX_ERR_CUDA)
    with pytest.raises(vx.GpuUnavailableException, match="injected"):
        vx.FlatScanAdapter().build(np.zeros((4, 3), np.float32), vx.SimilarityFunction.COSINE)


def test_argument_validation_before_gpu():
    import vectors_b200 as vx

    f = vx.FlatScanAdapter()
    with pytest.raises(vx.NullPointerException):
        f.build(None, vx.SimilarityFunction.COSINE)
    with pytest.raises(vx.NullPointerException):
        f.build(np.zeros((2, 2), np.float32), None)
    # empty index: searches return empty outcomes, bad k / empty batch are rejected
    with pytest.raises(vx.IllegalArgumentException):
        f.search_batch([], 3)
    with pytest.raises(vx.IllegalArgumentException):
        f.search_batch([[1.0, 2.0]], 0)
    with pytest.raises(vx.NullPointerException):
        f.search_batch(None, 3)
    with pytest.raises(vx.NullPointerException):
        f.search(None, 3)
    out = f.search_batch([[1.0, 2.0], [3.0, 4.0]], 3)
    assert len(out) == 2 and all(len(o.ordinals) == 0 for o in out)
    # the SPI's default overloads: multi-start and predicate searches delegate to search
    assert len(f.search([1.0, 2.0], 3, 0, 1.0, 4).ordinals) == 0
    assert len(f.search_with_predicate([1.0, 2.0], 3, 0, 1.0, lambda o: o % 2 == 0).ordinals) == 0
    with pytest.raises(vx.IllegalArgumentException):
        f.search_with_predicate([1.0, 2.0], 0, 0, 1.0, lambda o: True)
    with pytest.raises(vx.IllegalArgumentException):
        vx.SearchOutcome(np.zeros(2, np.int32), np.zeros(3, np.float32))


def test_quantized_builds_reject_mismatched_shapes():
    # the C entry points read n x width elements of each array: a mismatch must raise before
    # the library is called (no GPU needed), as a Java array of the wrong length would
    import vectors_b200 as vx

    a = vx.QuantizedFlatScanAdapter()
    dot = vx.SimilarityFunction.DOT_PRODUCT
    codes = np.zeros((5, 8), np.int8)
    with pytest.raises(vx.IllegalArgumentException, match="corrections"):
        a.build_sq8(codes, np.zeros(4, np.float32), -1.0, 1.0, dot)
    with pytest.raises(vx.IllegalArgumentException, match="vectors"):
        a.build_sq8(codes, np.zeros(5, np.float32), -1.0, 1.0, dot, vectors=np.zeros((5, 7), np.float32))
    with pytest.raises(vx.IllegalArgumentException, match="corrections"):
        a.build_sq4(np.zeros((5, 4), np.uint8), np.zeros(6, np.float32), 8, -1.0, 1.0, dot)
    with pytest.raises(vx.IllegalArgumentException, match="words"):
        a.build_bq(np.zeros((5, 1), np.uint64), 100, dot)
    with pytest.raises(vx.IllegalArgumentException, match="vectors"):
        a.build_bq(np.zeros((5, 2), np.uint64), 100, dot, vectors=np.zeros((4, 100), np.float32))
    with pytest.raises(vx.IllegalArgumentException, match="words"):
        a.build_bbq(np.zeros((5, 3), np.uint64), np.zeros((5, 3), np.float32), np.zeros(100, np.float32), 100, dot)
    with pytest.raises(vx.IllegalArgumentException, match="vectors"):
        a.build_fp16(np.zeros((5, 8), np.uint16), dot, vectors=np.zeros((5, 9), np.float32))
    assert a.size() == 0


def test_ivf_builds_reject_mismatched_shapes():
    import vectors_b200 as vx

    cent = np.zeros((4, 16), np.float32)
    off = np.array([0, 2, 3, 5, 6], np.int64)
    ords = np.arange(6, dtype=np.int32)
    cb = np.zeros(256 * 16, np.float32)
    codes = np.zeros((6, 2), np.uint8)
    l2 = vx.SimilarityFunction.EUCLIDEAN
    p = vx.IvfPqAdapter()
    with pytest.raises(vx.IllegalArgumentException, match="list_offsets"):
        p.build_prebuilt(cent, off[:4], ords, cb, codes, 2, 256, l2)
    with pytest.raises(vx.IllegalArgumentException, match="list_ordinals"):
        p.build_prebuilt(cent, off, ords[:5], cb, codes, 2, 256, l2)
    with pytest.raises(vx.IllegalArgumentException, match="codes"):
        p.build_prebuilt(cent, off, ords, cb, codes[:, :1], 2, 256, l2)
    with pytest.raises(vx.IllegalArgumentException, match="codebooks"):
        p.build_prebuilt(cent, off, ords, cb[:100], codes, 2, 256, l2)
    with pytest.raises(vx.IllegalArgumentException, match="vectors"):
        p.build_prebuilt(cent, off, ords, cb, codes, 2, 256, l2, vectors=np.zeros((5, 16), np.float32))
    f = vx.IvfFlatAdapter()
    with pytest.raises(vx.IllegalArgumentException, match="list_ordinals"):
        f.build_prebuilt(cent, off, ords[:4], np.zeros((6, 16), np.float32), l2)


def test_null_pointer_status_from_c():
    import ctypes as C

    import vectors_b200._native as N

    st = N.lib().vx_flat_build(0, None, 5, 4, 4, 0, C.byref(C.c_void_p()))
    assert st in (N.VX_ERR_NULL_POINTER, N.VX_ERR_GPU_UNAVAILABLE)
    assert N.lib().vx_device_count(None) == N.VX_ERR_NULL_POINTER
    assert "null" in N.last_error()


def test_build_argument_statuses_before_the_gpu():
    # shape, pointer and range checks of the newer build calls run before any device work, so
    # these statuses hold with or without a GPU
    import ctypes as C

    import vectors_b200._native as N

    L = N.lib()
    out = C.c_void_p()
    f = np.zeros(64, np.float32)
    w = np.zeros(64, np.uint64)
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    # BBQ: centroid required; more than 2048 dimensions unsupported
    assert L.vx_bbq_build(0, p(w), p(f), None, 1, 64, 1, None, 64, C.byref(out)) == N.VX_ERR_NULL_POINTER
    assert L.vx_bbq_build(0, p(w), p(f), p(f), 1, 3000, 1, None, 3000, C.byref(out)) == N.VX_ERR_UNSUPPORTED
    assert "2048" in N.last_error()
    assert L.vx_bbq_build(0, p(w), p(f), p(f), 1, 0, 1, None, 0, C.byref(out)) == N.VX_ERR_INVALID_ARGUMENT
    # SQ4: codes required for a non-empty index
    assert L.vx_sq4_build(0, None, p(f), 4, 8, -1.0, 1.0, 1, None, 8, C.byref(out)) == N.VX_ERR_NULL_POINTER
    # IVF-flat: partitions validated on the host
    cent = np.zeros((2, 4), np.float32)
    rows = np.zeros((3, 4), np.float32)
    ords = np.array([0, 1, 2], np.int32)
    bad_start = np.array([1, 2, 3], np.int64)
    assert L.vx_ivfflat_build(0, p(cent), 2, 4, p(bad_start), p(ords), p(rows), 3, 4, 0, 1,
                              C.byref(out)) == N.VX_ERR_INVALID_ARGUMENT
    bad_ord = np.array([0, 5, 2], np.int32)
    off = np.array([0, 2, 3], np.int64)
    assert L.vx_ivfflat_build(0, p(cent), 2, 4, p(off), p(bad_ord), p(rows), 3, 4, 0, 1,
                              C.byref(out)) == N.VX_ERR_INVALID_ARGUMENT
    assert "out of range" in N.last_error()
    assert not out.value


def test_pair_split_entry_points_check_arguments_before_the_gpu():
    # vx_ivf_route_dist_device / vx_ivfflat_scan_pairs_device / vx_ivfflat_merge_pairs_device:
    # null handles and buffers are refused before any device work
    import ctypes as C

    import vectors_b200._native as N

    L = N.lib()
    buf = np.zeros(64, np.float32).ctypes.data_as(C.c_void_p)
    assert L.vx_ivf_route_dist_device(None, buf, 1, 4, 1, buf, buf, None) == N.VX_ERR_NULL_POINTER
    assert L.vx_ivfflat_scan_pairs_device(None, buf, 1, 4, 1, 1, buf, buf, buf, None) == N.VX_ERR_NULL_POINTER
    assert L.vx_ivfflat_merge_pairs_device(None, 1, 1, 1, buf, buf, buf, buf, 0.0, buf, buf, buf,
                                           None) == N.VX_ERR_NULL_POINTER
    assert "null" in N.last_error()
