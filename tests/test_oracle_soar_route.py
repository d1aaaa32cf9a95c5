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
