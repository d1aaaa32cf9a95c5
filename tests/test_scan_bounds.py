"""The scan epilogue's pass-mask bounds (vectors_b200/csrc/gemm_scan.cu), restated in numpy float32
and checked on the CPU: each must admit every column whose exact score reaches the lane's
threshold tf (a superset; the appends then test the exact keys).

* sq8dot_adj_bound(tf) for SQ8 DOT_PRODUCT / COSINE, score = max((1 + adj) / 2, 0) with NaN
  passing through (ScalarQuantizedVectors.java:88-107), and for BBQ DOT, score =
  max((1 + approx) / 2, 0) with NaN -> 0 (BinaryQuantizedVectors.java:110-275), where tf <= 0
  passes every column;
* bq_min_raw(tf, D) for sign-bit BQ, score = -((D - raw) >> 1) = -h (BinaryQuantizedVectors.java:88-106).
"""
import numpy as np

F = np.float32


def _sq8dot_score(adj):
    h = F(F(F(1) + adj) * F(0.5))
    return h if h >= 0 else (h if h != h else F(0))


def _bbqdot_score(approx):
    s = F(F(F(1) + approx) * F(0.5))
    return s if s > 0 else F(0)


def _sq8dot_adj_bound(tf):
    # the device function: -inf for tf <= 0 or NaN, tf itself once 2 tf would overflow, else
    # (2 tf - 1) less (|2 tf| + 1) * 2^-20
    if not (tf > F(0)):
        return F(-np.inf)
    if not (tf < F(1e38)):
        return tf
    two = F(2) * tf
    return F(F(two - F(1)) - F(F(abs(two) + F(1)) * F(9.5367431640625e-7)))


def _bq_min_raw(tf, d):
    u = F(-tf)
    if not (u >= 0):
        return d + 1
    if u >= F(16777216.0):
        return -d
    return d - 2 * int(np.floor(u)) - 1


def _thresholds(rng):
    return (list(rng.uniform(0, 2, 400).astype(F)) + list((10.0 ** rng.uniform(-45, 38.5, 400)).astype(F))
            + [F(1e-30), F(1e-38), F(1.5e-45), F(0.5), F(0.5000001), F(1), F(3e38), F(1e-7), F(np.inf), F(1e38),
               F(1.7e38), F(-1), F(0), F(-0.0), F(np.nan), F(-np.inf)])


def _values_near(a, rng):
    vals = [F(np.inf), F(-np.inf), F(3.4e38), F(-3.4e38), F(0), F(np.nan)]
    if np.isfinite(a):
        x = a
        for _ in range(48):
            x = np.nextafter(x, F(-np.inf), dtype=F)
        for _ in range(96):
            vals.append(x)
            x = np.nextafter(x, F(np.inf), dtype=F)
        vals += list(rng.normal(float(a), abs(float(a)) * 1e-3 + 1e-6, 40).astype(F))
    return vals


def test_sq8_dot_bound_admits_every_column_reaching_the_threshold():
    rng = np.random.default_rng(0)
    with np.errstate(all="ignore"):
        for tf in _thresholds(rng):
            lo = _sq8dot_adj_bound(tf)
            a = F(F(2) * tf - F(1)) if np.isfinite(tf) and abs(tf) < F(1e38) else F(0)
            for x in _values_near(a, rng):
                if _sq8dot_score(x) >= tf:
                    assert x >= lo, (tf, x, lo)


def test_bbq_dot_bound_admits_every_column_reaching_the_threshold():
    # above 0 the SQ8 bound; at or below 0 the device passes every column (NaN approx included)
    rng = np.random.default_rng(1)
    with np.errstate(all="ignore"):
        for tf in _thresholds(rng):
            lo = _sq8dot_adj_bound(tf)
            a = F(F(2) * tf - F(1)) if np.isfinite(tf) and abs(tf) < F(1e38) else F(0)
            for x in _values_near(a, rng):
                if _bbqdot_score(x) >= tf:
                    assert (not tf > 0) or x >= lo, (tf, x, lo)


def test_bq_raw_bound_admits_every_distance_reaching_the_threshold():
    for d in (8, 96, 100, 1024, 2048):
        tfs = ([F(-x) for x in range(0, d + 3)] + [F(-x - 0.5) for x in range(0, d, 7)]
               + [F(0.5), F(1), F(np.inf), F(-np.inf), F(np.nan), F(-0.0), F(0.0), F(-3e7)])
        for tf in tfs:
            lo = _bq_min_raw(tf, d)
            for h in range(0, d + 1):
                raw = d - 2 * h
                if F(-((d - raw) >> 1)) >= tf:
                    assert raw >= lo, (d, tf, h, lo)
