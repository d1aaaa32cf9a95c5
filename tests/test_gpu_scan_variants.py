"""The 1-CTA tcgen05 scan, the scan without the pilot sweep or without pooled floors, the
fp16 scans of wide streams on 4 epilogue warps instead of 8, the
popcount BQ / BBQ scans, BQ / BBQ on the tensor scan in row windows, searches split into several query chunks (small scratch budget) and the
IVF-PQ scan with one table per (query, list) pair agree with the oracle too (each variant in
its own process: the library reads the switches once)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# bq_windows: BQ / BBQ above the int8 operand budget on the tensor scan in 23,296-row windows
# (96 dims: 128 bytes per row, 3 MB per window), six windows for the 120k rows
@pytest.mark.parametrize("env", [{"VX_GEMM_1SM": "1"}, {"VX_SCAN_PILOT": "0"},
                                 {"VX_BQ_TENSOR_BYTES": "0", "VX_BQ_WINDOW_BYTES": "0"},
                                 {"VX_BQ_TENSOR_BYTES": "0", "VX_BQ_WINDOW_BYTES": "3000000"},
                                 {"VX_SCRATCH_BYTES": "50000000"}, {"VX_SCAN_POOL": "0"}, {"VX_EPI_WARPS": "4"}],
                         ids=["one_cta", "no_pilot", "bq_popcount", "bq_windows", "query_chunks", "no_pooled_floors",
                              "four_epilogue_warps"])
def test_scan_variant_matches_oracle(env):
    e = dict(os.environ)
    e.update(env)
    e["PYTHONPATH"] = ROOT + os.pathsep + e.get("PYTHONPATH", "")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "variant_child.py")], env=e,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "variant ok" in r.stdout


@pytest.mark.parametrize("env", [{"VX_ADC_GROUPED": "0"}], ids=["per_pair_tables"])
def test_adc_variant_matches_oracle(env):
    e = dict(os.environ)
    e.update(env)
    e["PYTHONPATH"] = ROOT + os.pathsep + e.get("PYTHONPATH", "")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "variant_child.py"), "ivf"], env=e,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "variant ok" in r.stdout
