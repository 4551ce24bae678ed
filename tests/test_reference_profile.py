"""The runner's --profile summary lands on the GEMM (no GPU).

Pantheon's --profile wraps a workload in Nsight Compute and summarises the CSV
with summarize_hardware_counter_file, taking the counters of the kernel that
owns most of the profiled runtime (dominant_profiled_kernel,
pantheon.py:3720-3860).  Two captures of the quantized_gemm binary on a B200
are committed (commands in profiles/quantized_gemm_launch_list.md):
  * ncu_launches_qg_all.csv: every launch of the run (fill, golden, warm-up,
    timed batches, verification), as --profile sees it;
  * ncu_launches_qg_timed.csv: the same run filtered to the binary's NVTX range
    of the timed batches (--nvtx --nvtx-include "qg:timed/").
The runner's own summariser must name the INT8 GEMM kernel as the dominant one
in the first, and the second must hold nothing but GEMM launches.
"""
import csv
from pathlib import Path

import pytest

from tests.reference_runner import load_runner

GOLDEN = Path(__file__).resolve().parent / "golden"
ALL = GOLDEN / "ncu_launches_qg_all.csv"
TIMED = GOLDEN / "ncu_launches_qg_timed.csv"


def _rows(path):
    lines = path.read_text().splitlines()
    start = next(i for i, line in enumerate(lines) if "Metric Name" in line and "Metric Value" in line)
    return list(csv.DictReader(lines[start:]))


def _time_by_kernel(path):
    out = {}
    for r in _rows(path):
        if r["Metric Name"].strip() != "gpu__time_duration.sum":
            continue
        scale = {"ns": 1.0, "nsecond": 1.0, "us": 1e3, "usecond": 1e3, "ms": 1e6, "msecond": 1e6,
                 "s": 1e9, "second": 1e9}[r["Metric Unit"].strip()]
        out[r["Kernel Name"]] = out.get(r["Kernel Name"], 0.0) + float(r["Metric Value"].replace(",", "")) * scale
    return out


def test_gemm_owns_the_profiled_runtime():
    t = _time_by_kernel(ALL)
    assert len(t) >= 3                      # the fill / verify kernels are in the capture too
    top = max(t, key=t.get)
    assert "gemm_i8" in top
    assert t[top] / sum(t.values()) > 0.9


def test_nvtx_filtered_capture_holds_only_the_timed_gemms():
    kernels = {r["Kernel Name"] for r in _rows(TIMED)}
    assert kernels and all("gemm_i8" in k for k in kernels)


def test_runner_summary_names_the_gemm():
    runner = load_runner()
    if runner is None:
        pytest.skip("reference runner (pantheon.py) not found; set PANTHEON_REFERENCE")
    s = runner.summarize_hardware_counter_file(str(ALL))
    assert "gemm_i8" in s["Counter Kernel"]
    assert float(s["Counter Kernel Runtime Share"].split()[0]) > 90.0
    assert s["Counter Kernel Launches"] >= 20
