"""Restatement of how Pantheon's runner reads a workload's output, for the tests.

Follows parse_kernel_output (pantheon.py:3421-3513) and find_skip_reason
(pantheon.py:3404-3418) of the reference, rule by rule:
  * a non-zero exit code is a FAIL with unit ERR;
  * every "Throughput: <value> <unit>" line is read with any whitespace; the
    last one is the score; a non-finite value is a FAIL;
  * "[SDC FAULT]" anywhere is a FAIL;
  * "Verification: FAIL..." is a FAIL even with exit code 0;
  * "Skipping..." with no error is a SKIP; a zero throughput without a skip is a FAIL;
  * "[PANTHEON]" lines and lines starting with "->" are kept for the log, with
    the runner's own notes (non-finite score, zero score, skip reason) and,
    after a non-zero exit, stderr.
Written for the tests only: the GPU tests read live binary output with it where
the runner module is not available.  tests/test_reference_runner.py pins it to
the runner's own decisions on recorded B200 runs (tests/golden/runner_readings.json).
"""
from __future__ import annotations

import math


def find_skip_reason(out: str, err: str = ""):
    for text in (out, err):
        for line in (text or "").splitlines():
            line = line.strip()
            if line.startswith("Skipping"):
                return line
            if "Skipping" in line and ("[PANTHEON]" in line or line.startswith("->")):
                return line
    return None


def parse_kernel_output(out: str, err: str, returncode: int, test_name: str | None = None):
    throughput, unit, status, had_error = "N/A", "", "PASS", False
    lines_kept = []
    throughput_line = False
    skipped = find_skip_reason(out, err)
    if returncode != 0:
        throughput, unit, status, had_error = 0.0, "ERR", "FAIL", True
    for line in (out or "").split("\n"):
        if "Throughput:" in line:
            try:
                parts = line.split("Throughput:")[1].strip().split()
                value = float(parts[0])
            except (ValueError, IndexError):
                continue
            if not math.isfinite(value):
                if not had_error:
                    lines_kept.append(f"[PANTHEON] Workload reported a non-finite throughput ({parts[0]}); "
                                      "recorded as a failure.")
                throughput, unit, status, had_error = 0.0, "ERR", "FAIL", True
                continue
            if not had_error:
                throughput, throughput_line = value, True
                if len(parts) > 1:
                    unit = parts[1]
        elif "[SDC FAULT]" in line:
            throughput, unit, status, had_error = 0.0, "ERR", "FAIL", True
            lines_kept.append(line.strip())
        elif line.strip().startswith("Verification:"):
            verdict = line.split("Verification:", 1)[1].strip().upper()
            if verdict.startswith("FAIL"):
                throughput, unit, status, had_error = 0.0, "ERR", "FAIL", True
            lines_kept.append(line.strip())
        elif "[PANTHEON]" in line or line.strip().startswith("->"):
            lines_kept.append(line.strip())
    if skipped and not had_error:
        throughput, unit, status = 0.0, "SKIP", "SKIP"
        if skipped not in lines_kept:
            lines_kept.append(skipped)
    elif not had_error and throughput_line and throughput == 0.0 and test_name not in (None, "baseline_metrics"):
        unit, status, had_error = "ERR", "FAIL", True
        lines_kept.append("[PANTHEON] Workload reported zero throughput without saying it skipped; "
                          "recorded as a failure.")
    if err and returncode != 0:
        lines_kept.append(err.strip())
    return throughput, unit, status, had_error, lines_kept
