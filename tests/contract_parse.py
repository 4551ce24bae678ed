"""Restatement of how Pantheon's runner reads a workload's output, for the tests.

Follows parse_kernel_output (pantheon.py:3421-3513) and find_skip_reason
(pantheon.py:3404-3418) of the reference, rule by rule:
  * a non-zero exit code is a FAIL with unit ERR;
  * every "Throughput: <value> <unit>" line is read with any whitespace; the
    last one is the score; a non-finite value is a FAIL;
  * "[SDC FAULT]" anywhere is a FAIL;
  * "Verification: FAIL..." is a FAIL even with exit code 0;
  * "Skipping..." with no error is a SKIP; a zero throughput without a skip is a FAIL;
  * "[PANTHEON]" lines and lines starting with "->" are kept for the log.
Written for the tests only; the runner itself is not part of this repository.
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
    elif not had_error and throughput_line and throughput == 0.0 and test_name not in (None, "baseline_metrics"):
        unit, status, had_error = "ERR", "FAIL", True
    return throughput, unit, status, had_error, lines_kept
