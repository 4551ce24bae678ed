"""Runner-side hook for the SDC-verifying workloads of this package.

Pantheon's verdict (pantheon.py:1220-1223, applied at :1326) files a failed
result row as a FAULT only for the workloads in ``DIAGNOSTIC_TESTS``; any other
failed workload is INCOMPLETE.  The three binaries built here -- ``quantized_gemm``,
``llm_decode`` and ``mma_virus`` -- compare every batch bitwise with a golden
result, so a failure of theirs is a silent-data-corruption finding, not a run
that did not finish.  Each also prints its mismatch count on a
``  -> Mismatches: <n>`` line.

Each also prints a ``  -> Golden Digest: 0x<16 hex digits>`` line: a digest of
its golden result, which the same arguments make equal on every healthy GPU of
a run.  A GPU whose golden result is wrong passes its own bitwise compares
(every launch matches its wrong golden), so only a comparison across GPUs
shows it.

This module gives the runner these facts without editing it:

* ``install(runner)`` adds the three workloads to ``runner.DIAGNOSTIC_TESTS``;
* ``mismatch_count(stdout)`` and ``golden_digest(stdout)`` read the count and the
  digest from a workload's stdout (the runner holds it as ``out`` where it
  parses each GPU's output, pantheon.py:4158-4269), and
  ``row_fields(test_name, stdout)`` turns them into columns for the result row
  (``build_result_row``, pantheon.py:3552);
* ``check_golden_digests(rows)``, given the result rows of all GPUs of a run,
  marks each row with a digest as agreeing or not with the other GPUs of the
  same workload, and sets the disagreeing rows' ``Status`` to FAIL, which
  ``assess_gpu`` (pantheon.py:1303-1460) files as a FAULT for these workloads
  once ``install`` has run.

The equivalent change inside the runner is three lines: the three names added
to the ``DIAGNOSTIC_TESTS`` literal, ``row.update(row_fields(test_name, out))``
after each GPU's ``build_result_row``, and ``check_golden_digests(results)``
before the verdicts are assessed.
"""
from __future__ import annotations

import re

SDC_VERIFYING_TESTS = frozenset({"quantized_gemm", "llm_decode", "mma_virus"})

ROW_FIELD = "SDC Mismatches"
DIGEST_FIELD = "Golden Digest"
AGREE_FIELD = "Golden Digest Agrees"

_MISMATCH_LINE = re.compile(r"^\s*->\s*Mismatches:\s*(\d+)\s*$")
_DIGEST_LINE = re.compile(r"^\s*->\s*Golden Digest:\s*(0x[0-9a-fA-F]{16})\s*$")


def install(runner) -> frozenset:
    """Add the SDC-verifying workloads to ``runner.DIAGNOSTIC_TESTS`` (idempotent).

    ``runner`` is the imported ``pantheon`` module (or anything with a mutable
    ``DIAGNOSTIC_TESTS`` set).  Returns the names that were added.
    """
    tests = getattr(runner, "DIAGNOSTIC_TESTS", None)
    if not isinstance(tests, set):
        raise TypeError("runner.DIAGNOSTIC_TESTS must be a set of workload names")
    added = frozenset(SDC_VERIFYING_TESTS - tests)
    tests.update(SDC_VERIFYING_TESTS)
    return added


def mismatch_count(stdout: str | None) -> int | None:
    """The workload's reported mismatch count (the last ``-> Mismatches:`` line), or None."""
    count = None
    for line in (stdout or "").splitlines():
        m = _MISMATCH_LINE.match(line)
        if m:
            count = int(m.group(1))
    return count


def golden_digest(stdout: str | None) -> str | None:
    """The workload's golden-result digest (the last ``-> Golden Digest:`` line, lower
    case), or None."""
    digest = None
    for line in (stdout or "").splitlines():
        m = _DIGEST_LINE.match(line)
        if m:
            digest = m.group(1).lower()
    return digest


def row_fields(test_name: str, stdout: str | None) -> dict:
    """Extra result-row columns for one GPU's run of an SDC-verifying workload:
    ``"SDC Mismatches"`` when it ran with ``--verify`` and ``"Golden Digest"`` when it
    printed one; nothing for other workloads."""
    if test_name not in SDC_VERIFYING_TESTS:
        return {}
    fields = {}
    n = mismatch_count(stdout)
    if n is not None:
        fields[ROW_FIELD] = n
    d = golden_digest(stdout)
    if d is not None:
        fields[DIGEST_FIELD] = d
    return fields


def check_golden_digests(rows) -> list:
    """Compare the golden digests of each workload across the GPUs of one run.

    ``rows`` are the run's result rows (``"Test Name"``, ``"GPU ID"`` and, from
    ``row_fields``, ``"Golden Digest"``).  Within each workload the digest that more
    than half of its rows report is taken as right; the rows with another digest
    disagree.  With no such majority (two GPUs that differ, say) no GPU can be
    trusted over the others and every row of that workload disagrees.  Every row
    with a digest gets ``"Golden Digest Agrees"``; a disagreeing row also gets
    ``"Status": "FAIL"``.  Returns the disagreeing rows.
    """
    groups = {}
    for row in rows:
        d = row.get(DIGEST_FIELD)
        if d is not None:
            groups.setdefault(row.get("Test Name"), []).append(row)
    bad = []
    for group in groups.values():
        counts = {}
        for row in group:
            counts[row[DIGEST_FIELD]] = counts.get(row[DIGEST_FIELD], 0) + 1
        top, n = max(counts.items(), key=lambda kv: kv[1])
        right = top if 2 * n > len(group) else None
        for row in group:
            agrees = row[DIGEST_FIELD] == right
            row[AGREE_FIELD] = agrees
            if not agrees:
                row["Status"] = "FAIL"
                bad.append(row)
    return bad
