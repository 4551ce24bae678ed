"""Runner-side hook for the SDC-verifying workloads of this package.

Pantheon's verdict (pantheon.py:1220-1223, applied at :1326) files a failed
result row as a FAULT only for the workloads in ``DIAGNOSTIC_TESTS``; any other
failed workload is INCOMPLETE.  The three binaries built here -- ``quantized_gemm``,
``llm_decode`` and ``mma_virus`` -- compare every batch bitwise with a golden
result, so a failure of theirs is a silent-data-corruption finding, not a run
that did not finish.  Each also prints its mismatch count on a
``  -> Mismatches: <n>`` line.

This module gives the runner both facts without editing it:

* ``install(runner)`` adds the three workloads to ``runner.DIAGNOSTIC_TESTS``;
* ``mismatch_count(stdout)`` reads the count from a workload's stdout (the
  runner holds it as ``out`` where it parses each GPU's output,
  pantheon.py:4158-4269), and ``row_fields(test_name, stdout)`` turns it into a
  column for the result row (``build_result_row``, pantheon.py:3552).

The equivalent change inside the runner is two lines: the three names added to
the ``DIAGNOSTIC_TESTS`` literal, and ``row.update(row_fields(test_name, out))``
after each GPU's ``build_result_row``.
"""
from __future__ import annotations

import re

SDC_VERIFYING_TESTS = frozenset({"quantized_gemm", "llm_decode", "mma_virus"})

ROW_FIELD = "SDC Mismatches"

_MISMATCH_LINE = re.compile(r"^\s*->\s*Mismatches:\s*(\d+)\s*$")


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


def row_fields(test_name: str, stdout: str | None) -> dict:
    """Extra result-row columns for one GPU's run: ``{"SDC Mismatches": n}`` for the
    SDC-verifying workloads that ran with ``--verify``, else nothing."""
    if test_name not in SDC_VERIFYING_TESTS:
        return {}
    n = mismatch_count(stdout)
    return {} if n is None else {ROW_FIELD: n}
