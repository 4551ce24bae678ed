"""The runner hook for the SDC-verifying workloads (no GPU): install into the reference
runner module itself (pantheon.py, found as tests/reference_runner.py describes), and
the mismatch count read from a workload's stdout as the binaries print it.  The
verdicts the hook changes are checked on recorded B200 runs in
tests/test_reference_runner.py."""
import types

import pytest

from pantheon_b200 import runner_hook
from tests.contract_parse import parse_kernel_output
from tests.reference_runner import load_runner


def test_install_adds_the_three_workloads_once():
    r = load_runner()
    if r is None:
        pytest.skip("reference runner (pantheon.py) not found; set PANTHEON_REFERENCE")
    before = set(r.DIAGNOSTIC_TESTS)
    assert not before & runner_hook.SDC_VERIFYING_TESTS
    added = runner_hook.install(r)
    assert added == {"quantized_gemm", "llm_decode", "mma_virus"}
    assert r.DIAGNOSTIC_TESTS == before | added
    assert runner_hook.install(r) == frozenset()
    # the names are the runner's own workload names (its registry), so its verdict finds them
    assert {r.TEST_REGISTRY[t]["bin"] for t in added} == set(added)


def test_install_needs_a_set():
    with pytest.raises(TypeError):
        runner_hook.install(types.SimpleNamespace())


FAILED_RUN = """[PANTHEON] GPU 0: Quantized GEMM (INT8 W8A8, sm_100a)
  -> Working Set:   640 MiB (1 operand copy)
Throughput: 2650.2 TOPS
[SDC FAULT][QUANTIZED_GEMM] Output mismatch! Word: 0 | Exp: 0x3f803f80 | Act: 0x3f803f00 | XOR: 0x00000080
  -> Mismatches:    1
Verification: FAIL (1 mismatches)
"""


def test_mismatch_count_and_row_fields():
    assert runner_hook.mismatch_count(FAILED_RUN) == 1
    assert runner_hook.row_fields("quantized_gemm", FAILED_RUN) == {"SDC Mismatches": 1}
    assert runner_hook.row_fields("march_test", FAILED_RUN) == {}
    clean = FAILED_RUN.replace("  -> Mismatches:    1", "  -> Mismatches:    0")
    assert runner_hook.row_fields("mma_virus", clean) == {"SDC Mismatches": 0}
    assert runner_hook.mismatch_count("Throughput: 1 TOPS\n") is None
    assert runner_hook.row_fields("llm_decode", "Throughput: 1 GB/s\n") == {}
    # the runner keeps the line in its log as well (lines starting with "->")
    kept = parse_kernel_output(FAILED_RUN, "", 1, "quantized_gemm")[4]
    assert "-> Mismatches:    1" in kept


def test_binary_prints_the_line_the_hook_reads():
    """The count line format in the binaries' source matches what the hook parses."""
    from pathlib import Path
    src = (Path(__file__).resolve().parent.parent / "pantheon_b200" / "csrc" / "quantized_gemm_main.cpp").read_text()
    assert '"  -> Mismatches:    " << mismatches' in src
    assert runner_hook.mismatch_count("  -> Mismatches:    12345") == 12345


CLEAN_RUN = """[PANTHEON] GPU 0: Quantized GEMM (INT8 W8A8, sm_100a)
  -> Working Set:   385 MiB (1 operand copy)
  -> Golden Digest: 0x{digest}
Throughput: 2665.02 TOPS
  -> Mismatches:    0
Verification: PASS (0 mismatches)
"""


def test_golden_digest_and_row_fields():
    out = CLEAN_RUN.format(digest="9E3779B97F4A7C15")
    assert runner_hook.golden_digest(out) == "0x9e3779b97f4a7c15"
    assert runner_hook.row_fields("quantized_gemm", out) == {"SDC Mismatches": 0, "Golden Digest": "0x9e3779b97f4a7c15"}
    assert runner_hook.golden_digest("  -> Golden Digest: 0x123\n") is None   # 16 hex digits or nothing
    assert runner_hook.row_fields("march_test", out) == {}
    # the runner keeps the line in its log
    assert "-> Golden Digest: 0x9E3779B97F4A7C15" in parse_kernel_output(out, "", 0, "quantized_gemm")[4]


def _rows(test, digests):
    return [{"Test Name": test, "GPU ID": g, "Status": "PASS", "Golden Digest": d} for g, d in enumerate(digests)]


def test_check_golden_digests_majority_and_ties():
    a, b = "0x" + "a" * 16, "0x" + "b" * 16
    rows = _rows("quantized_gemm", [a, a, b, a]) + _rows("llm_decode", [a, b]) + _rows("mma_virus", [b, b])
    rows.append({"Test Name": "quantized_gemm", "GPU ID": 9, "Status": "PASS"})   # no digest: untouched
    bad = runner_hook.check_golden_digests(rows)
    # quantized_gemm: GPU 2 is the outlier; llm_decode: two GPUs that differ, neither trusted
    assert sorted((r["Test Name"], r["GPU ID"]) for r in bad) == [("llm_decode", 0), ("llm_decode", 1),
                                                                  ("quantized_gemm", 2)]
    assert all(r["Status"] == "FAIL" and r["Golden Digest Agrees"] is False for r in bad)
    good = [r for r in rows if r not in bad and "Golden Digest" in r]
    assert len(good) == 5 and all(r["Status"] == "PASS" and r["Golden Digest Agrees"] is True for r in good)
    assert "Golden Digest Agrees" not in rows[-1]
    assert runner_hook.check_golden_digests(_rows("quantized_gemm", [a])) == []   # one GPU agrees with itself


def test_binary_prints_the_digest_line_the_hook_reads():
    from pathlib import Path
    src = (Path(__file__).resolve().parent.parent / "pantheon_b200" / "csrc" / "quantized_gemm_main.cpp").read_text()
    assert '"  -> Golden Digest: " << hex' in src and '"0x%016llx"' in src
