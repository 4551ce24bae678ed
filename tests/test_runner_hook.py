"""The runner hook for the SDC-verifying workloads (no GPU): install into a stand-in
runner module, and the mismatch count read from a workload's stdout as the binaries
print it."""
import types

import pytest

from pantheon_b200 import runner_hook
from tests.contract_parse import parse_kernel_output


def _runner():
    # the reference's own set at pantheon.py:1220-1223
    return types.SimpleNamespace(DIAGNOSTIC_TESTS={
        "march_test", "galpat", "memory_hammer", "memory_retention", "memory_retention_bake", "ras_validator"})


def test_install_adds_the_three_workloads_once():
    r = _runner()
    added = runner_hook.install(r)
    assert added == {"quantized_gemm", "llm_decode", "mma_virus"}
    assert {"march_test", "quantized_gemm", "llm_decode", "mma_virus"} <= r.DIAGNOSTIC_TESTS
    assert runner_hook.install(r) == frozenset()
    assert len(r.DIAGNOSTIC_TESTS) == 9


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
