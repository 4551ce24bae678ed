"""The llm_decode drop-in binary (W4A16 decode GEMV) on a B200, read the way the runner reads it.

Same argv and flags as the reference's llm_decode (kernels/llm_decode/llm_decode.cpp:59-115);
`Throughput:` in GB/s (the decode step is a stream over the weights), tokens/s on an
"  -> Tokens/s:" log line, `Verification: PASS|FAIL`, exit 1 on a mismatch.
"""
import subprocess

import pytest

from tests.contract_parse import parse_kernel_output

pytestmark = pytest.mark.gpu


def _run(*args, timeout=600):
    from pantheon_b200 import DECODE_BIN_PATH
    return subprocess.run([str(DECODE_BIN_PATH), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def test_default_decode_verifies(cuda_device):
    """No shape flags: configs[3] at M=1 (K=8192, N=28672), as the runner launches llm_decode."""
    p = _run(0, 2, 50, "--verify")
    assert p.returncode == 0, p.stdout + p.stderr
    t, unit, status, _, kept = parse_kernel_output(p.stdout, p.stderr, p.returncode, "llm_decode")
    assert status == "PASS" and unit == "GB/s" and t > 500.0
    assert "LLM Decode" in p.stdout
    assert any(line.startswith("-> Tokens/s:") for line in kept)
    assert "Verification: PASS (0 mismatches)" in p.stdout


@pytest.mark.parametrize("m", [8, 16])
def test_decode_batches_verify(cuda_device, m):
    p = _run(0, 1, 50, "--verify", "--m", m)
    assert p.returncode == 0, p.stdout + p.stderr
    t, unit, status, _, _ = parse_kernel_output(p.stdout, p.stderr, p.returncode, "llm_decode")
    assert status == "PASS" and unit == "GB/s" and t > 0


def test_decode_injected_fault_fails(cuda_device):
    p = _run(0, 1, 50, "--verify", "--inject_error", "--n", 4096, "--k", 4096)
    assert p.returncode != 0
    assert "Verification: FAIL" in p.stdout
    assert "[SDC FAULT][LLM_DECODE]" in p.stdout
    assert parse_kernel_output(p.stdout, p.stderr, p.returncode, "llm_decode")[2] == "FAIL"


def test_decode_reference_flags_accepted(cuda_device):
    """The reference's launch knobs parse (and clamp) without changing the contract."""
    p = _run(0, 1, 30, "--verify", "--block_size", 512, "--grid_size", 0, "--kernel_loops", 7, "--warmup_iters", 2,
             "--sync_mode", 2, "--n", 2048, "--k", 2048)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "Kernel Loops:  7" in p.stdout
