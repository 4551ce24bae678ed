"""The quantized_gemm drop-in binary on a B200, read the way the runner reads it.

Mirrors the reference CI's clean/inject pair (.github/workflows/ci.yml:81-101;
tests/test_kernel_contract.py:174-183): a clean `--verify` run must print
`Verification: PASS` and exit 0; `--inject_error` must print FAIL (plus an
[SDC FAULT] line) and exit non-zero; output goes through the runner's parse rules.
"""
import subprocess

import pytest

from tests.contract_parse import parse_kernel_output

pytestmark = pytest.mark.gpu


def _run(*args, timeout=600):
    from pantheon_b200 import BIN_PATH
    return subprocess.run([str(BIN_PATH), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def test_device_check_accepts_the_b200(cuda_device, qglib):
    """qg_device_check is QG_OK on the sm_100 device (elsewhere the binaries print Skipping: and exit 0)."""
    assert qglib.qg_device_check(0) == 0


def test_clean_verify_passes(cuda_device):
    p = _run(0, 2, 50, "--verify", "--m", 2048, "--n", 2048, "--k", 2048)
    assert p.returncode == 0, p.stdout + p.stderr
    t, unit, status, err, kept = parse_kernel_output(p.stdout, p.stderr, p.returncode, "quantized_gemm")
    assert status == "PASS" and unit == "TOPS" and t > 0
    assert "Verification: PASS (0 mismatches)" in p.stdout
    assert any(line.startswith("-> Mismatches:") for line in kept)


def test_injected_fault_fails(cuda_device):
    p = _run(0, 1, 50, "--verify", "--inject_error", "--m", 1024, "--n", 1024, "--k", 1024)
    assert p.returncode != 0
    assert "Verification: FAIL" in p.stdout
    assert "[SDC FAULT]" in p.stdout
    assert parse_kernel_output(p.stdout, p.stderr, p.returncode, "quantized_gemm")[2] == "FAIL"
    # the runner hook reads the binary's count line (what the runner would record in the row)
    from pantheon_b200 import runner_hook
    assert runner_hook.row_fields("quantized_gemm", p.stdout)["SDC Mismatches"] >= 1


def test_default_configuration_runs(cuda_device):
    """No shape flags: configs[1] (INT8 8192^3, bf16 out), as the runner launches it."""
    p = _run(0, 2, 99, "--verify")
    assert p.returncode == 0, p.stdout + p.stderr
    t, unit, status, _, _ = parse_kernel_output(p.stdout, p.stderr, p.returncode, "quantized_gemm")
    assert status == "PASS" and unit == "TOPS" and t > 100.0


def test_unknown_flags_are_ignored(cuda_device):
    p = _run(0, 1, 50, "--verify", "--block_size", 128, "--grid_size", 7, "--sync_mode", 1, "--frobnicate",
             "--m", 512, "--n", 512, "--k", 512, "--kernel_loops", 5, "--warmup_iters", 1)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "Verification: PASS" in p.stdout


@pytest.mark.parametrize("fmt,shape", [("fp8", (1024, 1024, 2048)), ("nvfp4", (1024, 1024, 2048)), ("w4a16", (4, 4096, 2048))])
def test_other_formats_verify(cuda_device, fmt, shape):
    m, n, k = shape
    p = _run(0, 1, 50, "--verify", "--format", fmt, "--m", m, "--n", n, "--k", k)
    assert p.returncode == 0, p.stdout + p.stderr
    t, unit, status, _, _ = parse_kernel_output(p.stdout, p.stderr, p.returncode, "quantized_gemm")
    assert status == "PASS" and t > 0 and unit == ("GB/s" if fmt == "w4a16" else "TOPS")
    pi = _run(0, 1, 50, "--verify", "--inject_error", "--format", fmt, "--m", m, "--n", n, "--k", k)
    assert pi.returncode != 0 and "[SDC FAULT]" in pi.stdout


def _loops(stdout: str) -> int:
    return int(next(line for line in stdout.splitlines() if "-> Kernel Loops:" in line).split(":")[1])


@pytest.mark.parametrize("value", [-1, 0])
def test_invalid_kernel_loops_use_one(cuda_device, value):
    """normalize_kernel_launch_config (common.h:285-288): kernel_loops < 1 warns and uses 1."""
    p = _run(0, 1, 50, "--verify", "--m", 512, "--n", 512, "--k", 512, "--kernel_loops", value)
    assert p.returncode == 0, p.stdout + p.stderr
    assert f"invalid kernel_loops {value}; using 1." in p.stderr
    assert _loops(p.stdout) == 1
    assert "Verification: PASS" in p.stdout


def test_huge_kernel_loops_clamped_and_batch_bounded(cuda_device):
    """Above 1e6 the reference clamps to 1e6 (common.h:289-297); a batch is further capped at
    about one second of measured launch time, so a batch (the unit of verification) always
    ends well inside the run's duration and the runner's kill timeout."""
    p = _run(0, 1, 50, "--verify", "--m", 2048, "--n", 2048, "--k", 2048, "--kernel_loops", 2000000000)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "clamping to 1000000." in p.stderr
    assert "per batch)." in p.stderr
    loops = _loops(p.stdout)
    assert 1 <= loops < 1000000
    assert "Verification: PASS" in p.stdout


def test_invalid_warmup_iters_use_zero(cuda_device):
    """common.h:300-304: warmup_iters < 0 warns and uses 0."""
    p = _run(0, 1, 50, "--verify", "--m", 512, "--n", 512, "--k", 512, "--warmup_iters", -1)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "invalid warmup_iters -1; using 0." in p.stderr
    assert "Verification: PASS" in p.stdout
