"""The mma_virus drop-in binary (dense tcgen05 tensor furnace; fp32 on the CUDA cores) on a B200, read the way the
runner reads it.

Same argv and vendor-GEMM flags as the reference's mma_virus (kernels/mma_virus/mma_virus.cpp:
181-441 with kernels/common/vendor_gemm.h:32-55): default BF16 8192^3 with FP32 accumulate,
`--gemm_type bf16|fp16|tf32|fp32|fp8|auto`, `--gemm_size` / `--gemm_m/n/k`; `Throughput: <x> TFLOPS`,
every batch compared bitwise with the first GEMM's output, `Verification: PASS|FAIL (<n> errors)`,
exit 1 on a mismatch.
"""
import subprocess

import pytest

from tests.contract_parse import parse_kernel_output

pytestmark = pytest.mark.gpu


def _run(*args, timeout=600):
    from pantheon_b200 import MMA_BIN_PATH
    return subprocess.run([str(MMA_BIN_PATH), *map(str, args)], capture_output=True, text=True, timeout=timeout)


def test_default_furnace_verifies(cuda_device):
    """No flags beyond the runner's: BF16 8192^3, as `TEST_REGISTRY["mma_virus"]` launches it."""
    p = _run(0, 2, 50, "--verify")
    assert p.returncode == 0, p.stdout + p.stderr
    t, unit, status, _, kept = parse_kernel_output(p.stdout, p.stderr, p.returncode, "mma_virus")
    assert status == "PASS" and unit == "TFLOPS" and t > 200.0
    assert "Tensor Engine: tcgen05 GEMM (BF16 8192x8192x8192, FP32 accumulate)" in p.stdout
    assert "Verification: PASS (0 errors)" in p.stdout


@pytest.mark.parametrize("gemm_type, name", [("fp16", "FP16"), ("tf32", "TF32"), ("fp8", "FP8 (E4M3)"),
                                             ("BF16", "BF16"), ("fp32", "FP32")])
def test_gemm_types_verify(cuda_device, gemm_type, name):
    p = _run(0, 1, 50, "--verify", "--gemm_type", gemm_type, "--gemm_size", 4096)
    assert p.returncode == 0, p.stdout + p.stderr
    t, unit, status, _, _ = parse_kernel_output(p.stdout, p.stderr, p.returncode, "mma_virus")
    assert status == "PASS" and unit == "TFLOPS" and t > 0
    assert f"({name} 4096x4096x4096" in p.stdout
    engine = "CUDA-core FP32 GEMM" if name == "FP32" else "tcgen05 GEMM"
    assert f"Tensor Engine: {engine} ({name} 4096x4096x4096" in p.stdout


def test_gemm_shape_flags_round_to_16(cuda_device):
    """vendor_gemm.h:537: m, n, k are rounded down to multiples of 16."""
    p = _run(0, 1, 50, "--verify", "--gemm_m", 1000, "--gemm_n", 520, "--gemm_k", 777)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "(BF16 992x512x768, FP32 accumulate)" in p.stdout


def test_injected_fault_fails(cuda_device):
    p = _run(0, 1, 50, "--verify", "--inject_error", "--gemm_size", 2048)
    assert p.returncode == 1
    assert "Verification: FAIL" in p.stdout
    assert "[SDC FAULT][MMA_VIRUS]" in p.stdout
    assert parse_kernel_output(p.stdout, p.stderr, p.returncode, "mma_virus")[2] == "FAIL"
    from pantheon_b200 import runner_hook
    assert runner_hook.row_fields("mma_virus", p.stdout)["SDC Mismatches"] >= 1


def test_auto_picks_a_format(cuda_device):
    """vendor_gemm.h:426-505: every format is probed; BF16 stays unless another leads by the margin."""
    p = _run(0, 1, 50, "--verify", "--gemm_type", "auto", "--gemm_probe_ms", 200, "--gemm_size", 4096)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "-> Selected " in p.stdout
    if "No energy meter" not in p.stdout:
        for name in ("BF16", "FP16", "TF32", "FP8 (E4M3)", "FP32"):
            assert f"-> Probe {name}:" in p.stdout
    assert parse_kernel_output(p.stdout, p.stderr, p.returncode, "mma_virus")[2] == "PASS"


def test_reference_wmma_knobs_are_ignored(cuda_device):
    p = _run(0, 1, 50, "--verify", "--block_size", 256, "--grid_size", 0, "--kernel_loops", 10000, "--sync_mode", 2,
             "--mma_acc", 16, "--mma_groups", 4, "--mma_reuse", 1, "--init_pattern", 1, "--gemm", 1,
             "--gemm_size", 2048)
    assert p.returncode == 0, p.stdout + p.stderr
    assert parse_kernel_output(p.stdout, p.stderr, p.returncode, "mma_virus")[2] == "PASS"
