"""The dense tensor-furnace GEMMs held to the reference's own furnace GEMM, on a B200.

The reference's mma_virus drives cuBLASLt through its PantheonGemm
(kernels/common/vendor_gemm.h:197-360).  oracle/_ref/vendor_gemm_check (built
by oracle/Makefile from the reference's header where it lies, plus
oracle/vendor_gemm_check.cu) initialises that object at one format and shape
-- it allocates and fills its own operands with its own generator -- runs it
once, runs this library's GEMM of the same format on the same device
operands, and compares the outputs element by element.  Bar: every element
within 1e-2 of max(|ref|, rms(ref)) (the furnace's outputs are bf16 / fp16 /
fp32 of fp32 accumulations in different orders), and no non-finite values.
"""
import json
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

CHECK = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "vendor_gemm_check"


@pytest.mark.parametrize("fmt", ["bf16", "fp16", "tf32", "fp8", "fp32"])
@pytest.mark.parametrize("shape", [(1024, 1024, 1024), (4096, 4096, 4096), (768, 1280, 2048)])
def test_matches_the_reference_furnace_gemm(cuda_device, qglib, fmt, shape):
    if not CHECK.exists():
        pytest.fail("oracle/_ref/vendor_gemm_check was not built (make -C oracle with the reference tree)")
    p = subprocess.run([str(CHECK), fmt, *map(str, shape)], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout + p.stderr
    r = json.loads(p.stdout.strip().splitlines()[-1])
    if "unavailable" in r:
        pytest.skip(f"the reference's GEMM cannot run here: {r['unavailable']}")
    assert r["nonfinite"] == 0
    assert r["over_1e-2"] == 0, r
    assert r["max_rel"] < 1e-2, r
