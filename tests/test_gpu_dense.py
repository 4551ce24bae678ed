"""Tensor-furnace GEMMs (bf16 and e4m3 operands, fp32 accumulate) on the tcgen05 path
against the CPU oracle: f32 output within 1e-4 relative (accumulation order), bf16
output within 1e-2 (|y - ref| <= tol * max(|ref|, rms(ref))).  M >= 256 runs on CTA pairs."""
import numpy as np
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu

SHAPES = [(128, 256, 256), (130, 200, 512), (256, 512, 1024), (1000, 1000, 1024), (384, 128, 2048), (64, 1, 64)]


def _operands(kind, M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((M + N, K), generator=g)
    if kind == 1:
        t = x.to(torch.bfloat16)
        bits = t.view(torch.int16).numpy().view(np.uint16)
    else:
        t = (x * 40).to(torch.float8_e4m3fn)
        bits = t.view(torch.uint8).numpy()
    return t[:M].contiguous(), t[M:].contiguous(), bits[:M], bits[M:]


@pytest.mark.parametrize("kind", [1, 2], ids=["bf16", "e4m3"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_dense_gemm_matches_oracle(cuda_device, oracle, kind, shape):
    M, N, K = shape
    if kind == 2 and K % 16:
        pytest.skip("e4m3 rows must be a multiple of 16 bytes")
    tA, tB, A, B = _operands(kind, M, N, K, seed=M + N + K + kind)
    dA = (tA if kind == 1 else tA.view(torch.uint8)).to(cuda_device)
    dB = (tB if kind == 1 else tB.view(torch.uint8)).to(cuda_device)
    f = pb.gemm_bf16 if kind == 1 else pb.gemm_e4m3
    y32 = f(dA, dB, alpha=0.75, out_type=pb.QG_OUT_F32)
    ybf = f(dA, dB, alpha=0.75, out_type=pb.QG_OUT_BF16)
    torch.cuda.synchronize()
    assert pb.device_status(0) == 0
    ref32 = oracle.gemm_dense(kind, A, B, alpha=0.75, out_type=1)
    assert oracle.max_rel_err(y32.cpu().numpy(), ref32, 1) < 1e-4
    refbf = oracle.gemm_dense(kind, A, B, alpha=0.75, out_type=0)
    assert oracle.max_rel_err(ybf.view(torch.int16).cpu().numpy().view(np.uint16), refbf, 0) < 1e-2


def test_dense_gemm_is_reproducible(cuda_device):
    """A deterministic kernel reproduces itself bit for bit (the furnace's verification rule)."""
    g = torch.Generator().manual_seed(3)
    A = torch.randn((2048, 2048), generator=g).to(torch.bfloat16).to(cuda_device)
    B = torch.randn((1024, 2048), generator=g).to(torch.bfloat16).to(cuda_device)
    a = pb.gemm_bf16(A, B)
    b = pb.gemm_bf16(A, B)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
