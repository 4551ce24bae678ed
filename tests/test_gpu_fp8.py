"""FP8 e4m3 block-128 tcgen05 GEMM: parity with the CPU oracle, through the C ABI.

M=N=8192, K=16384; values N(0,1) with each block's absmax mapped to
448; fp32 1x128 (A) and 128x128 (B) scales; fp32 accumulation promoted per
K block; bf16 output; tolerance 1e-2 relative (|y - ref| <= 1e-2 * max(|ref|,
rms(ref))).  The tensor core's fp32 partial of a K block may round differently
from the oracle's exact partial, so the bar is the tolerance; the fp32 output
is additionally held to 1e-5.  The device quantiser must reproduce the
oracle's e4m3 bytes and scales bit for bit.
"""
import numpy as np
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu
RTOL = 1e-2


def _np(t):
    return t.detach().cpu().numpy()


def test_quantiser_matches_oracle(cuda_device, oracle):
    M, N, K = 130, 300, 512
    A, B, sa, sb = pb.gen_fp8(M, N, K, seed=6, tid0=8)
    rA, rB, rsa, rsb = oracle.fp8_operands(M, N, K, seed=6, copy=1)
    np.testing.assert_array_equal(_np(A), rA)
    np.testing.assert_array_equal(_np(B), rB)
    np.testing.assert_array_equal(_np(sa).view(np.uint32), rsa.view(np.uint32))
    np.testing.assert_array_equal(_np(sb).view(np.uint32), rsb.view(np.uint32))


SHAPES = [(128, 256, 128), (256, 512, 1024), (130, 200, 384), (1, 17, 128), (1000, 1000, 2048), (384, 128, 4096),
          (512, 136, 256), (768, 64, 128), (300, 1100, 640)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gemm_fp8_matches_oracle(cuda_device, oracle, shape):
    M, N, K = shape
    A, B, sa, sb = oracle.fp8_operands(M, N, K, seed=M + 3 * N + K)
    d = [torch.from_numpy(x).to(cuda_device) for x in (A, B, sa, sb)]
    y32 = pb.gemm_fp8_b128(*d, out_type=pb.QG_OUT_F32)
    ybf = pb.gemm_fp8_b128(*d, out_type=pb.QG_OUT_BF16)
    torch.cuda.synchronize()
    assert pb.device_status(0) == 0
    ref32 = oracle.gemm_fp8(A, B, sa, sb, out_type=1)
    assert oracle.max_rel_err(_np(y32), ref32, 1) < 1e-5
    refbf = oracle.gemm_fp8(A, B, sa, sb, out_type=0)
    assert oracle.max_rel_err(_np(ybf.view(torch.int16)).view(np.uint16), refbf, 0) < RTOL


def test_full_size_config2_sampled_rows(cuda_device, oracle):
    """configs[2] at full size: 12 sampled rows against the oracle, then bitwise self-reproduction."""
    M, N, K = 8192, 8192, 16384
    with pb.Workload(pb.QG_FMT_FP8, M, N, K, seed=2) as w:
        w.fill(2)
        w.golden()
        A = _np(w.tensor(0, 0)).reshape(M, K)
        B = _np(w.tensor(0, 1)).reshape(N, K)
        sa = _np(w.tensor(0, 2, torch.float32)).reshape(M, K // 128)
        sb = _np(w.tensor(0, 3, torch.float32)).reshape(N // 128, K // 128)
        Y = _np(w.tensor(0, w.SLOT_OUT, torch.int16)).view(np.uint16).reshape(M, N)
        rows = np.array([0, 127, 128, 4097, 8191] + list(np.random.default_rng(2).integers(0, M, 7)), dtype=np.int32)
        ref = oracle.gemm_fp8(A, B, sa, sb, out_type=0, rows=rows)
        assert oracle.max_rel_err(Y[rows].copy(), ref, 0) < RTOL
        w.run(3)
        assert w.verify() == 0
        assert pb.device_status(0) == 0
