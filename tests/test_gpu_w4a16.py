"""W4A16 group-128 GEMV (1 row on the CUDA cores, 2-12 on warp MMAs, 13-16 on
tcgen05): parity with the CPU oracle, through the C ABI.

X bf16 [M in {1,8,16}, 8192] ~ N(0,1); W int4 [8192, 28672] uniform in
[-8,7]; fp16 scale and zero per 128 along K; bf16 output; tolerance 1e-2 relative
(|y - ref| <= 1e-2 * max(|ref|, rms(ref))), with fp32 accumulation.
Also: the device generator reproduces the oracle's operands bit for bit, the
split-K reduction makes the kernel reproduce itself bit for bit, and the
workspace's tickets are left ready for the next call.
"""
import numpy as np
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu
RTOL = 1e-2


def _np(t):
    return t.detach().cpu().numpy()


def _operands(oracle, M, N, K, seed, dev):
    X, W, S, Z = oracle.w4a16_operands(M, N, K, seed)
    return (X, W, S, Z), (torch.from_numpy(X.view(np.int16)).view(torch.bfloat16).to(dev),
                          torch.from_numpy(W.view(np.int32)).to(dev),
                          torch.from_numpy(S.view(np.int16)).view(torch.float16).to(dev),
                          torch.from_numpy(Z.view(np.int16)).view(torch.float16).to(dev))


def test_generator_matches_oracle(cuda_device, oracle):
    M, N, K = 3, 1028, 1024
    X, W, S, Z = pb.gen_w4a16(M, N, K, seed=5, tid0=8)
    rX, rW, rS, rZ = oracle.w4a16_operands(M, N, K, seed=5, copy=1)
    np.testing.assert_array_equal(_np(X.view(torch.int16)).view(np.uint16), rX)
    np.testing.assert_array_equal(_np(W).view(np.uint32), rW)
    np.testing.assert_array_equal(_np(S.view(torch.int16)).view(np.uint16), rS)
    np.testing.assert_array_equal(_np(Z.view(torch.int16)).view(np.uint16), rZ)


# 1 row runs on the CUDA cores, 2-12 on warp MMAs, 13-16 on tcgen05, more in chunks of 16
SHAPES = [(1, 512, 128), (1, 1028, 1024), (3, 2048, 2048), (8, 4096, 1024), (16, 1536, 4096),
          (17, 516, 256), (5, 28672, 256), (4, 300, 384), (12, 1028, 1024), (8, 128, 8192), (16, 36, 128),
          (34, 260, 512), (9, 2052, 1024), (13, 1028, 1024), (11, 36, 128),
          # the smallest widths: one or two live column quads of a super-tile
          (2, 4, 128), (9, 8, 128), (12, 4, 256), (13, 4, 128), (16, 4, 128)]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gemv_matches_oracle(cuda_device, oracle, shape):
    M, N, K = shape
    host, dev = _operands(oracle, M, N, K, seed=M * 7 + N, dev=cuda_device)
    y32 = pb.gemv_w4a16(*dev, out_type=pb.QG_OUT_F32)
    ybf = pb.gemv_w4a16(*dev, out_type=pb.QG_OUT_BF16)
    torch.cuda.synchronize()
    ref32 = oracle.gemv_w4a16(*host, out_type=1)
    assert oracle.max_rel_err(_np(y32), ref32, 1) < 1e-4
    refbf = oracle.gemv_w4a16(*host, out_type=0)
    assert oracle.max_rel_err(_np(ybf.view(torch.int16)).view(np.uint16), refbf, 0) < RTOL


# configs[3] at M = 1, 8, 16, each row-count boundary of the three kernels, and
# shapes whose warp-MMA grid runs in two waves (more groups per CTA than its
# shared memory can hold at once in one wave): 8 x 57344 x 8192, 4 x 65536 x 8192,
# 12 x 57344 x 8192.
FULL = [(1, 28672, 8192), (2, 28672, 8192), (3, 28672, 8192), (4, 28672, 8192), (5, 28672, 8192),
        (8, 28672, 8192), (9, 28672, 8192), (12, 28672, 8192), (13, 28672, 8192), (16, 28672, 8192),
        (8, 57344, 8192), (4, 65536, 8192), (12, 57344, 8192)]


@pytest.mark.parametrize("shape", FULL, ids=lambda s: "x".join(map(str, s)))
def test_full_size_config3(cuda_device, oracle, shape):
    """Full-size shapes; 256 sampled columns against the oracle, plus bitwise self-reproduction."""
    M, N, K = shape
    with pb.Workload(pb.QG_FMT_W4A16, M, N, K, seed=3) as w:
        w.fill(3)
        w.golden()
        X = _np(w.tensor(0, 0, torch.int16)).view(np.uint16).reshape(M, K)
        W = _np(w.tensor(0, 1, torch.int32)).view(np.uint32).reshape(K // 8, N)
        S = _np(w.tensor(0, 2, torch.int16)).view(np.uint16).reshape(K // 128, N)
        Z = _np(w.tensor(0, 3, torch.int16)).view(np.uint16).reshape(K // 128, N)
        Y = _np(w.tensor(0, w.SLOT_OUT, torch.int16)).view(np.uint16).reshape(M, N)
        cols = np.unique(np.concatenate([[0, 1, 511, 512, N - 1], np.random.default_rng(M).integers(0, N, 251)]))
        ref = oracle.gemv_w4a16(X, W, S, Z, out_type=0, cols=cols.astype(np.int32))
        assert oracle.max_rel_err(Y[:, cols].copy(), ref, 0) < RTOL
        w.run(5)
        assert w.verify() == 0
        assert pb.device_status(0) == 0


@pytest.mark.parametrize("M", [1, 2, 8, 12, 16])
@pytest.mark.parametrize("flags", ["weights", "activations", "both"])
def test_const_flags_are_bit_identical(cuda_device, oracle, M, flags):
    """QG_GEMV_WEIGHTS_CONST / QG_GEMV_ACTIVATIONS_CONST only move the first weight loads
    and the activations' quantisation before the dependency wait: back-to-back calls over
    fixed operands give the same bits as the default path."""
    N, K = 4096, 2048
    host, dev = _operands(oracle, M, N, K, seed=11, dev=cuda_device)
    ref = pb.gemv_w4a16(*dev, out_type=pb.QG_OUT_F32)
    kw = {"weights_const": flags in ("weights", "both"), "activations_const": flags in ("activations", "both")}
    outs = [pb.gemv_w4a16(*dev, out_type=pb.QG_OUT_F32, **kw) for _ in range(6)]
    torch.cuda.synchronize()
    for y in outs:
        assert torch.equal(y.view(torch.int32), ref.view(torch.int32))
    assert oracle.max_rel_err(_np(ref), oracle.gemv_w4a16(*host, out_type=1), 1) < 1e-4


@pytest.mark.parametrize("M", [2, 8, 12])
def test_workspace_reusable_and_checked(cuda_device, oracle, M):
    N, K = 2048, 2048
    host, dev = _operands(oracle, M, N, K, seed=1, dev=cuda_device)
    need = pb.gemv_w4a16_workspace_bytes(M, N, K)
    ws = torch.zeros((need,), dtype=torch.uint8, device=cuda_device)
    a = pb.gemv_w4a16(*dev, out_type=pb.QG_OUT_F32, workspace=ws)
    b = pb.gemv_w4a16(*dev, out_type=pb.QG_OUT_F32, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    with pytest.raises(pb.QGError):
        pb.gemv_w4a16(*dev, workspace=ws[: need - 4])
