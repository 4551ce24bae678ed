"""Tensor-furnace GEMMs (bf16 / fp16 / tf32 / e4m3 operands on the tcgen05 path, fp32
operands on the CUDA-core path; fp32 accumulate) against the CPU oracle: f32 output within 1e-4 relative (accumulation
order), bf16 / fp16 output within 1e-2 (|y - ref| <= tol * max(|ref|, rms(ref))).
M >= 256 runs on CTA pairs.  Also the dense workload contexts: operands from the
generator bit-exact against the oracle's restatement, golden / verify / inject."""
import numpy as np
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu

SHAPES = [(128, 256, 256), (130, 200, 512), (256, 512, 1024), (1000, 1000, 1024), (384, 128, 2048), (64, 1, 64)]

# oracle kind, device entry, torch storage
KINDS = {
    "bf16": (1, pb.gemm_bf16),
    "e4m3": (2, pb.gemm_e4m3),
    "fp16": (3, pb.gemm_f16),
    "tf32": (4, pb.gemm_tf32),
    "fp32": (5, pb.gemm_f32),
}


def _tf32(x: torch.Tensor) -> torch.Tensor:
    """fp32 values rounded to tf32 (nearest even at 10 mantissa bits), as fp32 words."""
    u = x.contiguous().view(torch.int32).to(torch.int64)
    u = (u + 0xFFF + ((u >> 13) & 1)) & ~0x1FFF
    return u.to(torch.int32).view(torch.float32)


def _operands(name, M, N, K, seed):
    """(device A, device B, oracle A bits, oracle B bits)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((M + N, K), generator=g)
    if name == "bf16":
        t = x.to(torch.bfloat16)
        bits = t.view(torch.int16).numpy().view(np.uint16)
    elif name == "fp16":
        t = x.to(torch.float16)
        bits = t.view(torch.int16).numpy().view(np.uint16)
    elif name == "tf32":
        t = _tf32(x)
        bits = t.view(torch.int32).numpy().view(np.uint32)
    elif name == "fp32":
        t = x.contiguous()
        bits = t.view(torch.int32).numpy().view(np.uint32)
    else:
        t = (x * 40).to(torch.float8_e4m3fn).view(torch.uint8)
        bits = t.numpy()
    return t[:M].contiguous(), t[M:].contiguous(), bits[:M], bits[M:]


@pytest.mark.parametrize("name", list(KINDS))
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_dense_gemm_matches_oracle(cuda_device, oracle, name, shape):
    M, N, K = shape
    kind, f = KINDS[name]
    if name == "e4m3" and K % 16:
        pytest.skip("e4m3 rows must be a multiple of 16 bytes")
    tA, tB, A, B = _operands(name, M, N, K, seed=M + N + K + kind)
    dA, dB = tA.to(cuda_device), tB.to(cuda_device)
    y32 = f(dA, dB, alpha=0.75, out_type=pb.QG_OUT_F32)
    ybf = f(dA, dB, alpha=0.75, out_type=pb.QG_OUT_BF16)
    y16 = f(dA, dB, alpha=0.75, out_type=pb.QG_OUT_F16)
    torch.cuda.synchronize()
    assert pb.device_status(0) == 0
    ref32 = oracle.gemm_dense(kind, A, B, alpha=0.75, out_type=1)
    assert oracle.max_rel_err(y32.cpu().numpy(), ref32, 1) < 1e-4
    refbf = oracle.gemm_dense(kind, A, B, alpha=0.75, out_type=0)
    assert oracle.max_rel_err(ybf.view(torch.int16).cpu().numpy().view(np.uint16), refbf, 0) < 1e-2
    # fp16 output: compared as fp32 values (the oracle's fp16 bits decoded by torch)
    ref16 = torch.from_numpy(oracle.gemm_dense(kind, A, B, alpha=0.75, out_type=3).view(np.int16)).view(torch.float16)
    assert oracle.max_rel_err(y16.float().cpu().numpy(), ref16.float().numpy(), 1) < 1e-2


def test_dense_gemm_is_reproducible(cuda_device):
    """A deterministic kernel reproduces itself bit for bit (the furnace's verification rule)."""
    g = torch.Generator().manual_seed(3)
    A = torch.randn((2048, 2048), generator=g).to(torch.bfloat16).to(cuda_device)
    B = torch.randn((1024, 2048), generator=g).to(torch.bfloat16).to(cuda_device)
    a = pb.gemm_bf16(A, B)
    b = pb.gemm_bf16(A, B)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


FORMATS = {pb.QG_FMT_BF16: (1, pb.QG_OUT_BF16, np.uint16), pb.QG_FMT_FP16: (3, pb.QG_OUT_F16, np.uint16),
           pb.QG_FMT_TF32: (4, pb.QG_OUT_F32, np.uint32), pb.QG_FMT_E4M3: (2, pb.QG_OUT_BF16, np.uint8),
           pb.QG_FMT_FP32: (5, pb.QG_OUT_F32, np.uint32)}
_ORACLE_OUT = {pb.QG_OUT_BF16: 0, pb.QG_OUT_F32: 1, pb.QG_OUT_F16: 3}


@pytest.mark.parametrize("fmt", list(FORMATS), ids=["bf16", "fp16", "tf32", "e4m3", "fp32"])
def test_dense_workload_matches_oracle(cuda_device, oracle, fmt):
    """The workload's own operands (generator stream) bit-exact against the oracle's,
    its GEMM within tolerance on sampled rows, golden / verify / inject on the device."""
    kind, out_type, dt = FORMATS[fmt]
    M, N, K = 512, 768, 1024
    with pb.Workload(fmt, M, N, K, copies=2, seed=5, out_type=out_type) as w:
        w.fill(5)
        w.golden()
        w.run(6)
        w.synchronize()
        assert w.verify() == 0
        for copy in range(2):
            A0, B0 = oracle.dense_operands(fmt, M, N, K, seed=5, copy=copy)
            A = w.tensor(copy, 0).cpu().numpy().view(dt).reshape(M, K)
            B = w.tensor(copy, 1).cpu().numpy().view(dt).reshape(N, K)
            np.testing.assert_array_equal(A, A0)
            np.testing.assert_array_equal(B, B0)
        rows = np.array([0, 1, 255, 256, 511], dtype=np.int32)
        ref = oracle.gemm_dense(kind, A0, B0, out_type=_ORACLE_OUT[out_type], rows=rows)
        ob = w.tensor(1, 5).cpu().numpy()
        if out_type == pb.QG_OUT_F32:
            y = ob.view(np.float32).reshape(M, N)[rows]
            assert oracle.max_rel_err(y, ref, 1) < 1e-4
        elif out_type == pb.QG_OUT_F16:
            y = torch.from_numpy(ob.view(np.int16).reshape(M, N)[rows].copy()).view(torch.float16).float().numpy()
            r = torch.from_numpy(ref.view(np.int16)).view(torch.float16).float().numpy()
            assert oracle.max_rel_err(y, r, 1) < 1e-2
        else:
            y = ob.view(np.uint16).reshape(M, N)[rows]
            assert oracle.max_rel_err(y, ref, 0) < 1e-2
        w.inject()
        assert w.verify() >= 1


def test_dense_workload_odd_output_is_fully_verified(cuda_device):
    """M*N odd with a 2-byte output: the last element is inside a verified word."""
    with pb.Workload(pb.QG_FMT_BF16, 33, 17, 64, seed=2, out_type=pb.QG_OUT_BF16) as w:
        w.fill(2)
        w.golden()
        w.run(3)
        w.synchronize()
        assert w.verify() == 0
