"""Parity against an independent implementation on the same device: the vendor
library (cuBLAS through torch) as a second checker beside the CPU oracle.

* INT8: the raw INT32 accumulators of our tcgen05 kernel equal cuBLAS's
  integer GEMM (`torch._int_mm`) bit for bit.
* NVFP4: our GEMM's bf16 output equals cuBLAS's NVFP4 GEMM (`scaled_mm` with
  1x16 ue4m3 block scales in the swizzled 32x4x4 layout, which is the tcgen05
  scale-atom layout our kernel reads, plus the fp32 per-tensor scales) bit for
  bit.

The library is only the checker here; the product path never calls it.
"""
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(256, 256, 256), (1024, 2048, 512), (4096, 4096, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
def test_int8_accumulators_equal_cublas(cuda_device, shape):
    M, N, K = shape
    A = pb.gen_i8(M * K, seed=3, tensor_id=0)[:M * K].view(M, K)
    B = pb.gen_i8(N * K, seed=3, tensor_id=1)[:N * K].view(N, K)
    ours = pb.gemm_i8(A, B, None, None, out_type=pb.QG_OUT_S32)
    try:
        ref = torch._int_mm(A, B.t())
    except (RuntimeError, AttributeError) as e:
        pytest.skip(f"torch._int_mm unavailable here: {e}")
    torch.cuda.synchronize()
    assert torch.equal(ours, ref)


@pytest.mark.parametrize("shape", [(256, 256, 512), (1024, 512, 2048), (4096, 4096, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
def test_nvfp4_equals_cublas(cuda_device, shape):
    import torch.nn.functional as F
    if not all(hasattr(torch, n) for n in ("float4_e2m1fn_x2", "float8_e4m3fn")) or not hasattr(F, "scaled_mm"):
        pytest.skip("this torch has no NVFP4 scaled_mm")
    M, N, K = shape
    A, sfa, B, sfb, g = pb.gen_nvfp4(M, N, K, seed=4)
    ga, gb = [float(x) for x in g.cpu()]
    ours = pb.gemm_nvfp4(A, sfa, B, sfb, ga, gb)
    try:
        ref = F.scaled_mm(A.view(torch.float4_e2m1fn_x2), B.view(torch.float4_e2m1fn_x2).t(),
                          [sfa.view(torch.float8_e4m3fn), torch.tensor(ga, device=A.device)],
                          [F.ScalingType.BlockWise1x16, F.ScalingType.TensorWise],
                          [sfb.view(torch.float8_e4m3fn), torch.tensor(gb, device=A.device)],
                          [F.ScalingType.BlockWise1x16, F.ScalingType.TensorWise],
                          swizzle_a=[F.SwizzleType.SWIZZLE_32_4_4, F.SwizzleType.NO_SWIZZLE],
                          swizzle_b=[F.SwizzleType.SWIZZLE_32_4_4, F.SwizzleType.NO_SWIZZLE],
                          output_dtype=torch.bfloat16)
    except (RuntimeError, NotImplementedError, TypeError) as e:
        pytest.skip(f"NVFP4 scaled_mm unavailable here: {e}")
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16))
