"""The NVFP4 oracle, pinned against an independent numpy evaluation (no GPU).

* quantisation: per-tensor scale G = absmax/(448*6); every 16-element block's
  ue4m3 scale is e4m3(blockmax/6/G) (checked against torch's float8_e4m3fn
  cast); decoded codes times scales reproduce the normal draws to within the
  e2m1 grid's resolution;
* GEMM: the oracle against float64 numpy on the dequantised operands;
* the tcgen05 scale-factor atom layout helper places each scale where the
  layout formula says.
"""
import numpy as np
import pytest
import torch


def test_nvfp4_quantisation(oracle):
    M, N, K = 5, 7, 256
    A, SFA, GA, B, SFB, GB = oracle.nvfp4_operands(M, N, K, seed=11)
    x = oracle.gen_normal_f32(M * K, 11, 0).reshape(M, K)
    assert GA == np.float32(np.float32(np.abs(x).max()) / np.float32(2688.0))
    bmax = np.abs(x.reshape(M, K // 16, 16)).max(axis=2).astype(np.float32)
    t = (bmax / np.float32(6.0)).astype(np.float32) / GA
    ref_sf = torch.from_numpy(t.astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy() & 0x7F
    np.testing.assert_array_equal(SFA, ref_sf)
    deq = oracle.nvfp4_dequant(A, SFA, GA)
    # e2m1 keeps one mantissa bit: |x - q*s| <= half a grid step of the block (1/4 of its scale * 2)
    step = np.repeat(oracle.e4m3_to_f32(SFA).astype(np.float64) * float(GA), 16, axis=1)
    assert np.all(np.abs(deq - x) <= step * 1.0 + 1e-12)


@pytest.mark.parametrize("shape", [(4, 8, 256), (33, 130, 512), (128, 256, 256)])
def test_nvfp4_gemm_oracle_matches_numpy(oracle, shape):
    M, N, K = shape
    A, SFA, GA, B, SFB, GB = oracle.nvfp4_operands(M, N, K, seed=M + N)
    ref = oracle.nvfp4_dequant(A, SFA, GA) @ oracle.nvfp4_dequant(B, SFB, GB).T
    y = oracle.gemm_nvfp4(A, SFA, GA, B, SFB, GB, out_type=1)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())


def test_scale_atom_layout(oracle):
    R, K = 300, 512
    sf = np.random.default_rng(0).integers(0, 127, (R, K // 16), dtype=np.uint8)
    atoms = oracle.sf_to_atoms(sf).reshape((R + 127) // 128, K // 64, 512)
    for r in (0, 31, 32, 95, 127, 128, 200, 299):
        for j in (0, 3, 4, 17, 31):
            assert atoms[r // 128, j // 4, (r % 32) * 16 + ((r // 32) % 4) * 4 + j % 4] == sf[r, j]
