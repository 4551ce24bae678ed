"""The FP8 block-128 oracle, pinned against numpy / torch (no GPU).

* quantisation: every block's absmax maps to 448 (within e4m3 rounding), the
  stored scale is absmax/448, and q = e4m3(x * 448/absmax) matches torch's
  float8_e4m3fn cast of the same fp32 products;
* GEMM: the oracle's per-K-block promotion against a float64 numpy evaluation
  of sum_kb (A_kb B_kb^T) sa sb.
"""
import numpy as np
import pytest
import torch


def test_fp8_quantisation_rows_and_blocks(oracle):
    M, N, K = 3, 130, 256
    A, B, sa, sb = oracle.fp8_operands(M, N, K, seed=4)
    xa = oracle.gen_normal_f32(M * K, 4, 0).reshape(M, K)
    xb = oracle.gen_normal_f32(N * K, 4, 2).reshape(N, K)
    for r in range(M):
        for kb in range(K // 128):
            blk = xa[r, kb * 128:(kb + 1) * 128]
            amax = np.float32(np.abs(blk).max())
            assert sa[r, kb] == np.float32(amax / np.float32(448.0))
            inv = np.float32(np.float32(448.0) / amax)
            ref = torch.from_numpy((blk * inv).astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
            np.testing.assert_array_equal(A[r, kb * 128:(kb + 1) * 128], ref)
            assert np.abs(oracle.e4m3_to_f32(A[r, kb * 128:(kb + 1) * 128])).max() == 448.0
    for rb in range((N + 127) // 128):
        for kb in range(K // 128):
            blk = xb[rb * 128:(rb + 1) * 128, kb * 128:(kb + 1) * 128]
            amax = np.float32(np.abs(blk).max())
            assert sb[rb, kb] == np.float32(amax / np.float32(448.0))


@pytest.mark.parametrize("shape", [(4, 8, 128), (33, 130, 384), (128, 256, 256)])
def test_fp8_gemm_oracle_matches_numpy(oracle, shape):
    M, N, K = shape
    A, B, sa, sb = oracle.fp8_operands(M, N, K, seed=M + N)
    a = oracle.e4m3_to_f32(A).astype(np.float64)
    b = oracle.e4m3_to_f32(B).astype(np.float64)
    ref = np.zeros((M, N))
    for kb in range(K // 128):
        p = a[:, kb * 128:(kb + 1) * 128] @ b[:, kb * 128:(kb + 1) * 128].T
        ref += p * sa[:, kb][:, None].astype(np.float64) * np.repeat(sb[:, kb], 128)[:N][None, :].astype(np.float64)
    y = oracle.gemm_fp8(A, B, sa, sb, out_type=1)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    # the dequantised operands reproduce the normal draws to within e4m3 resolution
    xa = oracle.gen_normal_f32(M * K, M + N, 0).reshape(M, K)
    deq = a * np.repeat(sa, 128, axis=1)
    assert np.max(np.abs(deq - xa)) <= np.abs(xa).max() * 2.0 ** -4
