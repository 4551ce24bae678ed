"""The tensor-furnace GEMM oracle (bf16 / e4m3 operands, fp32 accumulate), checked
against float64 numpy on the decoded operands (no GPU)."""
import numpy as np
import pytest
import torch


@pytest.mark.parametrize("kind", [1, 2])
def test_dense_oracle_matches_numpy(oracle, kind):
    M, N, K = 5, 7, 96
    rng = np.random.default_rng(kind)
    x = rng.standard_normal((M + N, K)).astype(np.float32)
    if kind == 1:
        bits = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        dec = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).float().numpy()
    else:
        bits = torch.from_numpy(x * 40).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        dec = torch.from_numpy(bits).view(torch.float8_e4m3fn).float().numpy()
    A, B = bits[:M], bits[M:]
    ref = (dec[:M].astype(np.float64) @ dec[M:].astype(np.float64).T).astype(np.float32) * np.float32(0.5)
    y = oracle.gemm_dense(kind, A, B, alpha=0.5, out_type=1)
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6 * np.abs(ref).max())
    rows = np.array([4, 0], dtype=np.int32)
    np.testing.assert_array_equal(oracle.gemm_dense(kind, A, B, alpha=0.5, out_type=1, rows=rows), y[rows])
