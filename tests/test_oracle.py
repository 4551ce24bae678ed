"""The CPU oracle, pinned against independent implementations and the committed fixtures.

No GPU needed.  The oracle is test infrastructure (oracle/qg_oracle.h); these
tests are what makes it trustworthy as the checker of the CUDA kernels:
  * its INT8 GEMM against numpy's exact integer matmul;
  * its fp32 epilogue against numpy float32, its bf16 rounding against torch;
  * its e4m3 / f16 / bf16 / e2m1 converters against torch / numpy / enumeration;
  * its generator and configs[0] known answer against tests/golden/*.json.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_splitmix64_known_answer(oracle):
    # splitmix64's published first output for state 0 after one gamma step.
    assert oracle.lib().qgo_splitmix64(0x9E3779B97F4A7C15) == 0xE220A8397B1DCDAF


def test_generator_matches_fixture(oracle):
    fx = json.loads((GOLDEN / "generator.json").read_text())
    for seed, tid in [(0, 0), (1, 1), (12345, 7)]:
        assert sha(oracle.gen_i8(4096, seed, tid)) == fx[f"i8_{seed}_{tid}"]
        assert sha(oracle.gen_uniform_f32(4096, 0.001, 0.01, seed, tid)) == fx[f"u_{seed}_{tid}"]
        assert sha(oracle.gen_normal_f32(4096, seed, tid)) == fx[f"n_{seed}_{tid}"]
    assert oracle.lib().qgo_hash64(0, 0, 0) == fx["hash64_0_0_0"]


def test_generator_distributions(oracle):
    a = oracle.gen_i8(1 << 20, 5, 0).astype(np.int32)
    assert a.min() == -127 and a.max() == 127
    assert abs(a.mean()) < 0.5
    u = oracle.gen_uniform_f32(1 << 20, 0.001, 0.01, 5, 1)
    assert u.min() >= 0.001 and u.max() < 0.01
    n = oracle.gen_normal_f32(1 << 20, 5, 2).astype(np.float64)
    assert abs(n.mean()) < 0.01 and abs(n.std() - 1.0) < 0.01
    # tails follow the normal law: P(|x| > 3) ~ 0.0027
    assert 0.002 < np.mean(np.abs(n) > 3) < 0.0035
    # A and B streams differ
    assert not np.array_equal(oracle.gen_i8(4096, 5, 0), oracle.gen_i8(4096, 5, 1))


def test_logf_accuracy(oracle):
    xs = np.concatenate([np.geomspace(1e-7, 1.0, 2000), np.linspace(0.5, 2.0, 500)]).astype(np.float32)
    f = oracle.lib().qgo_logf
    got = np.array([f(float(x)) for x in xs], dtype=np.float64)
    ref = np.log(xs.astype(np.float64))
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-3)) < 2e-6


@pytest.mark.parametrize("shape", [(1, 1, 16), (7, 9, 32), (64, 96, 128), (130, 200, 48), (33, 257, 528)])
def test_gemm_i8_matches_numpy(oracle, shape):
    M, N, K = shape
    rng = np.random.default_rng(M * 1000 + N)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sa = rng.uniform(0.001, 0.01, M).astype(np.float32)
    sb = rng.uniform(0.001, 0.01, N).astype(np.float32)
    acc_ref = (A.astype(np.int64) @ B.astype(np.int64).T).astype(np.int32)
    s32 = oracle.gemm_i8(A, B, sa, sb, out_type=2)
    np.testing.assert_array_equal(s32, acc_ref)
    f32 = oracle.gemm_i8(A, B, sa, sb, out_type=1)
    f32_ref = ((acc_ref.astype(np.float32) * sa[:, None]).astype(np.float32) * sb[None, :]).astype(np.float32)
    np.testing.assert_array_equal(f32.view(np.uint32), f32_ref.view(np.uint32))
    bf = oracle.gemm_i8(A, B, sa, sb, out_type=0)
    bf_ref = torch.from_numpy(f32_ref).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(bf, bf_ref)


def test_gemm_i8_row_subset_and_checksums(oracle):
    M, N, K = 40, 50, 64
    A, B, sa, sb = oracle.int8_operands(M, N, K, seed=9)
    full, acc, ck = oracle.gemm_i8(A, B, sa, sb, out_type=0, want_acc=True, want_cksum=True)
    rows = np.array([0, 7, 39, 13], dtype=np.int32)
    sub, ck_sub = oracle.gemm_i8(A, B, sa, sb, out_type=0, rows=rows, want_cksum=True)
    np.testing.assert_array_equal(sub, full[rows])
    np.testing.assert_array_equal(ck_sub, ck[rows])
    w = ((np.arange(M, dtype=np.uint64)[:, None] * np.uint64(0x9E3779B1) +
          np.arange(N, dtype=np.uint64)[None, :] * np.uint64(0x85EBCA77)) & np.uint64(0xFFFFFFFF)) | np.uint64(1)
    ref = (((acc.astype(np.int64).astype(np.uint64) & np.uint64(0xFFFFFFFF)) * w) & np.uint64(0xFFFFFFFF)).sum(axis=1)
    np.testing.assert_array_equal(ck, (ref & np.uint64(0xFFFFFFFF)).astype(np.uint32))


def test_config1_known_answer(oracle):
    """INT8 512^3, seed 0, fp32 output -- golden fixture from numpy."""
    fx = json.loads((GOLDEN / "int8_config1.json").read_text())
    for case in fx["cases"]:
        M, N, K, seed = case["M"], case["N"], case["K"], case["seed"]
        A, B, sa, sb = oracle.int8_operands(M, N, K, seed)
        f32, acc, ck = oracle.gemm_i8(A, B, sa, sb, out_type=1, want_acc=True, want_cksum=True)
        bf = oracle.gemm_i8(A, B, sa, sb, out_type=0)
        assert sha(acc) == case["acc_sha256"]
        assert sha(f32) == case["f32_sha256"]
        assert sha(bf) == case["bf16_sha256"]
        assert sha(ck) == case["row_cksum_sha256"]


def _sample_values():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.sample_values()


def test_converters_match_fixture_and_libraries(oracle):
    fx = json.loads((GOLDEN / "formats.json").read_text())
    v = _sample_values()
    assert sha(v) == fx["values_sha256"]
    L = oracle.lib()
    inr = v[np.abs(v) <= 448]
    e4 = np.array([L.qgo_f32_to_e4m3(float(x)) for x in inr], dtype=np.uint8)
    assert sha(e4) == fx["e4m3_sha256"]
    np.testing.assert_array_equal(e4, torch.from_numpy(inr).to(torch.float8_e4m3fn).view(torch.uint8).numpy())
    f16 = np.array([L.qgo_f32_to_f16(float(x)) for x in v], dtype=np.uint16)
    assert sha(f16) == fx["f16_sha256"]
    bf = np.array([L.qgo_f32_to_bf16(float(x)) for x in v], dtype=np.uint16)
    assert sha(bf) == fx["bf16_sha256"]
    e2 = np.array([L.qgo_f32_to_e2m1(float(x)) for x in v], dtype=np.uint8)
    assert sha(e2) == fx["e2m1_sha256"]


def test_e4m3_decode_table_matches_torch(oracle):
    codes = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).to(torch.float32).numpy()
    got = np.array([oracle.lib().qgo_e4m3_to_f32(int(c)) for c in codes], dtype=np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan], ref[~nan])


def test_e4m3_saturates(oracle):
    L = oracle.lib()
    assert L.qgo_f32_to_e4m3(1000.0) == 0x7E
    assert L.qgo_f32_to_e4m3(-470.0) == 0xFE
    assert L.qgo_f32_to_e4m3(455.0) == 0x7E


def test_f16_roundtrip_all_codes(oracle):
    L = oracle.lib()
    codes = np.arange(0, 65536, 7, dtype=np.uint16)
    vals = codes.view(np.float16).astype(np.float32)
    ok = np.isfinite(vals)
    got = np.array([L.qgo_f32_to_f16(float(x)) for x in vals[ok]], dtype=np.uint16)
    np.testing.assert_array_equal(got, codes[ok])


def test_count_mismatch_and_rel_err(oracle):
    a = np.arange(1000, dtype=np.uint32)
    b = a.copy()
    b[[3, 500, 999]] ^= 1
    assert oracle.lib().qgo_count_mismatch_u32(oracle._p(a), oracle._p(b), a.size) == 3
    r = np.linspace(-1, 1, 101).astype(np.float32)
    y = r * np.float32(1.001)
    assert oracle.max_rel_err(y, r, 1) < 2e-3


@pytest.mark.parametrize("shape", [(1, 8, 128), (3, 36, 256), (16, 64, 512)])
def test_gemv_w4a16_oracle_matches_numpy(oracle, shape):
    """The oracle's W4A16 GEMV against an independent float64 numpy evaluation."""
    M, N, K = shape
    X, W, S, Z = oracle.w4a16_operands(M, N, K, seed=M + N)
    ref = oracle.gemv_w4a16_numpy(X, W, S, Z).astype(np.float32)
    y = oracle.gemv_w4a16(X, W, S, Z, out_type=1)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5 * float(np.abs(ref).max()))
    cols = np.array([0, N - 1, N // 2], dtype=np.int32)
    np.testing.assert_array_equal(oracle.gemv_w4a16(X, W, S, Z, out_type=1, cols=cols), y[:, cols])


def test_w4a16_generator_distributions(oracle):
    X, W, S, Z = oracle.w4a16_operands(4, 1024, 1024, seed=3)
    x = oracle.bf16_bits_to_f32(X)
    assert abs(float(x.mean())) < 0.05 and abs(float(x.std()) - 1.0) < 0.05
    u = ((W[:, None, :] >> (4 * np.arange(8, dtype=np.uint32))[None, :, None]) & 0xF).ravel()
    assert u.min() == 0 and u.max() == 15 and abs(u.mean() - 7.5) < 0.05
    s = S.view(np.float16).astype(np.float32)
    z = Z.view(np.float16).astype(np.float32)
    # bounds after rounding to fp16
    assert s.min() >= np.float16(0.005) and s.max() <= np.float16(0.02) and z.min() >= -0.5 and z.max() <= 0.5
