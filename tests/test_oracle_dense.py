"""The tensor-furnace GEMM oracle (bf16 / fp16 / tf32 / e4m3 / fp32 operands, fp32
accumulate) and the dense operand generator, checked against float64 numpy and
torch's own format casts on the decoded operands (no GPU)."""
import numpy as np
import pytest
import torch


def _tf32_numpy(x):
    """Round fp32 values to tf32 (11 significant bits, nearest even) with numpy's own
    half-even rounding; an independent statement of qgo_f32_to_tf32_bits."""
    m, e = np.frexp(x.astype(np.float64))
    return np.ldexp(np.round(m * 2048.0) / 2048.0, e).astype(np.float32)


def _encode(kind, x):
    """(bit patterns, decoded fp32 values) of `x` in operand kind `kind`."""
    t = torch.from_numpy(x)
    if kind == 1:
        b = t.to(torch.bfloat16)
        return b.view(torch.int16).numpy().view(np.uint16), b.float().numpy()
    if kind == 3:
        h = t.to(torch.float16)
        return h.view(torch.int16).numpy().view(np.uint16), h.float().numpy()
    if kind == 4:
        v = _tf32_numpy(x)
        return v.view(np.uint32), v
    if kind == 5:
        return x.view(np.uint32), x
    q = (t * 40).to(torch.float8_e4m3fn)
    return q.view(torch.uint8).numpy(), q.float().numpy()


@pytest.mark.parametrize("kind", [1, 2, 3, 4, 5])
def test_dense_oracle_matches_numpy(oracle, kind):
    M, N, K = 5, 7, 96
    rng = np.random.default_rng(kind)
    x = rng.standard_normal((M + N, K)).astype(np.float32)
    bits, dec = _encode(kind, x)
    A, B = bits[:M], bits[M:]
    ref = (dec[:M].astype(np.float64) @ dec[M:].astype(np.float64).T).astype(np.float32) * np.float32(0.5)
    y = oracle.gemm_dense(kind, A, B, alpha=0.5, out_type=1)
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6 * np.abs(ref).max())
    rows = np.array([4, 0], dtype=np.int32)
    np.testing.assert_array_equal(oracle.gemm_dense(kind, A, B, alpha=0.5, out_type=1, rows=rows), y[rows])
    # bf16 and fp16 outputs are the fp32 result rounded once
    y16 = oracle.gemm_dense(kind, A, B, alpha=0.5, out_type=3)
    np.testing.assert_array_equal(y16, torch.from_numpy(y).to(torch.float16).view(torch.int16).numpy().view(np.uint16))
    yb = oracle.gemm_dense(kind, A, B, alpha=0.5, out_type=0)
    np.testing.assert_array_equal(yb, torch.from_numpy(y).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


def test_tf32_rounding_matches_numpy(oracle):
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(4000).astype(np.float32),
                        # ties at the 11th significant bit, both parities
                        np.array([1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, -(1.0 + 2.0 ** -11), 0.0, -0.0],
                                 dtype=np.float32)])
    got = np.array([oracle.lib().qgo_f32_to_tf32_bits(float(v)) for v in x], dtype=np.uint32)
    np.testing.assert_array_equal(got, _tf32_numpy(x).view(np.uint32))
    assert np.all(got & 0x1FFF == 0)


@pytest.mark.parametrize("fmt", [4, 5, 6, 7, 8])
def test_dense_generator_values(oracle, fmt):
    """Every generated operand is fmt(j / 32768 - 1) for the element's own hash."""
    n, seed, tid = 3000, 11, 9
    out = oracle.gen_dense(fmt, n, seed, tid)
    h = np.array([oracle.lib().qgo_hash64(seed, tid, i) for i in range(n)], dtype=np.uint64)
    v = ((h >> np.uint64(48)).astype(np.float64) / 32768.0 - 1.0).astype(np.float32)
    assert np.all(v >= -1.0) and np.all(v < 1.0)
    if fmt == 6:
        np.testing.assert_array_equal(out, _tf32_numpy(v).view(np.uint32))
    elif fmt == 8:
        np.testing.assert_array_equal(out, v.view(np.uint32))
    else:
        kind = {4: 1, 5: 3, 7: 2}[fmt]
        if kind == 2:
            want = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        else:
            want, _ = _encode(kind, v)
        np.testing.assert_array_equal(out, want)
    # distinct tensor ids are distinct streams
    assert not np.array_equal(out, oracle.gen_dense(fmt, n, seed, tid + 1))


def test_dense_oracle_matches_golden_known_answers(oracle):
    """tests/golden/dense.json: each operand format's GEMM on the dense generator's operands,
    from numpy's float64 matmul (exact for these operands) rounded by numpy / torch casts."""
    import hashlib
    import json
    from pathlib import Path
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    cases = json.loads((Path(__file__).parent / "golden" / "dense.json").read_text())["cases"]
    assert {c["name"] for c in cases} == {"bf16", "fp16", "tf32", "e4m3", "fp32"}
    for c in cases:
        kind = oracle.DENSE_FORMATS[c["format"]][0]
        A, B = oracle.dense_operands(c["format"], c["M"], c["N"], c["K"], c["seed"])
        assert sha(A) == c["A_sha256"] and sha(B) == c["B_sha256"], c["name"]
        f32 = oracle.gemm_dense(kind, A, B, alpha=1.0, out_type=1)
        assert sha(f32) == c["f32_sha256"], c["name"]
        out_type = {"bf16": 0, "f16": 3, "f32": 1}[c["out_type"]]
        assert sha(oracle.gemm_dense(kind, A, B, alpha=1.0, out_type=out_type)) == c["out_sha256"], c["name"]
