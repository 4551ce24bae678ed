"""Generate the committed golden fixtures of tests/golden/ (run from the repo root).

    python tests/golden/make_golden.py

The fixtures pin the CPU oracle against independent implementations:
  * int8_config1.json -- the workload's configs[0] (INT8 512x512x512, seed 0,
    fp32 output) and a ragged case: the INT32 accumulators from numpy's int64
    matmul, the fp32 epilogue from numpy float32 (one IEEE rounding per
    multiply), the bf16 output from torch's float32 -> bfloat16 cast, and the
    per-row checksums from numpy; each stored as a sha256 plus a few values.
  * generator.json -- sha256 of the first values of each generator stream,
    so a drift of the generator (CPU or GPU) is caught.
  * formats.json -- e4m3 / f16 / bf16 / e2m1 encodings of a fixed sample of
    fp32 values, from torch / numpy casts (the oracle's converters are checked
    against these).
  * dense.json -- the tensor-furnace GEMM (mma_virus) of each operand format
    (bf16, fp16, tf32, e4m3, fp32) on the dense generator's operands: C = A B^T from
    numpy's float64 matmul of the decoded operands, which is exact here (every
    operand is a multiple of 2^-15 of magnitude at most 1, so every product is a
    multiple of 2^-30 and a K <= 256 sum fits a double's 53 bits), rounded to
    fp32 by numpy and to the format's output type by torch's casts.
The operands themselves come from the oracle's generator (the GPU generator is
checked against it bit for bit in the GPU tests).
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import qg_oracle as O  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def cksum_weights(M: int, N: int) -> np.ndarray:
    m = np.arange(M, dtype=np.uint64)[:, None]
    n = np.arange(N, dtype=np.uint64)[None, :]
    w = (m * np.uint64(0x9E3779B1) + n * np.uint64(0x85EBCA77)) & np.uint64(0xFFFFFFFF)
    return (w | np.uint64(1)).astype(np.uint64)


def int8_case(M: int, N: int, K: int, seed: int) -> dict:
    A, B, sa, sb = O.int8_operands(M, N, K, seed)
    acc = (A.astype(np.int64) @ B.astype(np.int64).T)
    assert np.abs(acc).max() < 2**31
    acc32 = acc.astype(np.int32)
    f32 = (acc32.astype(np.float32) * sa[:, None]).astype(np.float32)
    f32 = (f32 * sb[None, :]).astype(np.float32)
    bf16 = torch.from_numpy(f32).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    w = cksum_weights(M, N)
    ck = ((acc32.astype(np.int64).astype(np.uint64) & np.uint64(0xFFFFFFFF)) * w) & np.uint64(0xFFFFFFFF)
    row_ck = (ck.sum(axis=1) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    return {
        "M": M, "N": N, "K": K, "seed": seed,
        "acc_sha256": sha(acc32), "f32_sha256": sha(f32), "bf16_sha256": sha(bf16),
        "row_cksum_sha256": sha(row_ck),
        "acc_head": acc32.ravel()[:8].tolist(), "f32_head": [float(x) for x in f32.ravel()[:8]],
        "row_cksum_head": row_ck[:8].tolist(),
    }


def generator_fixture() -> dict:
    out = {}
    for seed, tid in [(0, 0), (1, 1), (12345, 7)]:
        out[f"i8_{seed}_{tid}"] = sha(O.gen_i8(4096, seed, tid))
        out[f"u_{seed}_{tid}"] = sha(O.gen_uniform_f32(4096, 0.001, 0.01, seed, tid))
        out[f"n_{seed}_{tid}"] = sha(O.gen_normal_f32(4096, seed, tid))
    out["hash64_0_0_0"] = int(O.lib().qgo_hash64(0, 0, 0))
    return out


def sample_values() -> np.ndarray:
    rng = np.random.default_rng(2024)
    v = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * np.float32(50.0),
        rng.uniform(-448, 448, 4000).astype(np.float32),
        rng.uniform(-0.02, 0.02, 2000).astype(np.float32),
        rng.uniform(-7, 7, 2000).astype(np.float32),
        np.array([0.0, -0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 448.0, -448.0, 240.0, 0.001953125,
                  0.0009765625, 65504.0, 1e-8, 6.0, -6.0, 0.5, 1.5], dtype=np.float32),
    ])
    return v.astype(np.float32)


def formats_fixture() -> dict:
    v = sample_values()
    e4m3 = torch.from_numpy(v[np.abs(v) <= 448]).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    f16 = v.astype(np.float16).view(np.uint16)
    bf16 = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    res = {"values_sha256": sha(v), "e4m3_sha256": sha(e4m3), "f16_sha256": sha(f16), "bf16_sha256": sha(bf16)}
    res["e2m1_source"] = "enumeration of the e2m1 grid: nearest value, ties to the even code, satfinite at 6"
    # e2m1: nearest representable value, ties to the even code, from enumeration.
    grid = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)
    a = np.minimum(np.abs(v.astype(np.float64)), 6.0)
    d = np.abs(a[:, None] - grid[None, :])
    best = d.min(axis=1, keepdims=True)
    cand = (d == best)
    codes = np.array([np.flatnonzero(row)[0] if row.sum() == 1 else
                      [c for c in np.flatnonzero(row) if c % 2 == 0][0] for row in cand], dtype=np.uint8)
    codes = codes | (np.signbit(v).astype(np.uint8) << 3)
    res["e2m1_sha256"] = sha(codes)
    return res


DENSE = {  # format id: (name, storage dtype, decoder, output type name)
    4: ("bf16", np.uint16, lambda b: torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).float().numpy(), "bf16"),
    5: ("fp16", np.uint16, lambda b: b.view(np.float16).astype(np.float32), "f16"),
    6: ("tf32", np.uint32, lambda b: b.view(np.float32), "f32"),
    7: ("e4m3", np.uint8, lambda b: torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy(), "bf16"),
    8: ("fp32", np.uint32, lambda b: b.view(np.float32), "f32"),
}


def dense_case(fmt: int, M: int, N: int, K: int, seed: int) -> dict:
    name, _, decode, out = DENSE[fmt]
    A, B = O.dense_operands(fmt, M, N, K, seed)
    a, b = decode(A).astype(np.float64), decode(B).astype(np.float64)
    # the exactness premise: multiples of 2^-15, magnitude at most 1
    for x in (a, b):
        assert np.all(np.abs(x) <= 1) and np.all(np.mod(x * 32768.0, 1.0) == 0)
    f32 = (a @ b.T).astype(np.float32)
    t = torch.from_numpy(f32)
    outv = {"bf16": lambda: t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16),
            "f16": lambda: t.to(torch.float16).view(torch.int16).numpy().view(np.uint16),
            "f32": lambda: f32}[out]()
    return {"format": fmt, "name": name, "M": M, "N": N, "K": K, "seed": seed, "out_type": out,
            "A_sha256": sha(A), "B_sha256": sha(B), "f32_sha256": sha(f32), "out_sha256": sha(outv),
            "f32_head": [float(x) for x in f32.ravel()[:6]]}


def main() -> None:
    O.build()
    cases = [int8_case(512, 512, 512, 0), int8_case(130, 200, 48, 3)]
    (HERE / "int8_config1.json").write_text(json.dumps({"cases": cases}, indent=1) + "\n")
    (HERE / "generator.json").write_text(json.dumps(generator_fixture(), indent=1) + "\n")
    (HERE / "formats.json").write_text(json.dumps(formats_fixture(), indent=1) + "\n")
    dense = [dense_case(f, 48, 40, 256, 9) for f in sorted(DENSE)] + [dense_case(4, 33, 17, 128, 2)]
    (HERE / "dense.json").write_text(json.dumps({"cases": dense}, indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.glob("*.json")))


if __name__ == "__main__":
    main()
