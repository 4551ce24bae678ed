"""INT8 W8A8 tcgen05 GEMM: parity with the CPU oracle, through the C ABI.

Bit-exact is the bar for INT8 (configs[1]: "bit-exact INT32 check"):
  * the raw INT32 accumulators (QG_OUT_S32) equal numpy's integer matmul;
  * the fp32 and bf16 epilogues equal the oracle's bit for bit;
  * the per-row INT32 checksums equal the oracle's;
at small and ragged shapes in full, at configs[0] against the committed golden
fixture, and at the full configs[1] size (8192^3) on sampled rows plus the
size-independent properties (run-to-run bit identity, checksum agreement,
inject -> detected).
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _cpu(t):
    return t.detach().cpu().numpy()


def _bits(t):
    if t.dtype == torch.bfloat16:
        return _cpu(t.view(torch.int16)).view(np.uint16)
    if t.dtype == torch.float32:
        return _cpu(t).view(np.uint32)
    return _cpu(t)


def test_generator_matches_oracle_bitwise(cuda_device, oracle):
    n = (1 << 20) + 5
    for seed, tid in [(0, 0), (1, 1), (77, 9)]:
        np.testing.assert_array_equal(_cpu(pb.gen_i8(n, seed, tid)), oracle.gen_i8(n, seed, tid))
        np.testing.assert_array_equal(_cpu(pb.gen_uniform_f32(n, 0.001, 0.01, seed, tid)).view(np.uint32),
                                      oracle.gen_uniform_f32(n, 0.001, 0.01, seed, tid).view(np.uint32))
        np.testing.assert_array_equal(_cpu(pb.gen_normal_f32(n, seed, tid)).view(np.uint32),
                                      oracle.gen_normal_f32(n, seed, tid).view(np.uint32))


SHAPES = [
    (128, 256, 128),      # one tile, one K block
    (256, 512, 512),      # several tiles, several K blocks
    (512, 512, 512),      # configs[0] shape
    (130, 200, 48),       # ragged M, N and a K tail inside one block
    (1, 17, 16),          # smallest legal K, single row
    (1000, 1000, 1008),   # ragged everything, K not a multiple of 128
    (384, 768, 4096),     # deeper K
    (300, 8, 2064),       # N < 16
    (4096, 4096, 512),    # M >= 256: CTA pairs, several 256x256 tiles per pair
    (2560, 384, 256),     # pairs with a ragged N tile
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gemm_i8_matches_oracle(cuda_device, oracle, shape):
    M, N, K = shape
    A, B, sa, sb = oracle.int8_operands(M, N, K, seed=M + N + K)
    dA, dB = torch.from_numpy(A).to(cuda_device), torch.from_numpy(B).to(cuda_device)
    dsa, dsb = torch.from_numpy(sa).to(cuda_device), torch.from_numpy(sb).to(cuda_device)
    s32, ck = pb.gemm_i8(dA, dB, None, None, out_type=pb.QG_OUT_S32, row_checksums=True)
    f32 = pb.gemm_i8(dA, dB, dsa, dsb, out_type=pb.QG_OUT_F32)
    bf = pb.gemm_i8(dA, dB, dsa, dsb, out_type=pb.QG_OUT_BF16)
    torch.cuda.synchronize()
    assert pb.device_status(0) == 0
    acc_ref = (A.astype(np.int64) @ B.astype(np.int64).T).astype(np.int32)
    np.testing.assert_array_equal(_cpu(s32), acc_ref)
    _, ck_ref = oracle.gemm_i8(A, B, sa, sb, out_type=2, want_cksum=True)
    np.testing.assert_array_equal(_cpu(ck).view(np.uint32), ck_ref)
    np.testing.assert_array_equal(_bits(f32), oracle.gemm_i8(A, B, sa, sb, out_type=1).view(np.uint32))
    np.testing.assert_array_equal(_bits(bf), oracle.gemm_i8(A, B, sa, sb, out_type=0))


def test_config1_known_answer_through_workload(cuda_device):
    """configs[0] (512^3, seed 0, fp32 output) through the context API vs the golden fixture."""
    case = json.loads((GOLDEN / "int8_config1.json").read_text())["cases"][0]
    with pb.Workload(pb.QG_FMT_INT8, 512, 512, 512, seed=0, out_type=pb.QG_OUT_F32) as w:
        w.fill(0)
        w.golden()
        out = _cpu(w.tensor(0, w.SLOT_OUT, torch.float32)).reshape(512, 512)
        ck = _cpu(w.tensor(0, w.SLOT_CKSUM, torch.int32)).view(np.uint32)
        assert sha(out) == case["f32_sha256"]
        assert sha(ck) == case["row_cksum_sha256"]
        w.run(3)
        assert w.verify() == 0


def test_full_size_config2_sampled_rows_bit_exact(cuda_device, oracle):
    """8192^3, seed 1, bf16 output; 48 sampled rows bit-exact + row checksums."""
    M = N = K = 8192
    with pb.Workload(pb.QG_FMT_INT8, M, N, K, seed=1) as w:
        w.fill(1)
        w.golden()
        A = _cpu(w.tensor(0, 0, torch.int8)).reshape(M, K)
        B = _cpu(w.tensor(0, 1, torch.int8)).reshape(N, K)
        sa = _cpu(w.tensor(0, 2, torch.float32))
        sb = _cpu(w.tensor(0, 3, torch.float32))
        # the device generator produced exactly the oracle's operands
        rng = np.random.default_rng(0)
        idx = rng.integers(0, M * K, 4096)
        ref_A = oracle.gen_i8(M * K, 1, 0)
        np.testing.assert_array_equal(A.ravel()[idx], ref_A[idx])
        out = _cpu(w.tensor(0, w.SLOT_OUT, torch.int16)).view(np.uint16).reshape(M, N)
        ck = _cpu(w.tensor(0, w.SLOT_CKSUM, torch.int32)).view(np.uint32)
        rows = np.unique(np.concatenate([[0, 1, 127, 128, 4095, 8191], rng.integers(0, M, 42)])).astype(np.int32)
        ref, ref_ck = oracle.gemm_i8(A, B, sa, sb, out_type=0, rows=rows, want_cksum=True)
        np.testing.assert_array_equal(out[rows], ref)
        np.testing.assert_array_equal(ck[rows], ref_ck)
        # size-independent properties: the kernel reproduces itself bit for bit
        w.run(4)
        assert w.verify() == 0
        assert pb.device_status(0) == 0


def test_rotating_copies_and_injection(cuda_device):
    with pb.Workload(pb.QG_FMT_INT8, 1024, 2048, 1024, copies=3, seed=11) as w:
        w.fill(11)
        w.golden()
        w.run(7)
        assert w.verify() == 0
        w.inject()
        assert w.verify() == 1
        log = w.mismatch_log()
        assert len(log) == 1 and log[0][0] == 0 and (log[0][1] ^ log[0][2]) == 0x80


def test_verify_words_counts_every_lane(cuda_device):
    a = torch.arange(0, 4099, dtype=torch.int32, device=cuda_device)
    for lane in range(4):
        b = a.clone()
        b[8 + lane] ^= 0x100
        b[4098] ^= 1  # tail word
        n, log = pb.verify_words(b, a)
        assert n == 2
        assert sorted(e[0] for e in log) == [8 + lane, 4098]
