"""qg_golden_digest on a B200.

* The device digest equals its numpy restatement over the golden words (and,
  for INT8, the golden row checksums).
* Two contexts built with the same arguments give the same digest.
* Another seed gives another digest, and so does one flipped bit of the golden.

The restatement: the sum mod 2^64 of splitmix64(i * 0x9E3779B97F4A7C15 + w_i +
salt) over the 32-bit words w_i.  The salt is 0 for the output and
0xC2B2AE3D27D4EB4F for the row checksums.
"""
import numpy as np
import pytest
import torch

import pantheon_b200 as pb
from pantheon_b200.ops import _DeviceBytes

pytestmark = pytest.mark.gpu
GAMMA = np.uint64(0x9E3779B97F4A7C15)
CKSUM_SALT = 0xC2B2AE3D27D4EB4F


def _mix(z):
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def _digest(words: np.ndarray, salt: int) -> int:
    with np.errstate(over="ignore"):
        i = np.arange(words.size, dtype=np.uint64)
        return int(_mix(i * GAMMA + words.astype(np.uint64) + np.uint64(salt)).sum(dtype=np.uint64))


def _words(w, slot):
    return w.tensor(0, slot, torch.int32).cpu().numpy().view(np.uint32)


# every output here has a whole number of 32-bit words
CASES = [("int8", pb.QG_FMT_INT8, (256, 512, 256)), ("fp8", pb.QG_FMT_FP8, (256, 512, 1024)),
         ("nvfp4", pb.QG_FMT_NVFP4, (256, 512, 512)), ("w4a16_m8", pb.QG_FMT_W4A16, (8, 4096, 2048)),
         ("w4a16_m16", pb.QG_FMT_W4A16, (16, 4096, 2048)), ("bf16", pb.QG_FMT_BF16, (256, 256, 256))]


@pytest.mark.parametrize("name,fmt,shape", CASES, ids=[c[0] for c in CASES])
def test_digest_matches_restatement_and_other_contexts(cuda_device, name, fmt, shape):
    with pb.Workload(fmt, *shape, copies=2, seed=5) as w, pb.Workload(fmt, *shape, copies=1, seed=5) as v:
        for x in (w, v):
            x.fill(5)
            x.golden()
        d = w.golden_digest(0)
        expect = _digest(_words(w, w.SLOT_GOLDEN), 0)
        if fmt == pb.QG_FMT_INT8:
            expect = (expect + _digest(_words(w, w.SLOT_CKSUM), CKSUM_SALT)) % (1 << 64)
        assert d == expect
        # another context with the same arguments (and another copy count): the same digest
        assert v.golden_digest(0) == d
        # the copies of one context hold differently seeded operands
        assert w.golden_digest(1) != d


def test_digest_changes_with_the_seed_and_a_flipped_golden_bit(cuda_device):
    shape = (256, 512, 256)
    with pb.Workload(pb.QG_FMT_INT8, *shape, seed=5) as w, pb.Workload(pb.QG_FMT_INT8, *shape, seed=6) as v:
        w.fill(5)
        w.golden()
        v.fill(6)
        v.golden()
        d = w.golden_digest(0)
        assert v.golden_digest(0) != d
        ptr, nbytes = w.tensor_ptr(0, w.SLOT_GOLDEN)
        gold = torch.as_tensor(_DeviceBytes(ptr, nbytes), device=cuda_device)   # a view, not a copy
        gold[12345] ^= 0x10
        torch.cuda.synchronize()
        assert w.golden_digest(0) != d
        gold[12345] ^= 0x10
        torch.cuda.synchronize()
        assert w.golden_digest(0) == d


def test_digest_needs_a_golden(cuda_device):
    with pb.Workload(pb.QG_FMT_INT8, 256, 512, 256) as w:
        w.fill(1)
        with pytest.raises(pb.QGError):
            w.golden_digest(0)
