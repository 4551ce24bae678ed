"""Every launch checks its own result (qg_run's per-launch check) on a B200.

A batch is many launches that overwrite one output, and the final bitwise
compare sees only the last.  Here one launch in the middle of a batch reads a
corrupted operand (one bit flipped on the stream before it and flipped back
after it, so the launches after it are correct again and overwrite its
output): the final compare finds nothing, and the per-launch check must
(mma_virus.cpp:156-173 is the reference's compare; it too sees only the last
output).  A clean batch must report no difference, and the counts reach the
binary's output.
"""
import subprocess

import pytest

pytestmark = pytest.mark.gpu

# (case, shape, operand slot to corrupt, byte, bit): the bit is chosen to change the
# element a lot (an exponent bit of a bf16 / e4m3 value, bit 6 of an int8, the
# magnitude bit of an e2m1 code), so the wrong result survives rounding to bf16.
CASES = [
    ("int8", (128, 1024, 512), 0, 0, 6),           # single-CTA kernel (M < 256)
    ("int8_pair", (1024, 768, 256), 0, 4096, 6),   # CTA-pair kernel
    ("fp8", (256, 512, 1024), 0, 0, 6),
    ("nvfp4", (256, 512, 512), 0, 0, 2),
    ("bf16", (512, 512, 256), 0, 1, 6),
    ("e4m3", (256, 512, 256), 0, 0, 6),
    ("w4a16_m1", (1, 4096, 2048), 0, 1, 6),         # CUDA-core GEMV
    ("w4a16_m8", (8, 4096, 2048), 0, 1, 6),         # warp-MMA GEMV
    ("w4a16_m12", (12, 4096, 2048), 0, 1, 6),       # warp-MMA GEMV, three B fragments
    ("w4a16_m16", (16, 4096, 2048), 0, 1, 6),       # tcgen05 GEMV
]


def _fmt(name):
    import pantheon_b200 as pb
    return {"int8": pb.QG_FMT_INT8, "int8_pair": pb.QG_FMT_INT8, "fp8": pb.QG_FMT_FP8, "nvfp4": pb.QG_FMT_NVFP4,
            "bf16": pb.QG_FMT_BF16, "e4m3": pb.QG_FMT_E4M3, "w4a16_m1": pb.QG_FMT_W4A16,
            "w4a16_m8": pb.QG_FMT_W4A16, "w4a16_m12": pb.QG_FMT_W4A16, "w4a16_m16": pb.QG_FMT_W4A16}[name]


@pytest.mark.parametrize("name,shape,slot,byte,bit", CASES, ids=[c[0] for c in CASES])
def test_clean_batch_reports_nothing(cuda_device, name, shape, slot, byte, bit):
    import pantheon_b200 as pb
    with pb.Workload(_fmt(name), *shape, copies=2, seed=11) as w:
        w.fill(11)
        w.golden()
        w.run(6)
        assert w.verify() == 0
        assert w.verify_detail() == (0, 0, 6)


@pytest.mark.parametrize("name,shape,slot,byte,bit", CASES, ids=[c[0] for c in CASES])
def test_corrupted_middle_launch_is_caught(cuda_device, name, shape, slot, byte, bit):
    import pantheon_b200 as pb
    with pb.Workload(_fmt(name), *shape, copies=2, seed=11) as w:
        w.fill(11)
        w.golden()
        w.run(2)                              # copies 0, 1: clean
        w.flip_operand_bit(0, slot, byte, bit)
        w.run(1)                              # copy 0 with one operand bit flipped
        w.flip_operand_bit(0, slot, byte, bit)
        w.run(3)                              # copies 1, 0, 1: clean again, outputs overwritten
        total = w.verify()
        words, diffs, launches = w.verify_detail()
        assert words == 0, "the final outputs are clean: only the per-launch check can see the bad launch"
        assert diffs >= 1 and total == diffs
        assert launches == 6
        # the next batch starts from zero
        w.run(4)
        assert w.verify() == 0 and w.verify_detail() == (0, 0, 4)


def test_binary_reports_checked_launches(cuda_device):
    from pantheon_b200 import BIN_PATH
    p = subprocess.run([str(BIN_PATH), "0", "1", "50", "--verify", "--m", "1024", "--n", "1024", "--k", "1024"],
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout + p.stderr
    line = next(x for x in p.stdout.splitlines() if "-> Launches Checked:" in x)
    checked, total = line.split(":")[1].split("(")[0].split(" of ")
    assert int(checked) == int(total) > 0
