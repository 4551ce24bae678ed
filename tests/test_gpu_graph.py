"""qg_run_graph on a B200: a batch captured as a CUDA graph and replayed runs the same
launches as qg_run.

* Each format gives the golden result bit for bit, with every launch checked.
* A corruption in one batch is caught by the per-launch check of the replayed graph,
  even after a later batch overwrites that output.  The graph captured before
  qg_golden, which carries no checks, is not replayed after it.
* Batch lengths that start at different operand copies each get their own graph.
"""
import pytest
import torch

import pantheon_b200 as pb

pytestmark = pytest.mark.gpu

CASES = [("int8", pb.QG_FMT_INT8, (128, 1024, 512)), ("int8_pair", pb.QG_FMT_INT8, (1024, 768, 256)),
         ("fp8", pb.QG_FMT_FP8, (256, 512, 1024)), ("nvfp4", pb.QG_FMT_NVFP4, (256, 512, 512)),
         ("bf16", pb.QG_FMT_BF16, (512, 512, 256)), ("w4a16_m1", pb.QG_FMT_W4A16, (1, 4096, 2048)),
         ("w4a16_m8", pb.QG_FMT_W4A16, (8, 4096, 2048)), ("w4a16_m12", pb.QG_FMT_W4A16, (12, 4096, 2048)),
         ("w4a16_m16", pb.QG_FMT_W4A16, (16, 4096, 2048))]


@pytest.mark.parametrize("name,fmt,shape", CASES, ids=[c[0] for c in CASES])
def test_graph_batches_reproduce_the_golden_result(cuda_device, name, fmt, shape):
    with pb.Workload(fmt, *shape, copies=2, seed=7) as w:
        w.fill(7)
        w.golden()
        for n in (4, 4, 3, 3, 1):   # repeated lengths replay; odd ones start at either copy
            w.run_graph(n)
        torch.cuda.synchronize()
        assert w.verify() == 0
        assert w.verify_detail() == (0, 0, 15)
        assert pb.device_status(0) == 0


def test_graph_batch_catches_a_corruption_later_overwritten(cuda_device):
    shape = (1024, 768, 256)
    with pb.Workload(pb.QG_FMT_INT8, *shape, copies=2, seed=11) as w:
        w.fill(11)
        w.run_graph(2)        # captured before the golden run: no checks in it
        w.golden()
        s = torch.cuda.current_stream()
        w.flip_operand_bit(0, 0, 4096, 6, s)
        w.run_graph(2, s)     # copy 0 computes a wrong result
        w.flip_operand_bit(0, 0, 4096, 6, s)
        w.run_graph(2, s)     # ... which this batch overwrites with the right one
        torch.cuda.synchronize()
        assert w.verify() >= 1
        words, launch_diffs, launches = w.verify_detail()
        assert words == 0 and launch_diffs >= 1 and launches == 4
        w.run_graph(2)
        assert w.verify() == 0


def test_graph_and_eager_batches_interleave(cuda_device):
    with pb.Workload(pb.QG_FMT_W4A16, 8, 4096, 2048, copies=4, seed=3) as w:
        w.fill(3)
        w.golden()
        for _ in range(3):
            w.run(5)
            w.run_graph(8)
            w.run_graph(5)
        torch.cuda.synchronize()
        assert w.verify() == 0
        assert w.verify_detail()[2] == 54


def test_graph_cache_keeps_the_latest_batches(cuda_device):
    """More distinct batch lengths than the cache holds: the oldest graphs are evicted
    (after the device drains) and every batch still runs and checks correctly."""
    with pb.Workload(pb.QG_FMT_W4A16, 1, 4096, 2048, copies=1, seed=9) as w:
        w.fill(9)
        w.golden()
        total = 0
        for n in list(range(1, 21)) + [1, 2, 3]:
            w.run_graph(n)
            total += n
        torch.cuda.synchronize()
        assert w.verify() == 0
        assert w.verify_detail()[2] == total
