"""Run a few launches of one workload kernel, for profilers (ncu) and quick timing.

    python -m pantheon_b200.profile_case --format int8|fp8|nvfp4|w4a16|bf16|fp16|tf32|e4m3|fp32
                                         [--m M --n N --k K] [--iters 3] [--copies 1]

Fills the operands, computes the golden result (one launch), then runs
`--iters` launches and synchronizes.  Prints the mean device time per launch
measured with CUDA events (not meaningful under a profiler).
"""
from __future__ import annotations

import argparse
import sys

import torch

import pantheon_b200 as pb

FORMATS = {"int8": pb.QG_FMT_INT8, "fp8": pb.QG_FMT_FP8, "nvfp4": pb.QG_FMT_NVFP4, "w4a16": pb.QG_FMT_W4A16,
           "bf16": pb.QG_FMT_BF16, "fp16": pb.QG_FMT_FP16, "tf32": pb.QG_FMT_TF32, "e4m3": pb.QG_FMT_E4M3,
           "fp32": pb.QG_FMT_FP32}
# output type of each format (the dense furnace formats write their own type, tf32 / fp32 fp32, e4m3 bf16)
OUT_TYPES = {"fp16": pb.QG_OUT_F16, "tf32": pb.QG_OUT_F32, "fp32": pb.QG_OUT_F32}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--format", choices=sorted(FORMATS), default="int8")
    ap.add_argument("--m", type=int, default=0)
    ap.add_argument("--n", type=int, default=0)
    ap.add_argument("--k", type=int, default=0)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--copies", type=int, default=1)
    ap.add_argument("--seed", type=int, default=1)
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    with pb.Workload(FORMATS[a.format], a.m, a.n, a.k, copies=a.copies, seed=a.seed,
                     out_type=OUT_TYPES.get(a.format, pb.QG_OUT_BF16)) as w:
        w.fill(a.seed)
        w.golden()
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        w.run(a.iters, s)
        e1.record(s)
        w.synchronize()
        ms = e0.elapsed_time(e1) / max(a.iters, 1)
        mm = w.verify()
        print(f"{a.format}: {ms:.4f} ms/launch, {w.ops_per_launch / ms / 1e9:.1f} TOPS, "
              f"{w.bytes_per_launch / ms / 1e6:.1f} GB/s, mismatches {mm}")
        return 0 if mm == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
