"""Interleaved A/B of this library's GEMMs against the vendor library (cuBLAS through
torch) on the same operands and the same GPU, with the SM clock sampled per batch.

    python -m pantheon_b200.vendor_ab --format nvfp4|bf16|fp16|e4m3|int8 [--m M --n N --k K]
                                      [--batch 20] [--repeats 6]

Each repeat runs one batch of ours then one batch of the vendor GEMM (the
order alternates every repeat, so neither side always runs on the warmer or
cooler GPU), each batch device-timed with CUDA events.  The SM clock is read
through NVML (read-only) every 50 ms during each batch; a batch's rate is
also reported per GHz of its median clock, since on a 1 kW part both sides run
at whatever clock the power cap leaves and a raw comparison of batches run at
different clocks says little.  Prints one JSON line per batch and a summary
line: the median rate of each side, the median of the per-repeat ratios, and
the same for the clock-normalised rates.  A measurement tool: the product path
never calls the vendor library.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
import threading
import time

import torch

import pantheon_b200 as pb

DEFAULT_SHAPES = {"nvfp4": (16384, 16384, 16384), "bf16": (8192, 8192, 8192), "fp16": (8192, 8192, 8192),
                  "e4m3": (8192, 8192, 8192), "int8": (8192, 8192, 8192)}


class ClockPoll:
    """SM clock (MHz) of one GPU, read through NVML every `period` seconds while active."""

    def __init__(self, index: int, period: float = 0.05):
        self.samples: list[float] = []
        self.period = period
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._nv = pynvml
        except Exception:
            self._nv = None

    def __enter__(self):
        self.samples = []
        self._stop.clear()
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(float(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM)))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._nv is not None:
            self._t.join()

    def median(self):
        return statistics.median(self.samples) if self.samples else None


def setup(fmt: str, M: int, N: int, K: int):
    """(ours, theirs, work, out) -- two callables that each launch one GEMM on the
    current stream, on the same operands; the useful operations of one launch;
    the tensor ours() writes (theirs() returns its result)."""
    import torch.nn.functional as F
    dev = torch.device("cuda:0")
    if fmt == "nvfp4":
        A, sfa, B, sfb, g = pb.gen_nvfp4(M, N, K, seed=4)
        ga, gb = [float(x) for x in g.cpu()]
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        tga, tgb = torch.tensor(ga, device=dev), torch.tensor(gb, device=dev)
        a4, b4t = A.view(torch.float4_e2m1fn_x2), B.view(torch.float4_e2m1fn_x2).t()
        sa8, sb8 = sfa.view(torch.float8_e4m3fn), sfb.view(torch.float8_e4m3fn)

        def ours():
            pb.gemm_nvfp4(A, sfa, B, sfb, ga, gb, out=out)

        def theirs():
            return F.scaled_mm(a4, b4t, [sa8, tga], [F.ScalingType.BlockWise1x16, F.ScalingType.TensorWise],
                               [sb8, tgb], [F.ScalingType.BlockWise1x16, F.ScalingType.TensorWise],
                               swizzle_a=[F.SwizzleType.SWIZZLE_32_4_4, F.SwizzleType.NO_SWIZZLE],
                               swizzle_b=[F.SwizzleType.SWIZZLE_32_4_4, F.SwizzleType.NO_SWIZZLE],
                               output_dtype=torch.bfloat16)
    elif fmt == "int8":
        A = pb.gen_i8(M * K, seed=3, tensor_id=0)[:M * K].view(M, K)
        B = pb.gen_i8(N * K, seed=3, tensor_id=1)[:N * K].view(N, K)
        out = torch.empty((M, N), dtype=torch.int32, device=dev)
        Bt = B.t()

        def ours():
            pb.gemm_i8(A, B, None, None, out_type=pb.QG_OUT_S32, out=out)

        def theirs():
            return torch._int_mm(A, Bt)
    else:
        qfmt = {"bf16": pb.QG_FMT_BF16, "fp16": pb.QG_FMT_FP16, "e4m3": pb.QG_FMT_E4M3}[fmt]
        A = pb.gen_dense(qfmt, M, K, seed=5, tensor_id=0)
        B = pb.gen_dense(qfmt, N, K, seed=5, tensor_id=1)
        if fmt == "e4m3":
            out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            a8, b8t = A.view(torch.float8_e4m3fn), B.view(torch.float8_e4m3fn).t()
            one = torch.tensor(1.0, device=dev)

            def ours():
                pb.gemm_e4m3(A, B, 1.0, out_type=pb.QG_OUT_BF16, out=out)

            def theirs():
                return torch._scaled_mm(a8, b8t, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        else:
            ot = pb.QG_OUT_BF16 if fmt == "bf16" else pb.QG_OUT_F16
            out = torch.empty((M, N), dtype=A.dtype, device=dev)
            Bt = B.t()
            entry = pb.gemm_bf16 if fmt == "bf16" else pb.gemm_f16

            def ours():
                entry(A, B, 1.0, out_type=ot, out=out)

            def theirs():
                return torch.matmul(A, Bt)
    return ours, theirs, 2.0 * M * N * K, out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--format", choices=sorted(DEFAULT_SHAPES), default="nvfp4")
    ap.add_argument("--m", type=int, default=0)
    ap.add_argument("--n", type=int, default=0)
    ap.add_argument("--k", type=int, default=0)
    ap.add_argument("--batch", type=int, default=20)
    ap.add_argument("--repeats", type=int, default=6)
    a = ap.parse_args(argv)
    M, N, K = (a.m or DEFAULT_SHAPES[a.format][0], a.n or DEFAULT_SHAPES[a.format][1],
               a.k or DEFAULT_SHAPES[a.format][2])
    torch.cuda.set_device(0)
    ours, theirs, work, out = setup(a.format, M, N, K)
    s = torch.cuda.current_stream()
    for f in (ours, theirs):          # warm-up (and the vendor library's algorithm selection)
        for _ in range(3):
            f()
    torch.cuda.synchronize()
    # the two results on the same operands: largest difference relative to the
    # vendor result's rms (0 where both are bit-identical)
    ref = theirs().float()
    ours()
    torch.cuda.synchronize()
    agree = (out.float() - ref).abs().max().item() / max(ref.pow(2).mean().sqrt().item(), 1e-30)
    poll = ClockPoll(0)
    rates = {"ours": [], "vendor": []}
    per_ghz = {"ours": [], "vendor": []}
    for r in range(a.repeats):
        order = (("ours", ours), ("vendor", theirs)) if r % 2 == 0 else (("vendor", theirs), ("ours", ours))
        for name, f in order:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with poll:
                e0.record(s)
                for _ in range(a.batch):
                    f()
                e1.record(s)
                torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / a.batch
            tops = work / (ms / 1e3) / 1e12
            mhz = poll.median()
            rates[name].append(tops)
            per_ghz[name].append(tops / (mhz / 1000.0) if mhz else None)
            print(json.dumps({"repeat": r, "impl": name, "ms_per_launch": ms, "tops": tops, "sm_mhz": mhz}), flush=True)
    ratios = [o / v for o, v in zip(rates["ours"], rates["vendor"])]
    summary = {"format": a.format, "shape": [M, N, K], "batch": a.batch, "repeats": a.repeats,
               "ours_tops_median": statistics.median(rates["ours"]),
               "vendor_tops_median": statistics.median(rates["vendor"]),
               "ratio_median": statistics.median(ratios), "ratio_min": min(ratios), "ratio_max": max(ratios),
               "max_diff_over_rms": agree}
    if all(x is not None for x in per_ghz["ours"] + per_ghz["vendor"]):
        rg = [o / v for o, v in zip(per_ghz["ours"], per_ghz["vendor"])]
        summary.update({"ours_tops_per_ghz_median": statistics.median(per_ghz["ours"]),
                        "vendor_tops_per_ghz_median": statistics.median(per_ghz["vendor"]),
                        "ratio_per_ghz_median": statistics.median(rg)})
    print(json.dumps({"summary": summary}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
