"""Run the three drop-in binaries on a B200 and record what the runner would see.

    python tests/golden/capture_binary_runs.py OUT.json

Each case is one process launched the way Pantheon's runner launches a workload
(`<bin> 0 <duration> <mem_pct> --verify [--inject_error] [flags]`,
pantheon.py:3047-3055,3102); its argv, stdout, stderr and exit code are written
to OUT.json.  The committed copy (tests/golden/binary_runs.json) came from one
run of this script on a B200; make_runner_readings.py reads those outputs with
the reference runner's own parser and verdict, and the CPU tests hold both to
what the runner decides.  Needs the built binaries and a GPU; writes nothing else.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
LIB = ROOT / "pantheon_b200" / "lib"

# (case name, runner test name, binary, arguments after argv[0])
CASES = [
    ("quantized_gemm_clean", "quantized_gemm", "quantized_gemm", ["0", "3", "50", "--verify"]),
    ("quantized_gemm_inject", "quantized_gemm", "quantized_gemm", ["0", "2", "50", "--verify", "--inject_error"]),
    ("quantized_gemm_noverify", "quantized_gemm", "quantized_gemm", ["0", "2", "50"]),
    ("quantized_gemm_fp8", "quantized_gemm", "quantized_gemm", ["0", "2", "50", "--verify", "--format", "fp8"]),
    ("quantized_gemm_nvfp4", "quantized_gemm", "quantized_gemm", ["0", "2", "50", "--verify", "--format", "nvfp4"]),
    ("quantized_gemm_w4a16_m8", "quantized_gemm", "quantized_gemm",
     ["0", "2", "50", "--verify", "--format", "w4a16", "--m", "8"]),
    ("quantized_gemm_loops_invalid", "quantized_gemm", "quantized_gemm",
     ["0", "1", "50", "--verify", "--kernel_loops", "-1", "--warmup_iters", "-1"]),
    ("llm_decode_clean", "llm_decode", "llm_decode", ["0", "2", "50", "--verify"]),
    ("llm_decode_inject", "llm_decode", "llm_decode", ["0", "2", "50", "--verify", "--inject_error"]),
    ("mma_virus_clean", "mma_virus", "mma_virus", ["0", "2", "50", "--verify"]),
    ("mma_virus_fp8", "mma_virus", "mma_virus", ["0", "2", "50", "--verify", "--gemm_type", "fp8"]),
    ("mma_virus_inject", "mma_virus", "mma_virus", ["0", "2", "50", "--verify", "--inject_error"]),
]


def main(argv=None) -> int:
    out = Path((argv or sys.argv[1:])[0])
    runs = []
    for case, test, binary, args in CASES:
        p = subprocess.run([str(LIB / binary), *args], capture_output=True, text=True, timeout=600)
        runs.append({"case": case, "test": test, "argv": [binary, *args], "stdout": p.stdout, "stderr": p.stderr,
                     "returncode": p.returncode})
        print(f"{case}: rc={p.returncode}", flush=True)
    out.write_text(json.dumps(runs, indent=1) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
