"""Build the native parts of pantheon_b200 in-tree.

Outputs (git-ignored, but shipped with the tree to the GPU box):
  pantheon_b200/lib/libpantheon_qgemm.so   the C-ABI library (sm_100a kernels,
                                           static cudart; needs only libc at load)
  pantheon_b200/lib/quantized_gemm         the drop-in workload binary
                                           (rpath $ORIGIN -> the library beside it)

Every .cu file is compiled for sm_100a only:
  nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3
Usage: python -m pantheon_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = ROOT / "_build" / "obj"
LIB = LIB_DIR / "libpantheon_qgemm.so"
BIN = LIB_DIR / "quantized_gemm"
DECODE_BIN = LIB_DIR / "llm_decode"
MMA_BIN = LIB_DIR / "mma_virus"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                     "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, flush=True)


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def cuda_include() -> Path:
    """CUDA headers beside nvcc (the binary uses NVTX's header-only API)."""
    return Path(nvcc()).resolve().parent.parent / "include"


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))
    sources = sorted(CSRC.glob("*.cu"))
    cc = nvcc()
    jobs = []
    objs = []
    for src in sources:
        obj = OBJ_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs.append([cc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
            list(ex.map(lambda c: _run(c, verbose), jobs))
    if force or jobs or _stale(LIB, objs):
        _run([cc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs),
              "-Xlinker", "--exclude-libs,ALL"], verbose)
    main = CSRC / "quantized_gemm_main.cpp"
    for out, defs in ((BIN, []), (DECODE_BIN, ["-DQG_DECODE_BINARY"]), (MMA_BIN, ["-DQG_MMA_VIRUS_BINARY"])):
        if force or _stale(out, [main, LIB, ROOT / "include" / "pantheon_qgemm.h"]):
            _run(["g++", "-O2", "-std=c++17", *defs, f"-I{ROOT / 'include'}", f"-I{cuda_include()}", str(main),
                  "-o", str(out), f"-L{LIB_DIR}", "-lpantheon_qgemm", "-ldl", "-Wl,-rpath,$ORIGIN"], verbose)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    lib = build(force=a.force, verbose=a.verbose)
    print(f"built {lib}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
