"""Install the three drop-in workload binaries into a Pantheon build cache.

    python -m pantheon_b200.install_dropin --runner DIR [--platform CUDA] [--cache-dir DIR]

Pantheon's runner uses prebuilt workload binaries only while the build cache
of its platform and target is current (pantheon.py:2606-2671): the directory
`<cache root>/<version>/cuda-100a/` holds every workload binary of its
registry plus `.pantheon_build_cache.json`, whose content must equal the
runner's `build_cache_key` (platform, target "100a", a digest of its kernel
sources, the binary names).  Otherwise it re-runs `make -k` there, which would
rebuild the reference workloads over ours.

This script takes the runner itself (its `pantheon.py`, in `--runner DIR`) as
the authority on that key:
  1. it resolves the build directory with the runner's
     `configure_build_directory` (set PANTHEON_BUILD_CACHE_DIR, or pass
     --cache-dir, to choose the cache root; PANTHEON_CUDA_ARCH=100 names the
     target on a build node without a GPU);
  2. copies `quantized_gemm`, `llm_decode`, `mma_virus` and the library they
     load (`libpantheon_qgemm.so`, found beside them through their rpath)
     into it, over the reference builds of those three names;
  3. checks that the runner's other workload binaries are already there (built
     by the runner's own `make`, once, before this step);
  4. writes `.pantheon_build_cache.json` from the runner's `build_cache_key`,
     in the runner's own format, and confirms `is_build_cache_current`.
After a change to the runner's kernel sources the key changes, the runner
rebuilds everything, and this script has to be run again.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import shutil
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_DIR = PKG / "lib"
DROPIN_BINARIES = ("quantized_gemm", "llm_decode", "mma_virus")
LIBRARY = "libpantheon_qgemm.so"


class InstallError(RuntimeError):
    pass


def load_runner_module(runner_dir: str | os.PathLike):
    """Import the runner's pantheon.py from `runner_dir` (no byte-code written there)."""
    path = Path(runner_dir) / "pantheon.py"
    if not path.is_file():
        raise InstallError(f"no pantheon.py in {runner_dir}")
    spec = importlib.util.spec_from_file_location("_pantheon_runner_for_install", path)
    mod = importlib.util.module_from_spec(spec)
    old = sys.dont_write_bytecode
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(path.parent))  # the runner imports its sibling module `monitor`
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.path.remove(str(path.parent))
        sys.dont_write_bytecode = old
    return mod


def install(runner, platform: str = "CUDA", lib_dir: Path = LIB_DIR) -> Path:
    """Install the drop-in binaries into `runner`'s build directory for `platform` and
    write the cache file that makes the runner use them.  Returns the build directory."""
    for name in DROPIN_BINARIES + (LIBRARY,):
        if not (lib_dir / name).is_file():
            raise InstallError(f"{lib_dir / name} is missing: build with python -m pantheon_b200.build first")
    build_dir = Path(runner.configure_build_directory(platform))
    build_dir.mkdir(parents=True, exist_ok=True)
    # copy (not copy2): the installed files are new, so the runner's staleness check
    # (binary older than its sources) never reads them as a failed rebuild
    shutil.copy(lib_dir / LIBRARY, build_dir / LIBRARY)
    for name in DROPIN_BINARIES:
        shutil.copy(lib_dir / name, build_dir / name)
        os.chmod(build_dir / name, 0o755)
    missing = [p for p in runner.expected_build_binaries()
               if not (os.path.isfile(p) and os.access(p, os.X_OK))]
    if missing:
        raise InstallError("the runner's other workload binaries are not built in "
                           f"{build_dir} (run its `make` there first): "
                           + ", ".join(sorted(os.path.basename(p) for p in missing)))
    key = runner.build_cache_key(platform)
    with open(runner.BUILD_CACHE_FILE, "w", encoding="utf-8") as f:
        json.dump(key, f, indent=2, sort_keys=True)
    if not runner.is_build_cache_current(platform):
        raise InstallError(f"the runner does not accept the cache written to {runner.BUILD_CACHE_FILE}")
    return build_dir


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--runner", required=True, help="directory holding Pantheon's pantheon.py")
    ap.add_argument("--platform", default="CUDA")
    ap.add_argument("--cache-dir", help="cache root (sets PANTHEON_BUILD_CACHE_DIR for the runner)")
    a = ap.parse_args(argv)
    if a.cache_dir:
        os.environ["PANTHEON_BUILD_CACHE_DIR"] = a.cache_dir
    try:
        build_dir = install(load_runner_module(a.runner), a.platform)
    except InstallError as e:
        print(f"install_dropin: {e}", file=sys.stderr)
        return 1
    print(f"installed {', '.join(DROPIN_BINARIES)} into {build_dir}; build cache current")
    return 0


if __name__ == "__main__":
    sys.exit(main())
