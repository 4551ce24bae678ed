"""The drop-in boundary held to the reference runner itself (no GPU).

* pantheon_b200.install_dropin puts the binaries into a build cache that the
  runner's own is_build_cache_current accepts (pantheon.py:2606-2671), so the
  runner uses them instead of rebuilding.
Tests that call the runner skip where it is not found (tests/reference_runner.py).
"""
import json
import os
from pathlib import Path

import pytest

from pantheon_b200 import install_dropin
from tests.reference_runner import load_runner

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture()
def runner():
    mod = load_runner()
    if mod is None:
        pytest.skip("reference runner (pantheon.py) not found; set PANTHEON_REFERENCE")
    return mod


def _dropin_env(monkeypatch, tmp_path):
    monkeypatch.setenv("PANTHEON_BUILD_CACHE_DIR", str(tmp_path / "cache"))
    monkeypatch.setenv("PANTHEON_CUDA_ARCH", "100")
    monkeypatch.delenv("TARGET_GFX", raising=False)
    monkeypatch.delenv("ENABLE_HIPRT", raising=False)


def _stand_ins_for_the_runners_own_builds(runner, build_dir: Path):
    """The other workload binaries of the runner's registry, which its own `make` builds
    once before the drop-in is installed; here empty executables stand in for them
    (nothing runs them)."""
    build_dir.mkdir(parents=True, exist_ok=True)
    for p in runner.expected_build_binaries():
        if os.path.basename(p) not in install_dropin.DROPIN_BINARIES:
            Path(p).write_text("#!/bin/sh\nexit 0\n")
            os.chmod(p, 0o755)


def test_install_makes_the_runner_use_the_dropin(runner, monkeypatch, tmp_path, qglib):
    _dropin_env(monkeypatch, tmp_path)
    build_dir = Path(runner.configure_build_directory("CUDA"))
    assert build_dir == tmp_path / "cache" / runner.PANTHEON_VERSION / "cuda-100a"
    _stand_ins_for_the_runners_own_builds(runner, build_dir)
    assert not runner.is_build_cache_current("CUDA")
    got = install_dropin.install(runner, "CUDA")
    assert got == build_dir
    assert runner.is_build_cache_current("CUDA")
    for name in install_dropin.DROPIN_BINARIES + (install_dropin.LIBRARY,):
        assert (build_dir / name).read_bytes() == (install_dropin.LIB_DIR / name).read_bytes()
    assert not set(install_dropin.DROPIN_BINARIES) & set(runner.stale_workload_binaries())
    # the cache file is the runner's own format
    cached = json.loads((build_dir / ".pantheon_build_cache.json").read_text())
    assert cached["target"] == "100a" and cached["platform"] == "CUDA"
    assert set(install_dropin.DROPIN_BINARIES) <= set(cached["binaries"])
    # a fresh runner process (a new import) sees the same cache as current
    again = load_runner()
    again.configure_build_directory("CUDA")
    assert again.is_build_cache_current("CUDA")
    # without one of our binaries the runner would rebuild
    (build_dir / "quantized_gemm").unlink()
    assert not again.is_build_cache_current("CUDA")


def test_install_refuses_an_incomplete_build_directory(runner, monkeypatch, tmp_path, qglib):
    _dropin_env(monkeypatch, tmp_path)
    with pytest.raises(install_dropin.InstallError, match="not built"):
        install_dropin.install(runner, "CUDA")


def test_install_script_end_to_end(runner, monkeypatch, tmp_path, qglib):
    """The command-line entry point does the same for a maintainer."""
    from tests.reference_runner import reference_dir
    _dropin_env(monkeypatch, tmp_path)
    build_dir = Path(runner.configure_build_directory("CUDA"))
    _stand_ins_for_the_runners_own_builds(runner, build_dir)
    assert install_dropin.main(["--runner", str(reference_dir())]) == 0
    assert runner.is_build_cache_current("CUDA")
