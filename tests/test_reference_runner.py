"""The drop-in boundary held to the reference runner itself (no GPU).

* Real outputs of the three binaries on a B200 (tests/golden/binary_runs.json)
  go through the runner's own parse_kernel_output and assess_gpu
  (pantheon.py:3421-3513, 1303-1460): a clean --verify run is a PASS with the
  workload's unit, an --inject_error run is a FAIL, and the GPU verdict is
  WATCH with the runner as shipped and FAULT once pantheon_b200.runner_hook is
  installed (pantheon.py:1220-1223 decides which failures are faults).
* The restated reader the GPU tests use (tests/contract_parse.py) agrees with
  the runner's decisions on those outputs, recorded in
  tests/golden/runner_readings.json by make_runner_readings.py; this part
  needs no reference tree.
* pantheon_b200.install_dropin puts the binaries into a build cache that the
  runner's own is_build_cache_current accepts (pantheon.py:2606-2671), so the
  runner uses them instead of rebuilding.
Tests that call the runner skip where it is not found (tests/reference_runner.py).
"""
import json
import os
from pathlib import Path

import pytest

from pantheon_b200 import install_dropin, runner_hook
from tests.contract_parse import parse_kernel_output
from tests.reference_runner import load_runner

GOLDEN = Path(__file__).resolve().parent / "golden"


def _runs():
    return json.loads((GOLDEN / "binary_runs.json").read_text())


def _readings():
    return {r["case"]: r for r in json.loads((GOLDEN / "runner_readings.json").read_text())}


@pytest.fixture()
def runner():
    mod = load_runner()
    if mod is None:
        pytest.skip("reference runner (pantheon.py) not found; set PANTHEON_REFERENCE")
    return mod


def test_recorded_runs_cover_every_binary_and_outcome():
    runs = _runs()
    assert {r["test"] for r in runs} == {"quantized_gemm", "llm_decode", "mma_virus"}
    for r in runs:
        clean = "--inject_error" not in r["argv"]
        assert (r["returncode"] == 0) == clean, r["case"]
        assert ("Verification: PASS" in r["stdout"]) == (clean and "--verify" in r["argv"]), r["case"]


def test_restated_reader_matches_the_runner_on_real_runs():
    """tests/contract_parse.py reads every recorded run exactly as the runner did."""
    readings = _readings()
    for run in _runs():
        want = readings[run["case"]]
        score, unit, status, had_error, lines = parse_kernel_output(run["stdout"], run["stderr"],
                                                                    run["returncode"], run["test"])
        assert (score, unit, status, had_error) == (want["score"], want["unit"], want["status"],
                                                     want["had_error"]), run["case"]
        assert lines == want["kept_lines"], run["case"]
        assert runner_hook.row_fields(run["test"], run["stdout"]).get(runner_hook.ROW_FIELD) == want["sdc_mismatches"]


def test_recorded_verdicts():
    """Clean runs: PASS rows, HEALTHY GPU.  Injected faults: FAIL rows, WATCH as shipped
    ("did not complete"), FAULT with the hook installed."""
    units = {"quantized_gemm": {"TOPS", "GB/s"}, "llm_decode": {"GB/s"}, "mma_virus": {"TFLOPS"}}
    readings = _readings()
    for run in _runs():
        r = readings[run["case"]]
        if run["returncode"] == 0:
            assert r["status"] == "PASS" and r["unit"] in units[run["test"]] and r["score"] > 0, run["case"]
            assert r["verdict_shipped"] == r["verdict_with_hook"] == "HEALTHY", run["case"]
        else:
            assert r["status"] == "FAIL" and r["unit"] == "ERR", run["case"]
            assert r["verdict_shipped"] == "WATCH" and r["verdict_with_hook"] == "FAULT", run["case"]
            assert r["sdc_mismatches"] >= 1


def test_runner_reads_real_runs_as_recorded(runner):
    """The live runner module reproduces the committed readings."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_runner_readings", GOLDEN / "make_runner_readings.py")
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    assert mk.readings(runner, _runs()) == json.loads((GOLDEN / "runner_readings.json").read_text())


def test_hook_turns_an_injected_fault_into_a_fault_verdict(runner):
    run = next(r for r in _runs() if r["case"] == "quantized_gemm_inject")
    score, unit, status, _, _ = runner.parse_kernel_output(run["stdout"], run["stderr"], run["returncode"],
                                                           "quantized_gemm")
    assert status == "FAIL"
    row = runner.build_result_row("quantized_gemm", 3, 2, 50, score, unit, {}, status=status)
    assert runner.assess_gpu([row], 3, "NVIDIA B200")["verdict"] == "WATCH"
    assert runner_hook.install(runner) == {"quantized_gemm", "llm_decode", "mma_virus"}
    row.update(runner_hook.row_fields("quantized_gemm", run["stdout"]))
    verdict = runner.assess_gpu([row], 3, "NVIDIA B200")
    assert verdict["verdict"] == "FAULT"
    assert any("quantized_gemm failed" in f for f in verdict["findings"]["faults"])
    assert row[runner_hook.ROW_FIELD] >= 1


def test_hook_files_a_golden_digest_outlier_as_a_fault(runner):
    """Four GPUs run the same clean workload; one reports another golden digest.  Each
    run passes its own compares, so only the cross-GPU check finds it: after
    check_golden_digests the runner's own verdict is FAULT for that GPU alone."""
    run = next(r for r in _runs() if r["case"] == "quantized_gemm_clean")
    runner_hook.install(runner)
    rows = []
    for gpu, digest in enumerate(["0x00c0ffee00c0ffee"] * 3 + ["0x00c0ffee00c0ffef"]):
        out = run["stdout"].replace("  -> Kernel Loops:", f"  -> Golden Digest: {digest}\n  -> Kernel Loops:")
        score, unit, status, _, kept = runner.parse_kernel_output(out, run["stderr"], run["returncode"], "quantized_gemm")
        assert status == "PASS" and f"-> Golden Digest: {digest}" in kept
        row = runner.build_result_row("quantized_gemm", gpu, 2, 50, score, unit, {}, status=status)
        row.update(runner_hook.row_fields("quantized_gemm", out))
        rows.append(row)
    assert runner.assess_gpu(rows, 3, "NVIDIA B200")["verdict"] != "FAULT"
    bad = runner_hook.check_golden_digests(rows)
    assert [r["GPU ID"] for r in bad] == [3]
    assert runner.assess_gpu(rows, 3, "NVIDIA B200")["verdict"] == "FAULT"
    assert all(runner.assess_gpu(rows, g, "NVIDIA B200")["verdict"] != "FAULT" for g in range(3))


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
