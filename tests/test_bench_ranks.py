"""bench.py's multi-rank host logic on CPU: two gloo ranks (no GPU).

The GPU bench runs one process per GPU under torchrun and reports the max over
ranks of each rank's device time; these tests drive the same reduction over
gloo, and check that the reference arm does its work on rank 0 only.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        # per-rank device times, mismatch counts and error flags differ; every rank must see the max
        got = bench.max_over_ranks([1.0 + rank, 10.0 - rank, float(rank == 1), 0.0], world)
        out[rank] = got
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_two_gloo_ranks():
    world, port = 2, _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_rank_main, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
        res = dict(out)
    assert res[0] == res[1] == [2.0, 10.0, 1.0, 0.0]


def test_max_over_ranks_single_process():
    assert bench.max_over_ranks([3.0, 4.0], 1) == [3.0, 4.0]


def test_reference_arm_runs_on_rank_0_only(capsys, monkeypatch):
    """Under torchrun every rank starts bench.py --impl reference; ranks > 0 exit 0 without work."""
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    assert bench.main(["--impl", "reference", "--gpus", "2", "--steps", "3", "--warmup", "3"]) == 0
    assert capsys.readouterr().out == ""


def _gather_main(rank, world, port, out):
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        # each rank's rate and mismatch count, as the secondary entries gather them
        out[rank] = bench.gather_over_ranks([100.0 + rank, float(rank)], world)
    finally:
        dist.destroy_process_group()


def test_gather_over_ranks_two_gloo_ranks():
    world, port = 2, _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_gather_main, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
        res = dict(out)
    assert res[0] == res[1] == [[100.0, 0.0], [101.0, 1.0]]


def test_gather_over_ranks_single_process():
    assert bench.gather_over_ranks([3.0, 4.0], 1) == [[3.0, 4.0]]


def test_reference_arm_line_has_our_config(capsys, monkeypatch):
    """The reference arm reports the same configuration, metric and unit as our arm; at a
    small GEMM size (patched in) each step computes the whole GEMM."""
    import json
    monkeypatch.setattr(bench, "M", 256)
    monkeypatch.setattr(bench, "N", 256)
    monkeypatch.setattr(bench, "K", 256)
    monkeypatch.setattr(bench, "reference_mock_rate", lambda: None)
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    assert bench.main(["--impl", "reference", "--steps", "2", "--warmup", "1"]) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    ours = bench.workload_spec("int8")
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == ours["unit"] == "TOPS"
    assert line["config"] == dict(ours["config"], parallelism="replicas x1 (independent instance per GPU)")
    assert line["cpu_baseline"]["rows_per_step"] == 256
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["value"] > 0


def test_roofline_picks_the_denominator_by_region_length():
    peaks = {"bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6500.0, "source": "measured"}
    wl = bench.workload_spec("int8")
    burst = bench.roofline(wl, 1.0, 1e-3, 0.01, peaks, traffic=1)
    sus = bench.roofline(wl, 1.0, 1e-3, 0.5, peaks, traffic=1)
    assert burst["peak"] == 3200.0 and sus["peak"] == 2800.0
    assert abs(sus["frac"] - 1000.0 / 2800.0) < 1e-12
    gemv = bench.roofline(bench.workload_spec("w4a16", 8), 0.125, 25e-6, 0.1, peaks, traffic=1)
    assert gemv["unit"] == "GB/s" and abs(gemv["achieved"] - 5000.0) < 1e-9 and gemv["peak"] == 6500.0
    fp4 = bench.roofline(bench.workload_spec("nvfp4"), 1.0, 1e-3, 0.5, peaks, traffic=1)
    assert fp4["peak"] == 5600.0
