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
