"""Host logic of bench.py's multi-GPU run (one process per GPU, independent replicas), on CPU
with world_size-2 gloo process groups: the max-over-ranks device time, the whole-job rate,
and the reference arm's rank handling (only rank 0 runs and prints)."""

from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, REPO)
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench.barrier(world)
        ms = [120.0, 150.0][rank]   # per-rank device time of the timed region
        m = bench.max_over_ranks(ms, world, 0)
        out[rank] = (m, bench.job_rate(512 * 5, world, m))
        bench.barrier(world)
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_job_rate_gloo_world2():
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
        res = dict(out)
    for rank in (0, 1):
        m, rate = res[rank]
        assert m == 150.0, "every rank sees the slowest rank's time"
        assert rate == pytest.approx(2 * 512 * 5 / 0.150), "whole-job tokens over the slowest rank's time"


def test_reference_arm_runs_on_rank0_only():
    """Under torchrun the reference arm's non-zero ranks exit 0 without work or output."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1", "--warmup", "3"], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_job_rate_single_rank():
    sys.path.insert(0, REPO)
    import bench
    assert bench.job_rate(512, 1, 250.0) == pytest.approx(2048.0)
