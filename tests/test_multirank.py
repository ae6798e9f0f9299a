"""The N > 1 host path of bench.py on CPU: two gloo ranks (the GPU run uses NCCL with one
process per GPU). Covers the rank bookkeeping the scaling run relies on: the job time is
the slowest rank's, whole-job rows/s counts every rank's rows, every rank passes the same
barriers, and the reference arm runs on rank 0 only."""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    import bench

    w, r, local = bench.dist_setup(backend="gloo")
    assert (w, r, local) == (world, rank, rank)
    # each rank "took" a different time; every rank must agree on the slowest one
    mine = 100.0 + 25.0 * rank
    bench.barrier(w)
    slowest = bench.max_over_ranks(mine, w, torch.device("cpu"))
    bench.barrier(w)
    out.put((rank, slowest, bench.weak_rows_per_s(w, bench.BATCH, 1000, slowest)))
    dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_job_time():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    got = sorted(out.get(timeout=5) for _ in range(world))
    slowest = 100.0 + 25.0 * (world - 1)
    for rank, value, rows in got:
        assert value == slowest
        assert rows == world * 64 * 1000 / (slowest / 1e3)


def test_reference_arm_only_on_rank_zero():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1")
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "3",
                          "--warmup", "3"], env=env, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0
    assert res.stdout.strip() == ""
