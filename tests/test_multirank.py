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


# ----------------------------------------------------------------------------------------
# vocab-sharded exchange on two gloo ranks, the oracle standing in for the two CUDA steps
# ----------------------------------------------------------------------------------------

SH_ROWS, SH_VOCAB, SH_WORLD = 6, 8192, 2


def _sharded_inputs():
    from sonic_sampler_b200 import workloads

    w = workloads.config2("cpu", seed=31, batch=SH_ROWS, vocab=SH_VOCAB)
    b = w["buffers"]
    ind = b.flags.packed[:, 0].to(torch.int32)
    ind[::3] |= 0x40  # greedy rows too
    b.flags.packed[:, 0] = ind.to(torch.uint16)
    kw = dict(grammar=b.grammar[:, 0], context_counts=b.repetition.counts.context,
              decode_counts=b.repetition.counts.decode, repetition_penalties=b.repetition.multiplicative,
              frequency_penalties=b.repetition.frequency, presence_penalties=b.repetition.presence,
              logit_bias=b.bias, temperature=b.temperature, top_k=b.top_k, top_p=b.top_p, min_p=b.min_p,
              top_k_logprobs=b.top_logprobs, gumbel_noise=b.weights.gumbel.target[:, 0], return_logprobs=True,
              block_n=1024)
    return w["logits"], b.flags.target, kw


def _sharded_rank_main(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import datetime

    import torch.distributed as dist

    from oracle import oracle
    from sonic_sampler_b200.interface.functional.singular import prepare_singular, vocab_sharded_exchange

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    logits, ind, kw = _sharded_inputs()
    shard = SH_VOCAB // world
    local = logits[:, rank * shard:(rank + 1) * shard].contiguous()
    sel, args = prepare_singular(local, ind, world_size=world, local_rank=rank, shard_size=shard, **kw)
    vocab_sharded_exchange(args, SH_ROWS, world, shard, torch.device("cpu"), extract=oracle.shard_candidates,
                           merge=oracle.merge_candidates)
    out.put((rank, sel.tokens.clone(), sel.logprobs.selected.view(torch.int16).clone()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_vocab_sharded_exchange_matches_unsharded():
    """Each rank extracts its shard's candidates, one all-gather exchanges them, and every rank
    merges and selects: both ranks return the same tokens and logprobs, and those equal the
    unsharded selection over the whole vocabulary (greedy rows included)."""
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.singular import prepare_singular

    port = _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_sharded_rank_main, args=(r, SH_WORLD, port, out)) for r in range(SH_WORLD)]
    for p in procs:
        p.start()
    got = sorted((out.get(timeout=90) for _ in range(SH_WORLD)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    logits, ind, kw = _sharded_inputs()
    ref, args = prepare_singular(logits, ind, **kw)
    oracle.fused_singular(args)
    stoch = ~(ind.to(torch.int32) & 0x40).bool()
    for _, tokens, lp in got:
        assert torch.equal(tokens, ref.tokens)
        assert torch.equal(lp[stoch], ref.logprobs.selected.view(torch.int16)[stoch])
