"""Vocab-sharded singular sampling (sonic_shard_candidates -> all-gather -> sonic_merge_candidates)
against the unsharded path on the same inputs: identical tokens, logprobs and top-Z.

The single-GPU tests emulate the ranks: each shard's candidates are computed on cuda:0 and
stacked as the all-gather would. The NCCL test runs real ranks, one per GPU, and is skipped
on a box with fewer than two GPUs."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from sonic_sampler_b200 import workloads

pytestmark = pytest.mark.gpu

BF16, F32 = torch.bfloat16, torch.float32


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from sonic_sampler_b200 import _abi

    _abi.load_library()
    return torch.device("cuda", 0)


def _kwargs(b, **extra):
    kw = dict(
        indicators=b.flags.target, grammar=b.grammar[:, 0], context_counts=b.repetition.counts.context,
        decode_counts=b.repetition.counts.decode, repetition_penalties=b.repetition.multiplicative,
        frequency_penalties=b.repetition.frequency, presence_penalties=b.repetition.presence, logit_bias=b.bias,
        temperature=b.temperature, top_k=b.top_k, top_p=b.top_p, min_p=b.min_p, top_k_logprobs=b.top_logprobs,
        gumbel_noise=b.weights.gumbel.target[:, 0], return_logprobs=True, max_top_logprobs=8,
        logprobs_dtype=F32,
    )
    kw.update(extra)
    return kw


def _case(dev, rows, vocab, seed, greedy_every=0):
    b = workloads.sampling_buffers(rows, 1, vocab, dev, seed, workloads.config2_params(rows, seed + 1), top_logprobs=8)
    if greedy_every:
        ind = b.flags.target.cpu().to(torch.int32)
        ind[::greedy_every] |= 0x40
        b.flags.packed[:, 0] = ind.to(torch.uint16).to(dev)
    x = workloads.peaked_logits(rows, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=seed)
    return x, b


def _emulated_sharded(x, kw, world, shard):
    """Run the three steps for every shard on one GPU; returns the merged selection."""
    from sonic_sampler_b200 import ops
    from sonic_sampler_b200.interface.functional.singular import prepare_singular

    rows = x.size(0)
    gathered = torch.empty(world, rows, 128, dtype=torch.int64, device=x.device)
    keep = []
    for r in range(world):
        local = x[:, r * shard:(r + 1) * shard]
        _, args = prepare_singular(local, world_size=world, local_rank=r, shard_size=shard, **kw)
        ops.launch_shard_candidates(args, gathered[r], x.device)
        keep.append(args)
    sel, args = prepare_singular(x[:, :shard], world_size=world, local_rank=0, shard_size=shard, **kw)
    args.vocab_size = shard * world
    ops.launch_merge_candidates(args, gathered, world, x.device)
    torch.cuda.synchronize()
    return sel


def _assert_same(sel, ref, z):
    assert torch.equal(sel.tokens.cpu(), ref.tokens.cpu())
    stoch = torch.ones(sel.tokens.size(0), dtype=torch.bool)
    a, b = sel.logprobs.selected.cpu(), ref.logprobs.selected.cpu()
    assert torch.equal(torch.isnan(a), torch.isnan(b))
    assert torch.equal(a.view(torch.int32)[~torch.isnan(a)], b.view(torch.int32)[~torch.isnan(b)])
    assert torch.equal(sel.logprobs.top_k.tokens.cpu()[stoch, :z], ref.logprobs.top_k.tokens.cpu()[stoch, :z])


@pytest.mark.parametrize("world,vocab", [(2, 32000), (4, 32000), (2, 128256), (8, 128256)])
def test_emulated_vocab_shards_match_unsharded(dev, world, vocab):
    from sonic_sampler_b200.interface.functional.singular import fused_singular

    rows = 24
    x, b = _case(dev, rows, vocab, seed=vocab + world)
    kw = _kwargs(b)
    ref = fused_singular(x, **kw)
    sel = _emulated_sharded(x, kw, world, vocab // world)
    _assert_same(sel, ref, 8)


def test_emulated_vocab_shards_greedy_lowest_index(dev):
    """Greedy rows take the largest value with the lowest global column: the unsharded rule with
    one tile (block_n >= V) is the same rule."""
    from sonic_sampler_b200.interface.functional.singular import fused_singular

    x, b = _case(dev, 16, 32000, seed=77, greedy_every=2)
    # plant cross-shard ties: the same top value in shard 0 and shard 1, on columns that no
    # processor changes differently (allowed by the grammar, no bias, no counts)
    tie = [100, 16000 + 5]
    x[:, tie] = 40.0
    b.grammar.view(torch.int32).fill_(-1)
    b.bias[:, tie] = 0
    b.repetition.counts.context[:, tie] = 0
    b.repetition.counts.decode[:, tie] = 0
    kw = _kwargs(b)
    ref = fused_singular(x, block_n=65536, **kw)
    sel = _emulated_sharded(x, kw, 2, 16000)
    assert torch.equal(sel.tokens.cpu(), ref.tokens.cpu())
    greedy = (b.flags.target.cpu().to(torch.int32) & 0x40) != 0
    assert (sel.tokens.cpu().view(-1)[greedy] == 100).all()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from sonic_sampler_b200.interface.functional.singular import fused_singular

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    vocab = 128256
    x, b = _case(dev, 32, vocab, seed=5)  # identical inputs on every rank (same seeds)
    kw = _kwargs(b)
    ref = fused_singular(x, **kw)
    shard = vocab // world
    sel = fused_singular(x[:, rank * shard:(rank + 1) * shard].contiguous(), world_size=world, local_rank=rank,
                         shard_size=shard, **kw)
    torch.cuda.synchronize()
    ok = torch.equal(sel.tokens, ref.tokens) and torch.equal(sel.logprobs.selected, ref.logprobs.selected)
    out.put((rank, bool(ok)))
    dist.barrier()
    dist.destroy_process_group()


def test_nccl_vocab_shards_match_unsharded(dev):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    assert sorted(out.get(timeout=5) for _ in range(world)) == [(0, True), (1, True)]


@pytest.mark.parametrize("world", [2, 4])
def test_emulated_logits_only_shards_match_unsharded_and_oracle(dev, world):
    """Logits-only rows (config 5's processing: top-k 64, top-p 0.95, Philox noise) take the
    logits-only kernel for the shard candidates. The merged selection equals the unsharded GPU
    path and the CPU oracle's unsharded selection. (Greedy rows are left to the one-tile test
    above: at V = 256000 the unsharded path's tile tie rule and the sharded lowest-column rule
    may pick different tied columns.)"""
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.singular import fused_singular, prepare_singular

    rows, vocab = 64, 256000
    c = workloads.config5(dev, seed=41, batch=rows, vocab=vocab)
    ind = c["indicators"].to(torch.int32)
    kw = dict(indicators=ind.to(torch.uint16), top_k=c["top_k"], top_p=c["top_p"], philox_seed=c["philox_seed"],
              philox_offset=5, return_logprobs=True, logprobs_dtype=F32, block_n=4096)
    ref = fused_singular(c["logits"], **kw)
    sel = _emulated_sharded(c["logits"], kw, world, vocab // world)
    assert torch.equal(sel.tokens.cpu(), ref.tokens.cpu())
    assert torch.equal(sel.logprobs.selected.cpu().view(torch.int32), ref.logprobs.selected.cpu().view(torch.int32))
    hk = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
    host, args = prepare_singular(c["logits"].cpu(), **hk)
    oracle.fused_singular(args)
    assert torch.equal(sel.tokens.cpu(), host.tokens)
