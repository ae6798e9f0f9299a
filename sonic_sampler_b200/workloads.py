"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs
There is no public dataset for this path; these stand in for real
LM-head outputs and request parameters.

Every generator builds on the given device with its own seeded generator, and returns
plain tensors in the reference's SamplingBuffers dtypes.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from sonic_sampler_b200.core.buffers import (
    Flags,
    GumbelNoise,
    RepetitionPenalties,
    SamplingBuffers,
    StochasticWeights,
    TokenCounts,
)
from sonic_sampler_b200.core.flags import MAX_K, Indicator

BF16 = torch.bfloat16
F32 = torch.float32
I32 = torch.int32


def _gen(device, seed: int) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def peaked_logits(rows: int, vocab: int, *, sigma: float, peaks: int, lift: float, device, seed: int,
                  dtype=BF16) -> Tensor:
    """N(0, sigma^2) rows plus `peaks` uniformly chosen tokens lifted by `lift`."""
    g = _gen(device, seed)
    x = torch.randn(rows, vocab, generator=g, device=device) * sigma
    pos = torch.rand(rows, vocab, generator=g, device=device).argsort(dim=-1)[:, :peaks]
    x.scatter_add_(1, pos, torch.full((rows, peaks), lift, device=device))
    return x.to(dtype)


def log_exponential(shape, device, seed: int) -> Tensor:
    """bf16 log(Exp(1)) noise from an fp32 uniform draw: log(-log u)."""
    u = torch.rand(shape, generator=_gen(device, seed), device=device).clamp_(min=torch.finfo(F32).tiny)
    return torch.log(-torch.log(u)).to(BF16)


def pack_bits(mask: Tensor) -> Tensor:
    """[..., V] bool -> [..., ceil(V/32)] uint32 words, bit i of word w = column 32w+i."""
    v = mask.size(-1)
    words = (v + 31) // 32
    pad = words * 32 - v
    m = torch.nn.functional.pad(mask.to(torch.int64), (0, pad)).view(*mask.shape[:-1], words, 32)
    w = (m << torch.arange(32, device=mask.device)).sum(-1)
    return (w - (w >= 2**31).to(torch.int64) * 2**32).to(torch.int32).view(torch.uint32)


@dataclass
class RequestParams:
    """Per-request sampling parameters of config 2 (reused by configs 3 and 5)."""

    temperature: list[float]
    top_k: list[int]
    top_p: list[float]
    min_p: list[float]


def config2_params(batch: int, seed: int) -> RequestParams:
    g = torch.Generator().manual_seed(seed)
    temperature = (torch.rand(batch, generator=g) + 0.5).tolist()            # U[0.5, 1.5]
    top_k = [(MAX_K, 20, 50)[int(i)] for i in torch.randint(0, 3, (batch,), generator=g)]  # 0 = off
    top_p = (0.8 + 0.2 * torch.rand(batch, generator=g)).tolist()            # U[0.8, 1.0]
    min_p = [(0.0, 0.05)[int(i)] for i in torch.randint(0, 2, (batch,), generator=g)]
    return RequestParams(temperature, top_k, top_p, min_p)


def sampling_buffers(slots: int, timesteps: int, vocab: int, device, seed: int, params: RequestParams, *,
                     history: int = 512, bias_tokens: int = 16, grammar_density: float = 0.3,
                     processors: bool = True, top_logprobs: int = 0, greedy: bool = False,
                     greedy_draft: bool = False) -> SamplingBuffers:
    """SamplingBuffers holding config-2 style parameters for every slot.

    Repetition: penalties 1.1 / 0.2 / 0.3 over a `history`-token history drawn uniformly from
    the vocabulary; both `counts.context` and `counts.decode` hold that history's histogram.
    Bias: `bias_tokens` random tokens with U[-5, 5]. Grammar: each bit set with probability
    `grammar_density`. Noise: bf16 log(Exp(1)) from fp32 uniforms.
    """
    dev = torch.device(device)
    g = _gen(dev, seed)
    hist = torch.randint(0, vocab, (slots, history), generator=g, device=dev)
    counts = torch.zeros(slots, vocab, dtype=I32, device=dev)
    counts.scatter_add_(1, hist, torch.ones_like(hist, dtype=I32))
    bias = torch.zeros(slots, vocab, dtype=BF16, device=dev)
    cols = torch.rand(slots, vocab, generator=g, device=dev).argsort(dim=-1)[:, :bias_tokens]
    bias.scatter_(1, cols, (torch.rand(slots, bias_tokens, generator=g, device=dev) * 10 - 5).to(BF16))
    grammar = pack_bits(torch.rand(slots, timesteps, vocab, generator=g, device=dev) < grammar_density)
    gumbel = log_exponential((2, slots, timesteps, vocab), dev, seed + 1)
    uniform = torch.rand(slots, timesteps, generator=g, device=dev).clamp_(min=torch.finfo(BF16).tiny).to(BF16)

    rep, freq, pres = (1.1, 0.2, 0.3) if processors else (1.0, 0.0, 0.0)
    target, draft = [], []
    for i in range(slots):
        j = i % len(params.temperature)
        ind = Indicator.from_params(
            grammar=processors, multiplicative=rep, frequency=freq, presence=pres, logit_bias=processors,
            temperature=params.temperature[j], top_k=1 if greedy else params.top_k[j], top_p=params.top_p[j],
            min_p=params.min_p[j], top_k_logprobs=top_logprobs, greedy_draft=greedy_draft,
        )
        target.append(int(ind))
        draft.append(int(ind.greedy()) if greedy_draft or greedy else int(ind.disable(Indicator.TOP_K_LOGPROBS)))
    rep_t = torch.full((slots,), rep, dtype=BF16, device=dev)
    return SamplingBuffers(
        grammar=grammar,
        repetition=RepetitionPenalties(counts=TokenCounts(context=counts, decode=counts.clone()),
                                       frequency=torch.full((slots,), freq, dtype=BF16, device=dev),
                                       presence=torch.full((slots,), pres, dtype=BF16, device=dev),
                                       multiplicative=rep_t),
        bias=bias,
        temperature=torch.tensor([params.temperature[i % len(params.temperature)] for i in range(slots)],
                                 dtype=BF16, device=dev),
        top_k=torch.tensor([params.top_k[i % len(params.top_k)] for i in range(slots)], dtype=I32, device=dev),
        top_p=torch.tensor([params.top_p[i % len(params.top_p)] for i in range(slots)], dtype=BF16, device=dev),
        min_p=torch.tensor([params.min_p[i % len(params.min_p)] for i in range(slots)], dtype=BF16, device=dev),
        top_logprobs=torch.full((slots,), top_logprobs, dtype=I32, device=dev),
        weights=StochasticWeights(uniform=uniform, gumbel=GumbelNoise(target=gumbel[0], draft=gumbel[1])),
        flags=Flags.from_values(target, draft, device=dev),
    )


# ------------------------------------------------------------------------------------------
# configs
# ------------------------------------------------------------------------------------------


def config1(device, seed: int = 0):
    """UnshardedBoundedTopK: B=8, V=32000, fp32 N(0, 2^2) + 8 peaks +10, k=32."""
    x = peaked_logits(8, 32000, sigma=2.0, peaks=8, lift=10.0, device=device, seed=seed, dtype=F32)
    return dict(logits=x, k=32)


def config2(device, seed: int = 0, batch: int = 64, vocab: int = 128256):
    """UnshardedFusedSingular.autoregressive decode, all processors, heterogeneous params."""
    logits = peaked_logits(batch, vocab, sigma=3.0, peaks=4, lift=12.0, device=device, seed=seed)
    buffers = sampling_buffers(batch, 1, vocab, device, seed + 100, config2_params(batch, seed + 200))
    return dict(logits=logits, buffers=buffers)


def config3(device, seed: int = 0, batch: int = 32, gamma: int = 4, vocab: int = 128256, varlen: bool = True):
    """UnshardedFusedMultistep stochastic verification: target logits (B, gamma+1, V) like config 2,
    q = softmax(target[:, :gamma] + N(0, 0.5^2)), drafted ~ q, draft lengths U{1..gamma}."""
    dev = torch.device(device)
    g = _gen(dev, seed + 7)
    logits = peaked_logits(batch * (gamma + 1), vocab, sigma=3.0, peaks=4, lift=12.0, device=dev,
                           seed=seed).view(batch, gamma + 1, vocab)
    buffers = sampling_buffers(batch, gamma + 1, vocab, dev, seed + 100, config2_params(batch, seed + 200),
                               top_logprobs=20)
    q = torch.softmax(logits[:, :gamma].float() + torch.randn(batch, gamma, vocab, generator=g, device=dev) * 0.5,
                      dim=-1)
    drafted = torch.multinomial(q.view(-1, vocab), 1, generator=g).view(batch, gamma).to(I32)
    tokens = torch.cat([drafted, torch.zeros(batch, 1, dtype=I32, device=dev)], dim=1).contiguous()
    out = dict(logits=logits, tokens=tokens, buffers=buffers, probabilities=q, gamma=gamma)
    if varlen:
        lengths = torch.randint(1, gamma + 1, (batch,), generator=torch.Generator().manual_seed(seed + 9)) + 1
        cu = torch.zeros(batch + 1, dtype=I32)
        cu[1:] = lengths.cumsum(0)
        rows = torch.cat([torch.arange(int(lengths[b])) + b * (gamma + 1) for b in range(batch)])
        out.update(
            cu_seqlens=cu.to(dev),
            flat_logits=logits.reshape(-1, vocab)[rows.to(dev)].contiguous(),
            flat_tokens=tokens.reshape(-1)[rows.to(dev)].contiguous(),
        )
    return out


def config4(device, seed: int = 0, active: int = 128, slots: int = 256, gamma: int = 3, draft_vocab: int = 32000,
            target_vocab: int = 128256):
    """Eagle-3 style cross-vocab greedy drafting with slot indirection, then greedy verification."""
    dev = torch.device(device)
    g = torch.Generator().manual_seed(seed)
    d2t = torch.randperm(target_vocab, generator=g)[:draft_vocab].to(torch.int64).to(dev)
    slot_mapping = torch.randperm(slots, generator=g)[:active].to(I32).to(dev)
    draft_logits = [peaked_logits(active, draft_vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=seed + 10 + t)
                    for t in range(gamma)]
    target_logits = peaked_logits(active * (gamma + 1), target_vocab, sigma=3.0, peaks=4, lift=12.0, device=dev,
                                  seed=seed + 20).view(active, gamma + 1, target_vocab)
    buffers = sampling_buffers(slots, gamma + 1, target_vocab, dev, seed + 100, config2_params(slots, seed + 200),
                               processors=False, greedy=True)
    return dict(d2t=d2t, slot_mapping=slot_mapping, draft_logits=draft_logits, target_logits=target_logits,
                buffers=buffers, gamma=gamma)


def config4_chain(c: dict, drafter, verifier, tokens: torch.Tensor):
    """One config-4 chain: `gamma` greedy drafting steps, each writing its token in place into
    column t of the per-request table `tokens` (reference interface/singular.py:41-55 with
    in_place=True), then the verification, which reads the drafted tokens from that table and
    overwrites it with its outputs. Five launches, no glue between them. (A drafting step reads
    the drafted tokens per slot, for repetition penalties only; config 4 sets none, so a
    per-request table serves both calls.)"""
    b, d2t, sm = c["buffers"], c["d2t"], c["slot_mapping"]
    for t in range(c["gamma"]):
        drafter.drafting(c["draft_logits"][t], b, timestep=t, tokens=tokens, in_place=True, slot_mapping=sm,
                         d2t_mapping=d2t, target_vocab=128256)
    return verifier(c["target_logits"], tokens, b, slot_mapping=sm, in_place=True)


def config5(device, seed: int = 0, batch: int = 1024, vocab: int = 256000):
    """B=1024, V=256000: top_k=64 -> top_p=0.95 -> Gumbel-max with counter-based Philox (seed 1234)."""
    dev = torch.device(device)
    logits = peaked_logits(batch, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=seed)
    ind = int(Indicator.TOP_K | Indicator.TOP_P)
    return dict(
        logits=logits,
        indicators=torch.full((batch,), ind, dtype=torch.uint16, device=dev),
        top_k=torch.full((batch,), 64, dtype=I32, device=dev),
        top_p=torch.full((batch,), 0.95, dtype=BF16, device=dev),
        philox_seed=1234,
    )


def runner(name: str, device, pdl: bool = True):
    """A no-argument callable that runs benchmark config `name` once through the public
    interface (config 2: UnshardedFusedSingular.autoregressive; 3: fused_multistep; 4: three
    cross-vocabulary greedy drafting steps and a greedy verification, as one chain;
    5: fused_singular with Philox noise; 1: UnshardedBoundedTopK; indexed_copy: the noise
    staging of GumbelNoise.stage_weights; config4_verify[_logits_only]: config 4's verification
    step alone). `pdl` sets the programmatic-dependent-launch attribute of the sampler launches
    (the interface objects' `pdl`, the functional calls' `enable_pdl`)."""
    dev = torch.device(device)
    if name == "config1":
        from sonic_sampler_b200.interface import UnshardedBoundedTopK

        c = config1(dev)
        topk = UnshardedBoundedTopK.initialize(32000, batch_size=8, k=c["k"], pdl=pdl)
        return lambda: topk(c["logits"])
    if name == "config2":
        from sonic_sampler_b200.interface import UnshardedFusedSingular

        c = config2(dev, seed=1000)
        sampler = UnshardedFusedSingular.initialize(128256, batch_size=64, pdl=pdl)
        return lambda: sampler.autoregressive(c["logits"], c["buffers"], logprobs=True)
    if name == "config3":
        from sonic_sampler_b200.interface.functional.multistep import fused_multistep

        c = config3(dev, seed=8)
        b = c["buffers"]
        kw = dict(grammar=b.grammar, context_counts=b.repetition.counts.context,
                  decode_counts=b.repetition.counts.decode, repetition_penalties=b.repetition.multiplicative,
                  frequency_penalties=b.repetition.frequency, presence_penalties=b.repetition.presence,
                  logit_bias=b.bias, temperature=b.temperature, top_k=b.top_k, top_p=b.top_p, min_p=b.min_p,
                  top_k_logprobs=b.top_logprobs, gumbel_noise=b.weights.gumbel.target, uniform_noise=b.weights.uniform)
        return lambda: fused_multistep(c["flat_logits"], b.flags.target, c["flat_tokens"], cu_seqlens=c["cu_seqlens"],
                                       lookahead=c["gamma"], max_top_logprobs=20, return_logprobs=True,
                                       draft_probabilities=c["probabilities"], block_n=4096, enable_pdl=pdl, **kw)
    if name == "config4":
        from sonic_sampler_b200.interface import UnshardedFusedMultistep, UnshardedFusedSingular

        c = config4(dev, seed=10)
        active, gamma = c["slot_mapping"].numel(), c["gamma"]
        drafter = UnshardedFusedSingular.initialize(32000, batch_size=active, lookahead=gamma, pdl=pdl)
        verifier = UnshardedFusedMultistep.initialize(128256, lookahead=gamma, batch_size=active, pdl=pdl)
        tokens = torch.zeros(active, gamma + 1, dtype=I32, device=dev)
        return lambda: config4_chain(c, drafter, verifier, tokens)
    if name in ("config4_verify", "config4_verify_logits_only"):
        # the chain's verification step alone, on drafted tokens the target partly accepts:
        # through UnshardedFusedMultistep with the buffers (the rows kernel sees grammar, count
        # and bias buffers, so its rows take singular_kernel), or through fused_multistep with
        # the per-slot scalars only (the rows take the logits-only kernel)
        from sonic_sampler_b200.interface import UnshardedFusedMultistep
        from sonic_sampler_b200.interface.functional.multistep import fused_multistep

        c = config4(dev, seed=10)
        b, gamma, sm = c["buffers"], c["gamma"], c["slot_mapping"]
        active = sm.numel()
        verifier = UnshardedFusedMultistep.initialize(128256, lookahead=gamma, batch_size=active, pdl=pdl)
        tokens = c["target_logits"].float().argmax(-1).to(I32)
        tokens[1::3, 1] = (tokens[1::3, 1] + 1) % 128256
        if name == "config4_verify":
            return lambda: verifier(c["target_logits"], tokens, b, slot_mapping=sm)
        return lambda: fused_multistep(c["target_logits"], b.flags.target, tokens, slot_mapping=sm, lookahead=gamma,
                                       temperature=b.temperature, top_k=b.top_k, top_p=b.top_p, min_p=b.min_p,
                                       gumbel_noise=b.weights.gumbel.target, uniform_noise=b.weights.uniform,
                                       block_n=verifier.block_n, scratchpad=verifier.scratchpad, enable_pdl=pdl)
    if name == "config5":
        from sonic_sampler_b200.interface.functional.singular import fused_singular

        c = config5(dev, seed=1)
        kw = dict(indicators=c["indicators"], top_k=c["top_k"], top_p=c["top_p"], block_n=4096,
                  philox_seed=c["philox_seed"], philox_offset=17, return_logprobs=True, enable_pdl=pdl)
        return lambda: fused_singular(c["logits"], **kw)
    if name == "indexed_copy":
        from sonic_sampler_b200.core.buffers import GumbelNoise

        # noise staging after verification: 256 slots x 4 steps x V=128256 bf16 rows, 128 slots
        # staged (every other one stochastic), 262.7 MB read + written
        g = _gen(dev, 3)
        draft = torch.randn(256, 4, 128256, generator=g, device=dev).to(BF16)
        noise = GumbelNoise(target=torch.zeros_like(draft), draft=draft)
        indices = torch.randperm(256, generator=torch.Generator().manual_seed(4))[:128].to(I32).to(dev)
        indicator = torch.zeros(256, dtype=torch.uint16, device=dev)
        return lambda: noise.stage_weights(indices, indicator)
    raise ValueError(f"unknown workload {name!r}")


def time_calls(fn, calls: int = 30, flush_bytes: int = 256 << 20) -> list[float]:
    """Microseconds of `calls` CUDA-graph replays of one captured `fn()`, each after an L2
    flush (a write of `flush_bytes`), timed with CUDA events on the replaying stream."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    flush = torch.empty(flush_bytes, dtype=torch.uint8, device="cuda")
    out = []
    for i in range(calls):
        flush.fill_(i & 0xFF)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        torch.cuda.synchronize()
        out.append(start.elapsed_time(end) * 1e3)
    return out


if __name__ == "__main__":
    # python -m sonic_sampler_b200.workloads <config> [calls]: run a config `calls` times on
    # cuda:0 (the target of the ncu commands that produced the profiles).
    # python -m sonic_sampler_b200.workloads <config> --time [--pdl off]: median and minimum
    # of 30 CUDA-graph replays, L2 flushed before each.
    import statistics
    import sys

    args = sys.argv[1:]
    pdl_on = not ("--pdl" in args and args[args.index("--pdl") + 1] == "off")
    fn = runner(args[0], "cuda", pdl=pdl_on)
    if "--time" in args:
        ts = time_calls(fn)
        print(f"{args[0]} pdl={'on' if pdl_on else 'off'}: median {statistics.median(ts):.1f} us, "
              f"min {min(ts):.1f} us over {len(ts)} graph replays")
    else:
        for _ in range(int(args[1]) if len(args) > 1 else 6):
            fn()
        torch.cuda.synchronize()
        print("ok", args[0])
