"""CUDA path against the CPU oracle at the benchmark configs' full sizes and on the edge
cases of the domain. Integer outputs (tokens, offsets, counts, candidate ids) must match
bit for bit; logprobs and probabilities too, since the kernels and the oracle share one
fixed fp32 operation order (tests/test_oracle_golden.py pins that oracle to the reference
within 1e-5)."""

from __future__ import annotations

import math

import pytest
import torch

from sonic_sampler_b200 import workloads

pytestmark = pytest.mark.gpu

BF16, F32, I32 = torch.bfloat16, torch.float32, torch.int32


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from sonic_sampler_b200 import _abi

    _abi.load_library()
    return torch.device("cuda", 0)


def bits(t):
    t = t.detach().cpu()
    if t.dtype == BF16:
        return t.view(torch.int16)
    if t.dtype == F32:
        return t.view(torch.int32)
    return t


def host(d: dict) -> dict:
    return {k: (v.detach().cpu().clone() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def buffer_kwargs(b, timestep: int | None = 0, draft: bool = False) -> dict:
    """fused_singular / fused_multistep keywords from a SamplingBuffers object (as the
    modular interface passes them)."""
    g = b.weights.gumbel.draft if draft else b.weights.gumbel.target
    kw = dict(
        indicators=b.flags.draft if draft else b.flags.target,
        grammar=b.grammar if timestep is None else b.grammar[:, timestep],
        context_counts=b.repetition.counts.context, decode_counts=b.repetition.counts.decode,
        repetition_penalties=b.repetition.multiplicative, frequency_penalties=b.repetition.frequency,
        presence_penalties=b.repetition.presence, logit_bias=b.bias, temperature=b.temperature, top_k=b.top_k,
        top_p=b.top_p, min_p=b.min_p, top_k_logprobs=b.top_logprobs,
        gumbel_noise=g if timestep is None else g[:, timestep],
    )
    if timestep is None:  # multistep: acceptance uniforms come from the buffers too
        kw["uniform_noise"] = b.weights.uniform
    return kw


def run_singular(logits, **kw):
    """(gpu selection, oracle selection, gpu kwargs, host kwargs)."""
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.singular import fused_singular, prepare_singular

    kh = host(kw)
    sel = fused_singular(logits, **kw)
    ref, args = prepare_singular(logits.detach().cpu().clone(), **kh)
    oracle.fused_singular(args)
    torch.cuda.synchronize()
    return sel, ref, kw, kh


def assert_selection_equal(sel, ref, kw=None, kh=None):
    assert torch.equal(sel.tokens.cpu(), ref.tokens)
    if sel.logprobs is not None:
        stoch = ~(kh["indicators"].to(torch.int32) & 0x40).bool()
        sm = kh.get("slot_mapping")
        rows = sel.tokens.size(0)
        mask = stoch[sm.long()] if sm is not None else stoch[:rows]
        a, b = sel.logprobs.selected.cpu()[mask], ref.logprobs.selected[mask]
        nan = torch.isnan(a.float())
        assert torch.equal(nan, torch.isnan(b.float()))  # fully masked rows: NaN on both sides
        assert torch.equal(bits(a)[~nan], bits(b)[~nan])
    if kw is not None and kw.get("decode_counts") is not None:
        assert torch.equal(kw["decode_counts"].cpu(), kh["decode_counts"])
    if sel.probabilities is not None:
        assert torch.equal(bits(sel.probabilities), bits(ref.probabilities))


# ----------------------------------------------------------------------------------------
# config 2: the benchmark workload
# ----------------------------------------------------------------------------------------


@pytest.mark.parametrize("lp_dtype", [BF16, F32])
def test_config2_full(dev, lp_dtype):
    w = workloads.config2(dev, seed=5)
    kw = buffer_kwargs(w["buffers"])
    sel, ref, kw, kh = run_singular(w["logits"], block_n=4096, update_counts=True, return_logprobs=True,
                                    max_top_logprobs=5, logprobs_dtype=lp_dtype, **kw)
    assert_selection_equal(sel, ref, kw, kh)


def test_config2_modular_matches_functional(dev):
    from sonic_sampler_b200.interface import UnshardedFusedSingular

    w = workloads.config2(dev, seed=6)
    sampler = UnshardedFusedSingular.initialize(128256, batch_size=64)
    sel = sampler.autoregressive(w["logits"], w["buffers"], logprobs=True)
    kw = buffer_kwargs(w["buffers"])
    _, ref, _, _ = run_singular(w["logits"], block_n=sampler.block_n, return_logprobs=True, max_top_logprobs=5, **kw)
    assert torch.equal(sel.tokens.cpu(), ref.tokens)


def test_config2_repeat_pdl_graph(dev):
    """Workspace reuse, PDL on/off and CUDA-graph replay all give the same result."""
    from sonic_sampler_b200.interface import UnshardedFusedSingular

    w = workloads.config2(dev, seed=7)
    s1 = UnshardedFusedSingular.initialize(128256, batch_size=64, pdl=True)
    s2 = UnshardedFusedSingular.initialize(128256, batch_size=64, pdl=False)
    outs = [s1.autoregressive(w["logits"], w["buffers"], logprobs=True) for _ in range(3)]
    outs.append(s2.autoregressive(w["logits"], w["buffers"], logprobs=True))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gs = s1.autoregressive(w["logits"], w["buffers"], logprobs=True)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    outs.append(gs)
    for o in outs[1:]:
        assert torch.equal(o.tokens, outs[0].tokens)
        assert torch.equal(bits(o.logprobs.selected), bits(outs[0].logprobs.selected))


# ----------------------------------------------------------------------------------------
# config 3: stochastic multistep verification (varlen and fixed)
# ----------------------------------------------------------------------------------------


def run_multistep(logits, tokens, **kw):
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.multistep import fused_multistep, prepare_multistep

    kh = host(kw)
    ver = fused_multistep(logits, kw["indicators"], tokens, **{k: v for k, v in kw.items() if k != "indicators"})
    ref, args = prepare_multistep(logits.cpu().clone(), kh["indicators"], tokens.cpu().clone(),
                                  **{k: v for k, v in kh.items() if k != "indicators"})
    oracle.fused_multistep(args)
    torch.cuda.synchronize()
    assert torch.equal(ver.offsets.cpu(), ref.offsets)
    assert torch.equal(ver.tokens.cpu(), ref.tokens)
    if kw.get("decode_counts") is not None:
        assert torch.equal(kw["decode_counts"].cpu(), kh["decode_counts"])
    return ver, ref, kw, kh


def _verify_logprobs_equal(ver, ref, ind, slots, margins):
    sel, rsel = ver.logprobs.selected.reshape(-1), ref.logprobs.selected.reshape(-1)
    for b, s in enumerate(slots):
        if int(ind[s]) & 0x40:
            continue
        rows = slice(margins[b], margins[b] + int(ver.offsets[b]) + 1)
        assert torch.equal(bits(sel[rows]), bits(rsel[rows]))


@pytest.mark.parametrize("qdtype", [F32, BF16])
def test_config3_varlen(dev, qdtype):
    w = workloads.config3(dev, seed=8)
    b = w["buffers"]
    kw = buffer_kwargs(b, timestep=None)
    ver, ref, kw, kh = run_multistep(w["flat_logits"], w["flat_tokens"], cu_seqlens=w["cu_seqlens"],
                                     lookahead=w["gamma"], max_top_logprobs=20, update_counts=True,
                                     return_logprobs=True, draft_probabilities=w["probabilities"].to(qdtype),
                                     block_n=4096, **kw)
    cu = w["cu_seqlens"].cpu().tolist()
    _verify_logprobs_equal(ver, ref, kh["indicators"], list(range(32)), cu[:-1])
    assert int(ver.offsets.max()) >= 1  # some drafts accepted


def test_config3_fixed_modular(dev):
    from sonic_sampler_b200.interface import UnshardedFusedMultistep

    w = workloads.config3(dev, seed=9, varlen=False)
    b = w["buffers"]
    ms = UnshardedFusedMultistep.initialize(128256, lookahead=w["gamma"], batch_size=32, max_top_logprobs=20)
    ver = ms(w["logits"], w["tokens"], b, probabilities=w["probabilities"], logprobs=True)
    kw = buffer_kwargs(b, timestep=None)
    _, ref, _, _ = run_multistep(w["logits"], w["tokens"], lookahead=w["gamma"], max_top_logprobs=20,
                                 return_logprobs=True, draft_probabilities=w["probabilities"],
                                 block_n=ms.block_n, **kw)
    assert torch.equal(ver.tokens.cpu(), ref.tokens)
    assert torch.equal(ver.offsets.cpu(), ref.offsets)


# ----------------------------------------------------------------------------------------
# config 4: cross-vocab greedy drafting chain + greedy verification in one CUDA graph
# ----------------------------------------------------------------------------------------


def test_config4_graph_chain(dev):
    """The benchmark's chain (workloads.config4_chain: drafting steps write their tokens in
    place into the per-request table the verification reads) captured in one CUDA graph,
    against the oracle replaying the same steps on the host."""
    from oracle import oracle
    from sonic_sampler_b200.interface import UnshardedFusedMultistep, UnshardedFusedSingular
    from sonic_sampler_b200.interface.functional.multistep import prepare_multistep
    from sonic_sampler_b200.interface.functional.singular import prepare_singular

    w = workloads.config4(dev, seed=10)
    b, gamma, d2t, sm = w["buffers"], w["gamma"], w["d2t"], w["slot_mapping"]
    active = sm.numel()
    drafter = UnshardedFusedSingular.initialize(32000, batch_size=active, lookahead=gamma)
    verifier = UnshardedFusedMultistep.initialize(128256, lookahead=gamma, batch_size=active)
    tokens = torch.zeros(active, gamma + 1, dtype=I32, device=dev)

    g = torch.cuda.CUDAGraph()
    workloads.config4_chain(w, drafter, verifier, tokens)  # warm-up outside capture
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        ver = workloads.config4_chain(w, drafter, verifier, tokens)
    tokens.fill_(-5)
    g.replay()
    torch.cuda.synchronize()

    # oracle replay of the same chain on the host (no repetition penalties: the drafting
    # steps read no drafted tokens)
    hb = b.to("cpu")
    htok = torch.full((active, gamma + 1), -5, dtype=I32)  # entries no step writes keep their value
    hsm, hd2t = sm.cpu(), d2t.cpu()
    for t in range(gamma):
        kw = buffer_kwargs(hb, timestep=t, draft=True)
        ref, args = prepare_singular(w["draft_logits"][t].cpu(), lookahead=gamma, target_vocab=128256,
                                     block_n=drafter.tuning(active)[2], slot_mapping=hsm, d2t_mapping=hd2t, **kw)
        oracle.fused_singular(args)
        htok[:, t] = ref.tokens[:, 0]
    drafted = htok[:, :gamma].clone()
    kw = buffer_kwargs(hb, timestep=None)
    rver, args = prepare_multistep(w["target_logits"].cpu(), kw.pop("indicators"), htok, lookahead=gamma,
                                   block_n=verifier.block_n, slot_mapping=hsm, output_tokens=htok, **kw)
    oracle.fused_multistep(args)
    assert torch.equal(ver.offsets.cpu(), rver.offsets)
    assert torch.equal(ver.tokens.cpu(), rver.tokens)
    # the verified prefix of every request is its drafted tokens
    got = tokens.cpu()
    for i in range(active):
        n = int(rver.offsets[i])
        assert torch.equal(got[i, :n], drafted[i, :n])


# ----------------------------------------------------------------------------------------
# configs 1 and 5: bounded top-k and large-vocabulary Philox sampling
# ----------------------------------------------------------------------------------------


@pytest.mark.parametrize("dtype", [F32, BF16])
def test_config1_topk(dev, dtype):
    from oracle import oracle
    from sonic_sampler_b200 import ops
    from sonic_sampler_b200.interface import UnshardedBoundedTopK

    w = workloads.config1(dev, seed=0)
    x, k = w["logits"].to(dtype), w["k"]
    topk = UnshardedBoundedTopK.initialize(32000, batch_size=8, k=k).clear()
    values, indices = topk(x)
    torch.cuda.synchronize()
    vals = values.reshape(-1)[: 8 * k].view(8, k).cpu()
    idx = indices.reshape(-1)[: 8 * k].view(8, k).cpu()
    hv = torch.empty(8 * k, dtype=dtype)
    hi = torch.empty(8 * k, dtype=I32)
    oracle.bounded_topk(ops.topk_args(x.cpu(), vocab_size=32000, k=k, block_n=topk.block_n, values=hv, indices=hi))
    assert torch.equal(idx, hi.view(8, k))
    assert torch.equal(bits(vals), bits(hv.view(8, k)))
    tv, ti = torch.topk(x.cpu().float(), k, dim=-1)
    torch.testing.assert_close(vals.float(), tv, rtol=0, atol=0)


def test_config5_philox_full(dev):
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.singular import fused_singular, prepare_singular

    w = workloads.config5(dev, seed=1)
    x = w["logits"]
    kw = dict(indicators=w["indicators"], top_k=w["top_k"], top_p=w["top_p"], block_n=4096,
              philox_seed=w["philox_seed"], philox_offset=17, return_logprobs=True, logprobs_dtype=F32)
    sel = fused_singular(x, **kw)
    torch.cuda.synchronize()
    rows = torch.arange(0, 1024, 16)  # oracle on a row sample
    kh = host(kw)
    kh["slot_mapping"] = rows.to(I32)
    ref, args = prepare_singular(x[rows].cpu(), **kh)
    oracle.fused_singular(args)
    assert torch.equal(sel.tokens[rows].cpu(), ref.tokens)
    assert torch.equal(bits(sel.logprobs.selected[rows]), bits(ref.logprobs.selected))


def test_philox_chi_squared(dev):
    """Counter-based noise: the empirical token distribution over many offsets matches the
    truncated softmax (top-k 8) of the row."""
    from sonic_sampler_b200.interface.functional.singular import fused_singular

    vocab, draws = 4096, 4096
    g = torch.Generator().manual_seed(3)
    row = torch.full((vocab,), -30.0)
    row[torch.randperm(vocab, generator=g)[:8]] = torch.tensor([2.0, 1.5, 1.0, 0.5, 0.0, -0.5, -1.0, -1.5])
    x = row.to(BF16).to(dev).expand(draws, vocab).contiguous()
    ind = torch.full((draws,), 0x80, dtype=torch.uint16, device=dev)
    top_k = torch.full((draws,), 8, dtype=I32, device=dev)
    # one row per slot, distinct slots -> independent counters
    sel = fused_singular(x, ind, top_k=top_k, block_n=1024, philox_seed=1234, philox_offset=0)
    toks = sel.tokens.flatten().cpu()
    support = torch.topk(row, 8).indices
    assert bool(torch.isin(toks, support).all())
    p = torch.softmax(row.to(BF16).float()[support], 0)
    counts = torch.stack([(toks == t).sum() for t in support]).double()
    expected = p.double() * draws
    chi2 = float(((counts - expected) ** 2 / expected).sum())
    # chi-squared with 7 degrees of freedom: P(chi2 > 24.32) = 0.001
    assert chi2 < 24.32, (chi2, counts.tolist(), expected.tolist())


# ----------------------------------------------------------------------------------------
# edge cases
# ----------------------------------------------------------------------------------------


def _params(dev, slots, vocab, seed, **kw):
    b = workloads.sampling_buffers(slots, 1, vocab, dev, seed, workloads.config2_params(slots, seed + 1), **kw)
    return b


@pytest.mark.parametrize("vocab", [130, 1000, 32001, 70001])
def test_ragged_vocab_scalar_path(dev, vocab):
    """Vocab sizes that are not multiples of 8 (scalar loads, ragged last split)."""
    b = _params(dev, 6, vocab, seed=vocab, top_logprobs=3)
    x = workloads.peaked_logits(6, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=vocab)
    sel, ref, kw, kh = run_singular(x, block_n=256, update_counts=True, return_logprobs=True, max_top_logprobs=4,
                                    **buffer_kwargs(b))
    assert_selection_equal(sel, ref, kw, kh)


def test_misaligned_logits_view(dev):
    """A logits view starting one element in (not 16-byte aligned) takes the scalar path."""
    b = _params(dev, 8, 8191, seed=2)
    base = workloads.peaked_logits(8, 8192, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=2)
    x = base[:, 1:]
    sel, ref, kw, kh = run_singular(x, block_n=1024, return_logprobs=True, **buffer_kwargs(b))
    assert_selection_equal(sel, ref, kw, kh)


def test_fully_masked_rows(dev):
    """Rows whose grammar masks every token: every logit is -inf."""
    b = _params(dev, 4, 4096, seed=3, grammar_density=0.0)
    x = workloads.peaked_logits(4, 4096, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=3)
    sel, ref, kw, kh = run_singular(x, block_n=1024, return_logprobs=True, **buffer_kwargs(b))
    assert_selection_equal(sel, ref, kw, kh)


def test_greedy_tie_rule_per_block_n(dev):
    """Equal maxima at offset 100 of tile 0 and offset 5 of tile 1: the reference's tile rule
    picks the smaller in-tile offset, so the answer depends on block_n."""
    from sonic_sampler_b200.interface.functional.singular import fused_singular

    x = torch.zeros(2, 8192, dtype=BF16, device=dev)
    x[:, 100] = 9.0
    x[0, 1024 + 5] = 9.0
    x[1, 4096 + 5] = 9.0
    ind = torch.full((2,), 0x40, dtype=torch.uint16, device=dev)
    assert fused_singular(x, ind, block_n=1024).tokens.flatten().tolist() == [1029, 4101]
    assert fused_singular(x, ind, block_n=4096).tokens.flatten().tolist() == [100, 4101]


def test_slot_mapping_int64_d2t_int32(dev):
    vd, vt, slots = 5000, 9000, 12
    b = _params(dev, slots, vt, seed=4, top_logprobs=2)
    x = workloads.peaked_logits(7, vd, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=4)
    d2t = torch.randperm(vt, generator=torch.Generator().manual_seed(4))[:vd].to(I32).to(dev)
    sm = torch.tensor([11, 3, 0, 7, 5, 9, 1], dtype=torch.int64, device=dev)
    probs = torch.zeros(slots, vt, dtype=BF16, device=dev)
    kw = buffer_kwargs(b)
    sel, ref, kw, kh = run_singular(x, block_n=1024, slot_mapping=sm, d2t_mapping=d2t, target_vocab=vt,
                                    return_probabilities=True, draft_probabilities=probs, update_counts=True,
                                    is_prefill=True, **kw)
    assert_selection_equal(sel, ref, kw, kh)


def test_d2t_drafting_counts_drafted_tokens_by_target_id(dev):
    """A drafting step after the first (drafted tokens counted as decoded, ops/prologue.py:175-193)
    through a draft-to-target table: the drafted tokens are target ids and must be matched
    against each column's target id, on the fast path (stochastic rows) and the exact path
    (greedy rows). The drafted tokens are the target ids of each row's best draft columns, so
    the repetition penalties change which candidates survive. Tokens, logprobs and draft
    probabilities match the oracle bit for bit."""
    vd, vt, slots, gamma = 6000, 9000, 12, 3
    b = _params(dev, slots, vt, seed=5, top_logprobs=2)
    ind = b.flags.target.cpu().to(torch.int32)
    ind[::3] = (ind[::3] & 0x3F) | 0x40  # some greedy rows (exact path)
    b.flags.packed[:, 0] = ind.to(torch.uint16).to(dev)
    x = workloads.peaked_logits(7, vd, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=5)
    d2t = torch.randperm(vt, generator=torch.Generator().manual_seed(5))[:vd].to(I32).to(dev)
    sm = torch.tensor([11, 3, 0, 7, 5, 9, 1], dtype=torch.int64, device=dev)
    drafted = torch.zeros(slots, gamma, dtype=I32, device=dev)
    best = d2t[x.float().topk(gamma, dim=-1).indices]  # [7, gamma] target ids of the best columns
    drafted[sm] = best.to(I32)
    probs = torch.zeros(slots, vt, dtype=BF16, device=dev)
    kw = buffer_kwargs(b)
    sel, ref, kw, kh = run_singular(x, block_n=1024, slot_mapping=sm, d2t_mapping=d2t, target_vocab=vt,
                                    lookahead=gamma, drafted_tokens=drafted, return_probabilities=True,
                                    draft_probabilities=probs, return_logprobs=True, **kw)
    assert_selection_equal(sel, ref, kw, kh)


def test_top_logprobs_request_above_capacity_is_clamped(dev):
    b = _params(dev, 4, 4096, seed=5, top_logprobs=9)
    x = workloads.peaked_logits(4, 4096, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=5)
    sel, ref, kw, kh = run_singular(x, block_n=1024, return_logprobs=True, max_top_logprobs=4, **buffer_kwargs(b))
    assert torch.equal(sel.tokens.cpu(), ref.tokens)
    assert torch.equal(bits(sel.logprobs.top_k.logprobs), bits(ref.logprobs.top_k.logprobs))
    assert torch.equal(sel.logprobs.top_k.tokens.cpu(), ref.logprobs.top_k.tokens)


def test_large_batch_many_rows(dev):
    """More rows than SMs x resident CTAs (several waves, one split per row)."""
    b = _params(dev, 2048, 4096, seed=6)
    x = workloads.peaked_logits(2048, 4096, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=6)
    sel, ref, kw, kh = run_singular(x, block_n=1024, update_counts=True, **buffer_kwargs(b))
    assert_selection_equal(sel, ref, kw, kh)


def test_empty_batch_is_a_no_op(dev):
    from sonic_sampler_b200.interface.functional.singular import fused_singular

    x = torch.empty(0, 4096, dtype=BF16, device=dev)
    sel = fused_singular(x, torch.zeros(4, dtype=torch.uint16, device=dev),
                         gumbel_noise=torch.zeros(4, 4096, dtype=BF16, device=dev))
    assert sel.tokens.shape == (0, 1)


def test_multistep_greedy_mixed_bf16_logprobs(dev):
    """Greedy and stochastic requests in one multistep batch, slot mapping, bf16 outputs."""
    gamma, vocab, batch, slots = 3, 32000, 6, 9
    b = workloads.sampling_buffers(slots, gamma + 1, vocab, dev, 12, workloads.config2_params(slots, 13),
                                   top_logprobs=3)
    ind = b.flags.target.cpu().to(torch.int32)
    ind[::3] = (ind[::3] & 0x3F) | 0x40
    b.flags.packed[:, 0] = ind.to(torch.uint16).to(dev)
    sm = torch.tensor([8, 0, 3, 4, 6, 1], dtype=I32, device=dev)
    x = workloads.peaked_logits(batch * (gamma + 1), vocab, sigma=3.0, peaks=4, lift=12.0, device=dev,
                                seed=14).view(batch, gamma + 1, vocab)
    tokens = x.float().argmax(-1).to(I32).contiguous()
    tokens[1, 2] = (tokens[1, 2] + 1) % vocab
    kw = buffer_kwargs(b, timestep=None)
    ver, ref, kw, kh = run_multistep(x, tokens, lookahead=gamma, block_n=2048, slot_mapping=sm,
                                     update_counts=True, return_logprobs=True, max_top_logprobs=3, **kw)
    margins = [i * (gamma + 1) for i in range(batch)]
    _verify_logprobs_equal(ver, ref, kh["indicators"], sm.cpu().tolist(), margins)


def test_multistep_ragged_vocab_long_lookahead(dev):
    """Multistep rows on the scalar path (vocabulary not a multiple of 8) with the longest
    lookahead: every step counts the drafted tokens before it."""
    gamma, vocab, batch = 15, 32001, 3
    b = workloads.sampling_buffers(batch, gamma + 1, vocab, dev, 21, workloads.config2_params(batch, 22),
                                   top_logprobs=2)
    x = workloads.peaked_logits(batch * (gamma + 1), vocab, sigma=3.0, peaks=4, lift=12.0, device=dev,
                                seed=23).view(batch, gamma + 1, vocab)
    tokens = x.float().argmax(-1).to(I32).contiguous()  # drafts the target likes: long accepts
    kw = buffer_kwargs(b, timestep=None)
    ver, ref, kw, kh = run_multistep(x, tokens, lookahead=gamma, block_n=4096, update_counts=True,
                                     return_logprobs=True, max_top_logprobs=2, **kw)
    _verify_logprobs_equal(ver, ref, kh["indicators"], list(range(batch)), [i * (gamma + 1) for i in range(batch)])


def test_multistep_varlen_single_row_requests(dev):
    """Varlen requests of one row (only the bonus token) next to full-length ones."""
    gamma, vocab, batch = 4, 128256, 6
    lengths = [1, 5, 1, 3, 5, 2]
    cu = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0)), dtype=I32)
    rows = int(cu[-1])
    b = workloads.sampling_buffers(batch, gamma + 1, vocab, dev, 31, workloads.config2_params(batch, 32))
    x = workloads.peaked_logits(rows, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=33)
    tokens = torch.randint(0, vocab, (rows,), generator=torch.Generator().manual_seed(34)).to(I32).to(dev)
    kw = buffer_kwargs(b, timestep=None)
    ver, ref, kw, kh = run_multistep(x, tokens, cu_seqlens=cu.to(dev), lookahead=gamma, block_n=4096,
                                     update_counts=True, return_logprobs=True, **kw)
    _verify_logprobs_equal(ver, ref, kh["indicators"], list(range(batch)), cu[:-1].tolist())


@pytest.mark.parametrize("vocab", [128256, 50001])
def test_plain_rows_no_processors(dev, vocab):
    """Calls without grammar, counts or bias take the logits-only kernel: greedy and stochastic
    rows, temperature, top-k / top-p / min-p, top-Z logprobs; aligned rows stream through the
    bulk-copy ring, an odd vocabulary through scalar loads."""
    rows = 40
    params = workloads.config2_params(rows, 61)
    ind = []
    for i in range(rows):
        from sonic_sampler_b200.core.flags import Indicator

        f = Indicator.from_params(temperature=params.temperature[i], top_k=1 if i % 5 == 0 else params.top_k[i],
                                  top_p=params.top_p[i], min_p=params.min_p[i], top_k_logprobs=6)
        ind.append(int(f))
    kw = dict(
        indicators=torch.tensor(ind, dtype=torch.int32).to(torch.uint16).to(dev),
        temperature=torch.tensor(params.temperature, dtype=BF16, device=dev),
        top_k=torch.tensor(params.top_k, dtype=I32, device=dev),
        top_p=torch.tensor(params.top_p, dtype=BF16, device=dev),
        min_p=torch.tensor(params.min_p, dtype=BF16, device=dev),
        top_k_logprobs=torch.full((rows,), 6, dtype=I32, device=dev),
        gumbel_noise=workloads.log_exponential((rows, vocab), dev, 62),
        return_logprobs=True, max_top_logprobs=6, logprobs_dtype=F32, block_n=4096,
    )
    x = workloads.peaked_logits(rows, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=63)
    sel, ref, kw, kh = run_singular(x, **kw)
    assert_selection_equal(sel, ref, kw, kh)


def _logits_only_multistep_kwargs(dev, batch, gamma, vocab, seed):
    """Per-request parameters without grammar, counts or bias: every third request greedy
    (with a temperature), the others stochastic with top-k / top-p / min-p and top-Z logprobs."""
    from sonic_sampler_b200.core.flags import Indicator

    params = workloads.config2_params(batch, seed)
    ind = []
    for i in range(batch):
        f = Indicator.from_params(temperature=params.temperature[i], top_k=1 if i % 3 == 0 else params.top_k[i],
                                  top_p=params.top_p[i], min_p=params.min_p[i], top_k_logprobs=4)
        ind.append(int(f))
    return dict(
        indicators=torch.tensor(ind, dtype=torch.int32).to(torch.uint16).to(dev),
        temperature=torch.tensor(params.temperature, dtype=BF16, device=dev),
        top_k=torch.tensor(params.top_k, dtype=I32, device=dev),
        top_p=torch.tensor(params.top_p, dtype=BF16, device=dev),
        min_p=torch.tensor(params.min_p, dtype=BF16, device=dev),
        top_k_logprobs=torch.full((batch,), 4, dtype=I32, device=dev),
        gumbel_noise=workloads.log_exponential((batch, gamma + 1, vocab), dev, seed + 1),
        uniform_noise=torch.rand(batch, gamma + 1, generator=torch.Generator().manual_seed(seed + 2))
        .clamp_(min=torch.finfo(BF16).tiny).to(BF16).to(dev),
    )


@pytest.mark.parametrize("batch,varlen", [(128, False), (7, True)], ids=["multiwave", "varlen"])
def test_multistep_logits_only(dev, batch, varlen):
    """Multistep calls without grammar, counts or bias stream their rows through the
    logits-only kernel (128 x 4 rows of 128256: a grid of several waves, one CTA per row;
    varlen: one wave, several splits a row). Greedy and stochastic requests, drafts the target
    partly accepts, a slot mapping; offsets, tokens and logprobs match the oracle bit for bit."""
    gamma, vocab = 3, 128256
    slots = batch + 5
    kw = _logits_only_multistep_kwargs(dev, slots, gamma, vocab, seed=90 + batch)
    sm = torch.randperm(slots, generator=torch.Generator().manual_seed(91))[:batch].to(I32).to(dev)
    if varlen:
        lengths = [1 + (i * 5) % (gamma + 1) for i in range(batch)]
        cu = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0)), dtype=I32)
        rows = int(cu[-1])
        x = workloads.peaked_logits(rows, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=92)
        tokens = x.float().argmax(-1).to(I32)
        tokens[1::4] = (tokens[1::4] + 7) % vocab  # some drafts the target rejects
        ver, ref, _, kh = run_multistep(x, tokens.contiguous(), cu_seqlens=cu.to(dev), lookahead=gamma,
                                        slot_mapping=sm, block_n=4096, return_logprobs=True, max_top_logprobs=4,
                                        **kw)
        margins = cu[:-1].tolist()
    else:
        x = workloads.peaked_logits(batch * (gamma + 1), vocab, sigma=3.0, peaks=4, lift=12.0, device=dev,
                                    seed=93).view(batch, gamma + 1, vocab)
        tokens = x.float().argmax(-1).to(I32)
        tokens[1::4, 1] = (tokens[1::4, 1] + 7) % vocab
        ver, ref, _, kh = run_multistep(x, tokens.contiguous(), lookahead=gamma, slot_mapping=sm, block_n=4096,
                                        return_logprobs=True, max_top_logprobs=4, **kw)
        margins = [i * (gamma + 1) for i in range(batch)]
    _verify_logprobs_equal(ver, ref, kh["indicators"], sm.cpu().tolist(), margins)
    assert int(ver.offsets.max()) >= 1


def test_multistep_logits_only_greedy_floor_edges(dev):
    """Greedy multistep rows on the logits-only kernel's floor test: ties made by the
    temperature, NaN logits, an all -inf row, two +inf values, a +-0 maximum, and a request
    without temperature."""
    gamma, vocab, batch = 1, 128256, 4
    rows = batch * (gamma + 1)
    x = workloads.peaked_logits(rows, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=95)
    g = torch.Generator().manual_seed(95)
    near = torch.randperm(vocab, generator=g)[:64]
    x[0, near] = (torch.full((64,), 20.0) + torch.arange(64) * 0.0625).to(BF16).to(dev)
    x[1, torch.randperm(vocab, generator=g)[:5]] = float("nan")
    x[2] = float("-inf")
    x[3, 777] = float("inf")
    x[3, 90001] = float("inf")
    x[4] = -x[4].abs() - 1.0
    x[4, 5000] = -0.0
    x[4, 70000] = 0.0
    ind = torch.tensor([0x60, 0x60, 0x60, 0x40], dtype=torch.int32).to(torch.uint16).to(dev)
    kw = dict(indicators=ind, temperature=torch.tensor([3.0, 0.9, 0.6, 1.0], dtype=BF16, device=dev),
              gumbel_noise=torch.zeros(batch, gamma + 1, vocab, dtype=BF16, device=dev),
              uniform_noise=torch.ones(batch, gamma + 1, dtype=BF16, device=dev))
    tokens = x.float().nan_to_num(nan=-1e30).argmax(-1).to(I32)
    run_multistep(x, tokens.contiguous(), lookahead=gamma, block_n=1024, **kw)


# ----------------------------------------------------------------------------------------
# rows that need fewer than 128 exact candidates (top-k below 128)
# ----------------------------------------------------------------------------------------

_KS = [2, 3, 7, 8, 9, 15, 16, 17, 31, 33, 63, 64, 65, 100, 127, 128]
_ZS = [0, 1, 5, 20]


def _small_k_case(dev, rows, vocab, seed, density):
    """Buffers whose rows cycle through top-k values around the per-warp cut boundaries (k = 8m,
    8m +- 1) and top-Z requests below and above k; logits on a coarse grid so that many values
    tie at the k-th place."""
    b = _params(dev, rows, vocab, seed=seed, grammar_density=density, top_logprobs=5)
    top_k = torch.tensor([_KS[i % len(_KS)] for i in range(rows)], dtype=I32)
    z = torch.tensor([_ZS[(i // len(_KS)) % len(_ZS)] for i in range(rows)], dtype=I32)
    ind = b.flags.target.cpu().to(torch.int32) & ~(0x40 | 0x80 | 0x400)
    ind |= torch.where((top_k > 1) & (top_k < 128), 0x80, 0).to(torch.int32)
    ind |= torch.where(z > 0, 0x400, 0).to(torch.int32)
    b.top_k.copy_(top_k.to(dev))
    b.top_logprobs.copy_(z.to(dev))
    b.flags.packed[:, 0] = ind.to(torch.uint16).to(dev)
    x = workloads.peaked_logits(rows, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=seed)
    x = (x.float() * 2).round().div(2).to(BF16)
    return x, b


def _assert_top_z_equal(sel, ref, kh, cap):
    """The first min(Z, cap) top logprobs and tokens of every row that asks for them (entries
    past Z are not written)."""
    z = kh["top_k_logprobs"].clamp(max=cap)
    want = (kh["indicators"].to(torch.int32) & 0x400) != 0
    a_lp, b_lp = bits(sel.logprobs.top_k.logprobs), bits(ref.logprobs.top_k.logprobs)
    a_tk, b_tk = sel.logprobs.top_k.tokens.cpu(), ref.logprobs.top_k.tokens
    for i in range(a_lp.size(0)):
        n = int(z[i]) if bool(want[i]) else 0
        assert torch.equal(a_lp[i, :n], b_lp[i, :n]), i
        assert torch.equal(a_tk[i, :n], b_tk[i, :n]), i


@pytest.mark.parametrize("density", [0.3, 0.002])
def test_small_top_k_rows(dev, density):
    """Rows with top-k < 128 keep only their first k candidates exact (the streaming cut comes
    from the k-th key). A sparse grammar leaves some splits with fewer than k allowed columns,
    which takes the -inf redo. Tokens, logprobs, top-Z (also Z > k) and counts must match."""
    x, b = _small_k_case(dev, 64, 128256, seed=71, density=density)
    sel, ref, kw, kh = run_singular(x, update_counts=True, return_logprobs=True, max_top_logprobs=20,
                                    logprobs_dtype=F32, **buffer_kwargs(b))
    assert_selection_equal(sel, ref, kw, kh)
    _assert_top_z_equal(sel, ref, kh, 20)


def test_small_top_k_rows_logits_only(dev):
    """The same rows through the logits-only kernel (no grammar, counts or bias)."""
    x, b = _small_k_case(dev, 64, 128256, seed=72, density=0.3)
    kw = buffer_kwargs(b)
    for key in ("grammar", "context_counts", "decode_counts", "logit_bias"):
        kw.pop(key)
    ind = kw["indicators"].cpu().to(torch.int32) & ~0x1f  # no grammar / penalty / bias bits
    kw["indicators"] = ind.to(torch.uint16).to(dev)
    sel, ref, kw, kh = run_singular(x, return_logprobs=True, max_top_logprobs=20, logprobs_dtype=F32, **kw)
    assert_selection_equal(sel, ref, kw, kh)
    _assert_top_z_equal(sel, ref, kh, 20)


@pytest.mark.parametrize("k", [1, 2, 8, 16, 64, 128])
def test_topk_small_k_with_ties(dev, k):
    from oracle import oracle
    from sonic_sampler_b200 import ops
    from sonic_sampler_b200.interface import UnshardedBoundedTopK

    rows, vocab = 8, 128256
    x = workloads.peaked_logits(rows, vocab, sigma=2.0, peaks=8, lift=10.0, device=dev, seed=k, dtype=F32)
    x = x.mul(2).round().div(2)
    topk = UnshardedBoundedTopK.initialize(vocab, batch_size=rows, k=k).clear()
    values, indices = topk(x)
    torch.cuda.synchronize()
    vals = values.reshape(-1)[: rows * k].view(rows, k).cpu()
    idx = indices.reshape(-1)[: rows * k].view(rows, k).cpu()
    hv = torch.empty(rows * k, dtype=F32)
    hi = torch.empty(rows * k, dtype=I32)
    oracle.bounded_topk(ops.topk_args(x.cpu(), vocab_size=vocab, k=k, block_n=topk.block_n, values=hv, indices=hi))
    assert torch.equal(idx, hi.view(rows, k))
    assert torch.equal(bits(vals), bits(hv.view(rows, k)))


# ----------------------------------------------------------------------------------------
# multistep with counter-based (Philox) noise
# ----------------------------------------------------------------------------------------


def test_multistep_philox_matches_oracle(dev):
    """Config-3 shapes with in-kernel acceptance uniforms and rejection noise: tokens,
    offsets, counts and logprobs equal the oracle's (which draws the same counters)."""
    w = workloads.config3(dev, seed=11)
    kw = buffer_kwargs(w["buffers"], timestep=None)
    kw.pop("gumbel_noise")
    kw.pop("uniform_noise")
    ver, ref, kw, kh = run_multistep(w["flat_logits"], w["flat_tokens"], cu_seqlens=w["cu_seqlens"],
                                     lookahead=w["gamma"], max_top_logprobs=20, update_counts=True,
                                     return_logprobs=True, draft_probabilities=w["probabilities"], block_n=4096,
                                     philox_seed=97, philox_offset=5, **kw)
    cu = w["cu_seqlens"].cpu().tolist()
    _verify_logprobs_equal(ver, ref, kh["indicators"], list(range(32)), cu[:-1])


def test_multistep_philox_residual_distribution(dev):
    """Every draft is rejected (its token is outside the row's candidates), so the token is
    drawn from the residual, here the target's top-8 softmax: the counts over many requests
    pass a chi-squared test, and every offset is 0."""
    from sonic_sampler_b200.interface.functional.multistep import fused_multistep

    requests, vocab = 4096, 4096
    g = torch.Generator().manual_seed(12)
    row = torch.full((vocab,), -30.0)
    support = torch.randperm(vocab, generator=g)[:8]
    row[support] = torch.tensor([2.0, 1.5, 1.0, 0.5, 0.0, -0.5, -1.0, -1.5])
    # gamma = 1: rows (step 0, bonus step) of every request; the drafted token is never a candidate
    logits = row.to(BF16).to(dev).expand(requests * 2, vocab).contiguous()
    outside = int(torch.topk(row, 200, largest=False).indices[0])
    drafted = torch.full((requests * 2,), outside, dtype=I32, device=dev)
    ind = torch.full((requests,), 0x80, dtype=torch.uint16, device=dev)
    top_k = torch.full((requests,), 8, dtype=I32, device=dev)
    ver = fused_multistep(logits, ind, drafted, lookahead=1, top_k=top_k, block_n=1024, philox_seed=4321)
    torch.cuda.synchronize()
    assert int(ver.offsets.abs().max()) == 0
    toks = ver.tokens.view(requests, 2)[:, 0].cpu()
    assert bool(torch.isin(toks, support).all())
    p = torch.softmax(row.to(BF16).float()[support], 0)
    counts = torch.stack([(toks == t).sum() for t in support]).double()
    expected = p.double() * requests
    chi2 = float(((counts - expected) ** 2 / expected).sum())
    assert chi2 < 24.32, (chi2, counts.tolist(), expected.tolist())  # 7 dof, P = 0.001


def test_greedy_temperature_floor_edges(dev):
    """Greedy rows whose only processor is a temperature take the tempered-value floor (and,
    on 4096-column splits, wide ring chunks): ties made by the division, NaN logits, an all
    -inf row, tied +inf values, a +-0 maximum and both temperature paths (divide, exact
    reciprocal) must match the oracle bit for bit."""
    V, rows = 128256, 8
    b = _params(dev, rows, V, seed=41, processors=False)
    x = workloads.peaked_logits(rows, V, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=41)
    g = torch.Generator().manual_seed(41)
    # row 1: many near-maximal values that collapse to one bf16 after dividing by 3
    near = torch.randperm(V, generator=g)[:64]
    x[1, near] = (torch.full((64,), 20.0) + torch.arange(64) * 0.0625).to(BF16).to(dev)
    # row 2: NaNs among the logits
    x[2, torch.randperm(V, generator=g)[:5]] = float("nan")
    # row 3: every logit -inf
    x[3] = float("-inf")
    # row 4: two +inf values in different tiles
    x[4, 777] = float("inf")
    x[4, 90001] = float("inf")
    # row 5: all negative but a -0.0 and a +0.0
    x[5] = -x[5].abs() - 1.0
    x[5, 5000] = -0.0
    x[5, 70000] = 0.0
    kw = buffer_kwargs(b)
    ind = torch.full((rows,), 0x60, dtype=torch.uint16)  # greedy + temperature
    ind[7] = 0x40  # greedy without temperature
    kw["indicators"] = ind.to(dev)
    temp = torch.tensor([0.7, 3.0, 0.9, 1.3, 0.6, 0.8, 0.5, 1.1], dtype=BF16)
    kw["temperature"] = temp.to(dev)
    sel, ref, kw, kh = run_singular(x, block_n=1024, **kw)
    assert_selection_equal(sel, ref, kw, kh)


def test_multiwave_logits_only_sub_splits(dev):
    """Logits-only grids of several waves stream each row in one CTA as sub-splits of 65536
    columns (V = 200003: four sub-splits, the last ragged). Mixed rows: stochastic with top-k /
    top-p / temperature and top-Z logprobs, greedy rows (the reference tile rule across
    sub-splits), and rows with fewer than 128 finite logits spread over the sub-splits (the
    redo that keeps -inf). Tokens and logprobs match the oracle bit for bit."""
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.singular import fused_singular, prepare_singular

    rows, vocab = 600, 200003
    x = workloads.peaked_logits(rows, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=77)
    g = torch.Generator(device=dev).manual_seed(78)
    sparse = torch.arange(2, rows, 7, device=dev)
    keep = torch.rand(sparse.numel(), vocab, generator=g, device=dev) < 50.0 / vocab
    x[sparse] = torch.where(keep, x[sparse], torch.full_like(x[sparse], float("-inf")))
    ind = torch.full((rows,), int(0x80 | 0x100 | 0x20 | 0x400), dtype=torch.int32)
    ind[::5] = 0x40 | 0x20  # greedy with temperature
    params = workloads.config2_params(rows, 79)
    kw = dict(indicators=ind.to(torch.uint16).to(dev),
              top_k=torch.tensor([k if k < 128 else 64 for k in params.top_k], dtype=I32, device=dev),
              top_p=torch.tensor(params.top_p, dtype=BF16, device=dev),
              temperature=torch.tensor(params.temperature, dtype=BF16, device=dev),
              top_k_logprobs=torch.full((rows,), 6, dtype=I32, device=dev), max_top_logprobs=6,
              gumbel_noise=workloads.log_exponential((rows, vocab), dev, 80), block_n=4096,
              return_logprobs=True, logprobs_dtype=F32)
    sel = fused_singular(x, **kw)
    torch.cuda.synchronize()
    sample = torch.cat([torch.arange(0, rows, 13), sparse[:20].cpu()]).unique()
    kh = host(kw)
    kh["slot_mapping"] = sample.to(I32)
    ref, args = prepare_singular(x[sample.to(dev)].cpu(), **kh)
    oracle.fused_singular(args)
    assert torch.equal(sel.tokens[sample].cpu(), ref.tokens)
    stoch = ~(ind[sample] & 0x40).bool()
    a, b = sel.logprobs.selected[sample].cpu()[stoch], ref.logprobs.selected[stoch]
    assert torch.equal(torch.isnan(a), torch.isnan(b))
    assert torch.equal(bits(a)[~torch.isnan(a)], bits(b)[~torch.isnan(b)])
    assert torch.equal(sel.logprobs.top_k.tokens[sample].cpu()[stoch], ref.logprobs.top_k.tokens[stoch])


def test_multiwave_general_kernel_one_cta_per_row(dev):
    """Calls with every processor whose grid would take several waves stream each row in one
    CTA of the general kernel (320 rows of V = 200003: one CTA covers all 98 chunks, its
    warps' keys carry warp-local column indices and meet only as 64-bit keys with global
    columns). Mixed greedy and stochastic rows with top-k / top-p / min-p, counts, bias,
    grammar and logprobs; a sample of rows matches the oracle bit for bit."""
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.singular import fused_singular, prepare_singular

    rows, vocab = 320, 200003
    b = _params(dev, rows, vocab, seed=81, top_logprobs=4)
    ind = b.flags.target.cpu().to(torch.int32)
    ind[::7] = (ind[::7] & 0x3F) | 0x40  # some greedy rows
    b.flags.packed[:, 0] = ind.to(torch.uint16).to(dev)
    x = workloads.peaked_logits(rows, vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=82)
    kw = buffer_kwargs(b)
    kw.update(return_logprobs=True, max_top_logprobs=4, logprobs_dtype=F32, block_n=4096)
    sel = fused_singular(x, **kw)
    torch.cuda.synchronize()
    sample = torch.arange(0, rows, 11)
    kh = host(kw)
    kh["slot_mapping"] = sample.to(I32)
    ref, args = prepare_singular(x[sample.to(dev)].cpu(), **kh)
    oracle.fused_singular(args)
    assert torch.equal(sel.tokens[sample].cpu(), ref.tokens)
    stoch = ~(ind[sample] & 0x40).bool()
    a, r = sel.logprobs.selected[sample].cpu()[stoch], ref.logprobs.selected[stoch]
    assert torch.equal(torch.isnan(a), torch.isnan(r))
    assert torch.equal(bits(a)[~torch.isnan(a)], bits(r)[~torch.isnan(r)])
    assert torch.equal(sel.logprobs.top_k.tokens[sample].cpu()[stoch], ref.logprobs.top_k.tokens[stoch])


def test_multiwave_multistep_rows_one_cta_per_row(dev):
    """A multistep call with every processor and 128 requests x 5 rows (a grid of several
    waves: one CTA per row of the general kernel in multistep mode), stochastic and greedy
    requests with draft probabilities: offsets, tokens, counts and logprobs match the oracle."""
    gamma, vocab, batch = 4, 128256, 128
    b = workloads.sampling_buffers(batch, gamma + 1, vocab, dev, 83, workloads.config2_params(batch, 84),
                                   top_logprobs=3)
    ind = b.flags.target.cpu().to(torch.int32)
    ind[::5] = (ind[::5] & 0x3F) | 0x40
    b.flags.packed[:, 0] = ind.to(torch.uint16).to(dev)
    x = workloads.peaked_logits(batch * (gamma + 1), vocab, sigma=3.0, peaks=4, lift=12.0, device=dev,
                                seed=85).view(batch, gamma + 1, vocab)
    tokens = x.float().argmax(-1).to(I32)
    tokens[1::3, 2] = (tokens[1::3, 2] + 3) % vocab
    q = torch.softmax(x[:, :gamma].float(), -1).contiguous()
    kw = buffer_kwargs(b, timestep=None)
    ver, ref, kw, kh = run_multistep(x, tokens.contiguous(), lookahead=gamma, block_n=4096, update_counts=True,
                                     return_logprobs=True, max_top_logprobs=3, draft_probabilities=q, **kw)
    _verify_logprobs_equal(ver, ref, kh["indicators"], list(range(batch)), [i * (gamma + 1) for i in range(batch)])
