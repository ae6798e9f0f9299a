"""CUDA path against the reference's own Triton kernels, run unmodified on the same B200 on
identical device inputs (tests/reference_gpu.py says where the reference comes from).

This pins parity to the reference as deployed: its libdevice fast exp/log and whatever
multiply-add contraction Triton applies on sm_100. The bar, per output:
- tokens, top-k indices, acceptance offsets, decode counts: bit for bit;
- logprobs: the reference writes bf16; our kernels run once more with fp32 logprobs, and the
  reference's bf16 value must be a round-to-nearest bf16 of some fp32 value within 1e-5 of
  ours (the 1e-5 fp32 tolerance, seen through the reference's bf16 output);
- multistep stage-2 probabilities (fp32): within 1e-5 absolute, candidate indices bit for bit.

Each test prints how many rows differ in any way, for the record.
"""

from __future__ import annotations

import pytest
import torch

from sonic_sampler_b200 import workloads

pytestmark = pytest.mark.gpu

BF16, F32, I32 = torch.bfloat16, torch.float32, torch.int32
TOL = 1e-5


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from tests import reference_gpu

    why = reference_gpu.unavailable()
    if why:
        pytest.skip(why)
    from sonic_sampler_b200 import _abi

    _abi.load_library()
    torch.cuda.set_device(0)
    return reference_gpu.load()


@pytest.fixture(scope="module")
def dev(ref):
    return torch.device("cuda", 0)


def lp_within(ref_bf16: torch.Tensor, ours_f32: torch.Tensor, tol: float = TOL) -> torch.Tensor:
    """Elementwise: is the reference's bf16 logprob RN_bf16(x) for some x within `tol` of ours?"""
    r = ref_bf16.float().cpu()
    o = ours_f32.float().cpu()
    lo = (o - tol).to(BF16).float()
    hi = (o + tol).to(BF16).float()
    ok = (r >= lo) & (r <= hi)
    return ok | (torch.isnan(r) & torch.isnan(o))


def report(name: str, **counts):
    print(f"[reference parity] {name}: " + ", ".join(f"{k}={v}" for k, v in counts.items()), flush=True)


def singular_kwargs(b, draft: bool = False, timestep: int = 0) -> dict:
    g = b.weights.gumbel.draft if draft else b.weights.gumbel.target
    return dict(
        indicators=b.flags.draft if draft else b.flags.target, grammar=b.grammar[:, timestep],
        context_counts=b.repetition.counts.context, decode_counts=b.repetition.counts.decode,
        repetition_penalties=b.repetition.multiplicative, frequency_penalties=b.repetition.frequency,
        presence_penalties=b.repetition.presence, logit_bias=b.bias, temperature=b.temperature, top_k=b.top_k,
        top_p=b.top_p, min_p=b.min_p, top_k_logprobs=b.top_logprobs, gumbel_noise=g[:, timestep],
    )


# ----------------------------------------------------------------------------------------
# config 1: UnshardedBoundedTopK (bf16, the reference's only logits dtype)
# ----------------------------------------------------------------------------------------


@pytest.mark.parametrize("k", [32, 128])
def test_config1_topk_matches_reference(ref, dev, k):
    from sonic_sampler_b200.interface import UnshardedBoundedTopK

    c = workloads.config1(dev)
    x = c["logits"].to(BF16)
    with torch.device(dev):
        theirs = ref.UnshardedBoundedTopK.initialize(32000, batch_size=8, k=k).clear()
    ours = UnshardedBoundedTopK.initialize(32000, batch_size=8, k=k).clear()
    tv, ti = theirs(x)
    ov, oi = ours(x)
    torch.cuda.synchronize()
    n = 8 * k  # both write row r's k results at flat offset r*k (reference quirk Q1)
    tv, ti = tv.reshape(-1)[:n].cpu(), ti.reshape(-1)[:n].cpu()
    ov, oi = ov.reshape(-1)[:n].cpu(), oi.reshape(-1)[:n].cpu()
    report(f"config1 k={k}", index_mismatch=int((ti != oi).sum()), value_mismatch=int((tv.view(torch.int16) != ov.view(torch.int16)).sum()))
    assert torch.equal(ti, oi)
    assert torch.equal(tv.view(torch.int16), ov.view(torch.int16))


# ----------------------------------------------------------------------------------------
# config 2: UnshardedFusedSingular.autoregressive, every processor, heterogeneous rows
# ----------------------------------------------------------------------------------------


def _config2_case(ref, dev, w, name: str, dropped_tail_ok: bool = False):
    """With `dropped_tail_ok`, a stochastic row's logprob may sit outside the tolerance only
    above ours: the reference then normalised over fewer candidates (it dropped trailing ones)."""
    from sonic_sampler_b200.interface import UnshardedFusedSingular
    from sonic_sampler_b200.interface.functional.singular import fused_singular

    logits = w["logits"]
    rows, vocab = logits.shape
    b_ref, b_ours, b_f32 = w["buffers"].to(dev), w["buffers"].to(dev), w["buffers"].to(dev)
    with torch.device(dev):
        theirs = ref.UnshardedFusedSingular.initialize(vocab, batch_size=rows)
    ours = UnshardedFusedSingular.initialize(vocab, batch_size=rows)
    assert ours.block_n == theirs.block_n  # same tile width: the greedy tie rule depends on it
    ts = theirs.autoregressive(logits, b_ref, update_counts=True, logprobs=True)
    os_ = ours.autoregressive(logits, b_ours, update_counts=True, logprobs=True)
    # our fp32 logprobs of the same call, for the tolerance check
    of = fused_singular(logits, **singular_kwargs(b_f32), block_n=ours.block_n, return_logprobs=True,
                        max_top_logprobs=ours.max_top_logprobs, logprobs_dtype=F32)
    torch.cuda.synchronize()

    stoch = ~(b_ref.flags.target.cpu().to(I32) & 0x40).bool()
    tok_bad = (ts.tokens.cpu() != os_.tokens.cpu()).view(-1)
    cnt_bad = (b_ref.repetition.counts.decode != b_ours.repetition.counts.decode).any(dim=1).cpu()
    lp_ok = lp_within(ts.logprobs.selected, of.logprobs.selected).view(-1)
    lp_bits = (ts.logprobs.selected.cpu().view(torch.int16) != os_.logprobs.selected.cpu().view(torch.int16)).view(-1)
    z = ours.max_top_logprobs
    zmask = torch.zeros(rows, z, dtype=torch.bool)
    for r in range(rows):
        ind = int(b_ref.flags.target[r])
        if stoch[r] and ind & 0x400:
            zmask[r, : min(int(b_ref.top_logprobs[r]), z)] = True
    ztok_bad = ((ts.logprobs.top_k.tokens.cpu() != os_.logprobs.top_k.tokens.cpu()) & zmask).any(dim=1)
    zlp_ok = (lp_within(ts.logprobs.top_k.logprobs, of.logprobs.top_k.logprobs) | ~zmask).all(dim=1)
    report(name, rows=rows, token_mismatch=int(tok_bad.sum()), count_rows_mismatch=int(cnt_bad.sum()),
           logprob_outside_1e5=int((~lp_ok & stoch).sum()), logprob_bf16_bits_differ=int((lp_bits & stoch).sum()),
           topz_token_mismatch=int(ztok_bad.sum()), topz_logprob_outside_1e5=int((~zlp_ok).sum()))
    assert not tok_bad.any(), tok_bad.nonzero().flatten().tolist()
    assert not cnt_bad.any()
    if dropped_tail_ok:
        off = ~lp_ok & stoch
        higher = ts.logprobs.selected.float().cpu().view(-1) > of.logprobs.selected.float().cpu().view(-1)
        report(name + " (rows where the reference dropped trailing candidates)", rows=int(off.sum()))
        assert bool(higher[off].all())
        assert not ztok_bad.any() and bool(zlp_ok[~off].all())
        return off
    assert bool(lp_ok[stoch].all())
    assert not ztok_bad.any() and bool(zlp_ok.all())


@pytest.mark.parametrize("seed", [5, 6])
def test_config2_matches_reference(ref, dev, seed):
    _config2_case(ref, dev, workloads.config2(dev, seed=seed), f"config2 seed={seed}")


def test_config2_mixed_greedy_matches_reference(ref, dev):
    """A third of the rows greedy (with every processor): the reference's greedy tile rule."""
    w = workloads.config2(dev, seed=11)
    b = w["buffers"]
    ind = b.flags.packed[:, 0].to(I32)
    ind[::3] |= 0x40
    b.flags.packed[:, 0] = ind.to(torch.uint16)
    b.flags.target_host = [int(v) for v in ind.tolist()]
    _config2_case(ref, dev, w, "config2 mixed greedy")


def test_config2_top_logprobs_matches_reference(ref, dev):
    """Rows asking for top-Z logprobs (indicator bit 0x400), Z = 5."""
    w = workloads.config2(dev, seed=12)
    b = w["buffers"]
    b.top_logprobs.fill_(5)
    ind = b.flags.packed[:, 0].to(I32) | 0x400
    b.flags.packed[:, 0] = ind.to(torch.uint16)
    b.flags.target_host = [int(v) for v in ind.tolist()]
    _config2_case(ref, dev, w, "config2 top-5 logprobs")


@pytest.mark.parametrize("variant", ["top_p_one", "top_p_one_no_min_p", "min_p_only"])
def test_config2_top_p_one_matches_reference(ref, dev, variant):
    """Every stochastic row with the TOP_P bit and top_p = 1.0 in bf16 (what a requested 0.999
    rounds to). Nucleus masking with p = 1 keeps every candidate that top-k and min-p leave: the
    reference's rule (ops/base.py:76-86) compares each prefix sum with the last one, and its
    prefix sums never decrease in exact or sequential arithmetic (its CPU path, its recorded
    vectors), nor in this restatement, which scales their maximum. On the GPU, Triton's parallel
    prefix sum can end an ulp below an earlier prefix and drop the last candidates of some rows.
    So tokens and counts must agree everywhere; a row's logprob may differ only where the
    reference normalised over fewer candidates (its logprob then lies above ours). The min-p
    variant shows the pivot itself agrees."""
    w = workloads.config2(dev, seed=15)
    b = w["buffers"]
    b.top_p.fill_(0.999)
    ind = b.flags.packed[:, 0].to(I32) | 0x100
    if variant == "top_p_one_no_min_p":
        ind &= ~0x200
    if variant == "min_p_only":
        ind = (ind & ~0x100) | 0x200
        b.min_p.fill_(0.05)
    b.flags.packed[:, 0] = ind.to(torch.uint16)
    b.flags.target_host = [int(v) for v in ind.tolist()]
    assert bool((b.top_p.float() == 1.0).all())
    off = _config2_case(ref, dev, w, f"config2 {variant}", dropped_tail_ok=(variant != "min_p_only"))
    if off is not None:
        assert int(off.sum()) <= 16  # a minority of rows (5 and 6 of 64 on a B200)


# ----------------------------------------------------------------------------------------
# config 3: fused_multistep, varlen stochastic verification with fp32 draft probabilities
# ----------------------------------------------------------------------------------------


def _multistep_kwargs(b) -> dict:
    return dict(
        grammar=b.grammar, context_counts=b.repetition.counts.context, decode_counts=b.repetition.counts.decode,
        repetition_penalties=b.repetition.multiplicative, frequency_penalties=b.repetition.frequency,
        presence_penalties=b.repetition.presence, logit_bias=b.bias, temperature=b.temperature, top_k=b.top_k,
        top_p=b.top_p, min_p=b.min_p, top_k_logprobs=b.top_logprobs, gumbel_noise=b.weights.gumbel.target,
        uniform_noise=b.weights.uniform,
    )


@pytest.mark.parametrize("varlen,q_dtype", [(True, BF16), (False, BF16)])
def test_config3_matches_reference(ref, dev, varlen, q_dtype):
    """Config 3 with bf16 draft probabilities: the reference's verification kernel does not
    compile with the fp32 ones config 3 specifies (test_reference_rejects_fp32_draft_probabilities);
    our fp32 path is pinned by the oracle tests instead."""
    from sonic_sampler_b200.interface.functional.multistep import fused_multistep

    c = workloads.config3(dev, seed=8, varlen=varlen)
    gamma, vocab = c["gamma"], 128256
    q = c["probabilities"].to(q_dtype)
    if varlen:
        logits, tokens, extra = c["flat_logits"], c["flat_tokens"], dict(cu_seqlens=c["cu_seqlens"])
    else:
        logits, tokens, extra = c["logits"], c["tokens"], {}
    rows = logits.reshape(-1, vocab).size(0)
    batch = c["tokens"].size(0)
    out = {}
    for who in ("theirs", "ours", "ours_f32"):
        b = c["buffers"].to(dev)
        vals = torch.zeros(rows, 128, dtype=F32, device=dev)
        idx = torch.full((rows, 128), -1, dtype=I32, device=dev)
        kw = dict(lookahead=gamma, max_top_logprobs=20, return_logprobs=True, update_counts=True,
                  draft_probabilities=q, block_n=4096, values=vals, indices=idx, **extra, **_multistep_kwargs(b))
        if who == "theirs":
            v = ref.fused_multistep(logits, b.flags.target, tokens.clone(), **kw)
        else:
            if who == "ours_f32":
                kw["logprobs_dtype"] = F32
            v = fused_multistep(logits, b.flags.target, tokens.clone(), **kw)
        out[who] = (v, vals, idx, b)
    torch.cuda.synchronize()
    (tv, tvals, tidx, tb), (ov, ovals, oidx, ob), (fv, _, _, _) = out["theirs"], out["ours"], out["ours_f32"]
    off_t, off_o = tv.offsets.cpu().view(-1), ov.offsets.cpu().view(-1)
    tok_bad = (tv.tokens.cpu() != ov.tokens.cpu())
    cnt_bad = (tb.repetition.counts.decode != ob.repetition.counts.decode).any(dim=1).cpu()
    # stage-2 buffers: fp32 probabilities within 1e-5, candidate ids exact (every row is stochastic)
    prob_bad = ((tvals - ovals).abs() > TOL).any(dim=1).cpu()
    idx_bad = (tidx != oidx).any(dim=1).cpu()
    # logprobs and top-20 only for steps <= accepted (reference quirk Q12)
    if varlen:
        cu = c["cu_seqlens"].cpu()
        pos = [(int(cu[b]) + s) for b in range(batch) for s in range(int(off_t[b]) + 1)]
        lp_t = tv.logprobs.selected.cpu()[pos]
        lp_f = fv.logprobs.selected.cpu()[pos]
        zt_t, zt_o = tv.logprobs.top_k.tokens.cpu()[pos], ov.logprobs.top_k.tokens.cpu()[pos]
        zl_t, zl_f = tv.logprobs.top_k.logprobs.cpu()[pos], fv.logprobs.top_k.logprobs.cpu()[pos]
    else:
        m = torch.arange(gamma + 1)[None, :] <= off_t[:, None]
        lp_t, lp_f = tv.logprobs.selected.cpu()[m], fv.logprobs.selected.cpu()[m]
        zt_t, zt_o = tv.logprobs.top_k.tokens.cpu()[m], ov.logprobs.top_k.tokens.cpu()[m]
        zl_t, zl_f = tv.logprobs.top_k.logprobs.cpu()[m], fv.logprobs.top_k.logprobs.cpu()[m]
    lp_ok = lp_within(lp_t, lp_f)
    zl_ok = lp_within(zl_t, zl_f)
    report(f"config3 varlen={varlen} q={q_dtype}", requests=batch, rows=rows,
           offset_mismatch=int((off_t != off_o).sum()), token_mismatch=int(tok_bad.sum()),
           count_rows_mismatch=int(cnt_bad.sum()), stage2_prob_rows_outside_1e5=int(prob_bad.sum()),
           stage2_index_rows_mismatch=int(idx_bad.sum()), logprob_outside_1e5=int((~lp_ok).sum()),
           topz_token_mismatch=int((zt_t != zt_o).sum()), topz_logprob_outside_1e5=int((~zl_ok).sum()),
           max_stage2_prob_diff=float((tvals - ovals).abs().max()))
    assert torch.equal(off_t, off_o)
    assert not tok_bad.any()
    assert not cnt_bad.any()
    assert not idx_bad.any()
    assert not prob_bad.any()
    assert bool(lp_ok.all()) and torch.equal(zt_t, zt_o) and bool(zl_ok.all())


def test_multistep_mixed_greedy_slots_matches_reference(ref, dev):
    """Config-3 shapes (fixed layout, bf16 draft probabilities) with every third request
    greedy and the requests mapped to slots by a permutation: greedy and stochastic
    verification side by side. Offsets, tokens and decode counts bit for bit; the stochastic
    requests' stage-2 candidate ids bit for bit and probabilities within 1e-5, their logprobs
    and top-20 within 1e-5 (neither implementation writes logprobs for greedy requests)."""
    from sonic_sampler_b200.interface.functional.multistep import fused_multistep

    c = workloads.config3(dev, seed=13, varlen=False)
    gamma, vocab = c["gamma"], 128256
    batch = c["tokens"].size(0)
    sm = torch.randperm(batch, generator=torch.Generator().manual_seed(14)).to(I32).to(dev)
    base = c["buffers"]
    ind = base.flags.packed[:, 0].to(I32)
    ind[::3] = (ind[::3] & 0x3F) | 0x40
    base.flags.packed[:, 0] = ind.to(torch.uint16)
    base.flags.target_host = [int(v) for v in ind.tolist()]
    q = c["probabilities"].to(BF16)
    rows = batch * (gamma + 1)
    out = {}
    for who in ("theirs", "ours", "ours_f32"):
        b = base.to(dev)
        vals = torch.zeros(rows, 128, dtype=F32, device=dev)
        idx = torch.full((rows, 128), -1, dtype=I32, device=dev)
        kw = dict(lookahead=gamma, max_top_logprobs=20, return_logprobs=True, update_counts=True,
                  draft_probabilities=q, block_n=4096, values=vals, indices=idx, slot_mapping=sm,
                  **_multistep_kwargs(b))
        if who == "theirs":
            v = ref.fused_multistep(c["logits"], b.flags.target, c["tokens"].clone(), **kw)
        else:
            if who == "ours_f32":
                kw["logprobs_dtype"] = F32
            v = fused_multistep(c["logits"], b.flags.target, c["tokens"].clone(), **kw)
        out[who] = (v, vals, idx, b)
    torch.cuda.synchronize()
    (tv, tvals, tidx, tb), (ov, ovals, oidx, ob), (fv, _, _, _) = out["theirs"], out["ours"], out["ours_f32"]
    off_t, off_o = tv.offsets.cpu().view(-1), ov.offsets.cpu().view(-1)
    greedy = (ind.cpu()[sm.long().cpu()] & 0x40).bool()  # per request
    stoch_rows = (~greedy).repeat_interleave(gamma + 1)
    tok_bad = (tv.tokens.cpu() != ov.tokens.cpu())
    cnt_bad = (tb.repetition.counts.decode != ob.repetition.counts.decode).any(dim=1).cpu()
    idx_bad = ((tidx != oidx).any(dim=1).cpu() & stoch_rows)
    prob_bad = (((tvals - ovals).abs() > TOL).any(dim=1).cpu() & stoch_rows)
    m = (torch.arange(gamma + 1)[None, :] <= off_t[:, None]) & ~greedy[:, None]
    lp_t, lp_f = tv.logprobs.selected.cpu()[m], fv.logprobs.selected.cpu()[m]
    zt_t, zt_o = tv.logprobs.top_k.tokens.cpu()[m], ov.logprobs.top_k.tokens.cpu()[m]
    zl_t, zl_f = tv.logprobs.top_k.logprobs.cpu()[m], fv.logprobs.top_k.logprobs.cpu()[m]
    lp_ok, zl_ok = lp_within(lp_t, lp_f), lp_within(zl_t, zl_f)
    report("multistep mixed greedy + slots", requests=batch, greedy_requests=int(greedy.sum()),
           offset_mismatch=int((off_t != off_o).sum()), token_mismatch=int(tok_bad.sum()),
           count_rows_mismatch=int(cnt_bad.sum()), stage2_index_rows_mismatch=int(idx_bad.sum()),
           stage2_prob_rows_outside_1e5=int(prob_bad.sum()), logprob_outside_1e5=int((~lp_ok).sum()),
           topz_token_mismatch=int((zt_t != zt_o).sum()), topz_logprob_outside_1e5=int((~zl_ok).sum()))
    assert int(greedy.sum()) > 0 and int((~greedy).sum()) > 0
    assert torch.equal(off_t, off_o)
    assert not tok_bad.any()
    assert not cnt_bad.any()
    assert not idx_bad.any() and not prob_bad.any()
    assert bool(lp_ok.all()) and torch.equal(zt_t, zt_o) and bool(zl_ok.all())


def test_reference_rejects_fp32_draft_probabilities(ref, dev):
    """The reference cannot verify with fp32 draft probabilities on the GPU: under Triton 3.6
    its `verify_drafted` (ops/verify.py:134-147) multiplies the bf16 uniforms by the fp32
    probabilities inside an `if`, and Triton refuses the type change when it compiles the
    kernel. Pinned here so the deviation record stays true."""
    import triton

    c = workloads.config3(dev, seed=8, varlen=False)
    b = c["buffers"].to(dev)
    with pytest.raises(triton.compiler.errors.CompilationError, match="verify_drafted"):
        ref.fused_multistep(c["logits"], b.flags.target, c["tokens"].clone(), lookahead=c["gamma"],
                            max_top_logprobs=20, return_logprobs=True, draft_probabilities=c["probabilities"],
                            block_n=4096, **_multistep_kwargs(b))


def test_reference_rejects_int64_d2t(ref, dev):
    """The reference cannot draft through an int64 d2t table on the GPU: its prologue
    (ops/prologue.py:382-386) reloads int32 column ids as the table's int64 entries inside an
    `if`, which Triton 3.6 refuses. Config 4 therefore compares against the reference with the
    same table as int32, while our side also runs the int64 table."""
    import triton

    c = workloads.config4(dev, seed=10)
    b = c["buffers"].to(dev)
    sm = c["slot_mapping"]
    with torch.device(dev):
        drafter = ref.UnshardedFusedSingular.initialize(32000, batch_size=sm.numel(), lookahead=c["gamma"])
    with pytest.raises(triton.compiler.errors.CompilationError, match="cols"):
        drafter.drafting(c["draft_logits"][0], b, timestep=0, slot_mapping=sm, d2t_mapping=c["d2t"],
                         target_vocab=128256)


# ----------------------------------------------------------------------------------------
# config 4: Eagle-3 cross-vocabulary greedy drafting with slot indirection + greedy verification
# ----------------------------------------------------------------------------------------


def test_config4_chain_matches_reference(ref, dev):
    from sonic_sampler_b200.interface import UnshardedFusedMultistep, UnshardedFusedSingular

    c = workloads.config4(dev, seed=10)
    gamma, d2t, sm = c["gamma"], c["d2t"], c["slot_mapping"]
    active = sm.numel()
    rows = sm.long()
    results = {}
    for who in ("theirs", "ours", "ours_i32"):
        b = c["buffers"].to(dev)
        # the reference needs the int32 table (test_reference_rejects_int64_d2t); ours runs both
        d2t = c["d2t"].to(I32) if who != "ours" else c["d2t"]
        if who == "theirs":
            with torch.device(dev):
                drafter = ref.UnshardedFusedSingular.initialize(32000, batch_size=active, lookahead=gamma)
                verifier = ref.UnshardedFusedMultistep.initialize(128256, lookahead=gamma, batch_size=active)
        else:
            drafter = UnshardedFusedSingular.initialize(32000, batch_size=active, lookahead=gamma)
            verifier = UnshardedFusedMultistep.initialize(128256, lookahead=gamma, batch_size=active)
        slot_tokens = torch.zeros(b.top_k.numel(), gamma + 1, dtype=I32, device=dev)
        drafted = []
        for t in range(gamma):
            sel = drafter.drafting(c["draft_logits"][t], b, timestep=t, tokens=slot_tokens if t else None,
                                   slot_mapping=sm, d2t_mapping=d2t, target_vocab=128256)
            slot_tokens[rows, t] = sel.tokens[:, 0]
            drafted.append(sel.tokens[:, 0].clone())
        tokens = slot_tokens[rows].contiguous()
        v = verifier(c["target_logits"], tokens, b, slot_mapping=sm, in_place=True)
        results[who] = (torch.stack(drafted).cpu(), v.tokens.cpu().clone(), v.offsets.cpu().clone())
    torch.cuda.synchronize()
    (td, tt, to), (od, ot, oo) = results["theirs"], results["ours"]
    report("config4 chain", requests=active, drafted_mismatch=int((td != od).sum()),
           verified_token_mismatch=int((tt != ot).sum()), offset_mismatch=int((to != oo).sum()))
    assert torch.equal(td, od)
    assert torch.equal(tt, ot)
    assert torch.equal(to, oo)
    for x, y in zip(results["ours"], results["ours_i32"]):
        assert torch.equal(x, y)


# ----------------------------------------------------------------------------------------
# stochastic drafting: UnshardedFusedSingular.drafting with the draft-probability output
# ----------------------------------------------------------------------------------------


@pytest.mark.parametrize("case", ["draft_vocab", "d2t_slots"])
def test_stochastic_drafting_matches_reference(ref, dev, case):
    """Two drafting steps of stochastic rows with every processor, through the modular
    `drafting` call of both implementations; the second step counts the first step's drafted
    tokens as decoded. `draft_vocab`: 64 slots drafting over their own 32000-token vocabulary.
    `d2t_slots`: 128 requests in 256 slots drafting over 32000 draft tokens mapped into a
    128256-token target vocabulary by an int32 table (the reference needs int32), the buffers
    and the probability output indexed by target id. Tokens must match bit for bit; the draft
    probabilities (bf16 in the reference) must be round-to-nearest bf16 values of our fp32
    probabilities within 1e-5."""
    from sonic_sampler_b200.interface import UnshardedFusedSingular

    gamma, draft_vocab = 3, 32000
    if case == "draft_vocab":
        slots, active, target_vocab = 64, 64, None
        sm, d2t = None, None
    else:
        slots, active, target_vocab = 256, 128, 128256
        g = torch.Generator().manual_seed(71)
        sm = torch.randperm(slots, generator=g)[:active].to(I32).to(dev)
        d2t = torch.randperm(target_vocab, generator=g)[:draft_vocab].to(I32).to(dev)
    bvocab = target_vocab or draft_vocab
    base = workloads.sampling_buffers(slots, gamma + 1, bvocab, dev, 72, workloads.config2_params(slots, 73))
    logits = [workloads.peaked_logits(active, draft_vocab, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=74 + t)
              for t in range(2)]
    rows = sm.long() if sm is not None else torch.arange(active, device=dev)
    out = {}
    for who, pdt in (("theirs", BF16), ("ours", BF16), ("ours_f32", F32)):
        b = base.to(dev)
        if who == "theirs":
            with torch.device(dev):
                drafter = ref.UnshardedFusedSingular.initialize(draft_vocab, batch_size=active, lookahead=gamma)
        else:
            drafter = UnshardedFusedSingular.initialize(draft_vocab, batch_size=active, lookahead=gamma)
        table = torch.zeros(slots, gamma + 1, dtype=I32, device=dev)  # drafted tokens per slot
        probs, toks = [], []
        for t in range(2):
            p = torch.zeros(slots, bvocab, dtype=pdt, device=dev)
            sel = drafter.drafting(logits[t], b, timestep=t, tokens=table if t else None, probabilities=p,
                                   slot_mapping=sm, d2t_mapping=d2t, target_vocab=target_vocab)
            table[rows, t] = sel.tokens[:, 0]
            toks.append(sel.tokens[:, 0].clone())
            probs.append(p)
        out[who] = (torch.stack(toks).cpu(), torch.stack(probs).cpu())
    torch.cuda.synchronize()
    (tt, tp), (ot, op), (_, fp) = out["theirs"], out["ours"], out["ours_f32"]
    ok = lp_within(tp, fp)
    report(f"stochastic drafting {case}", rows=active, token_mismatch=int((tt != ot).sum()),
           probability_outside_1e5=int((~ok).sum()),
           probability_bf16_bits_differ=int((tp.view(torch.int16) != op.view(torch.int16)).sum()),
           nonzero_probabilities=int((tp != 0).sum()))
    assert int((tp != 0).sum()) > 0
    assert torch.equal(tt, ot)
    assert bool(ok.all())


# ----------------------------------------------------------------------------------------
# noise staging: GumbelNoise.stage_weights (ops/copy.py indexed_copy)
# ----------------------------------------------------------------------------------------


@pytest.mark.parametrize("case", ["config_rows", "odd_rows_duplicates"])
def test_indexed_copy_matches_reference(ref, dev, case):
    """The draft noise of the indexed rows whose indicator lacks the greedy bit, copied into the
    target noise: 128 of 256 slots x 4 steps x 128256 bf16 (the bulk-copy ring), and rows of
    1001 values with repeated indices (the element-wise kernel). Bit for bit."""
    from sonic_sampler_b200.ops import indexed_copy

    g = torch.Generator().manual_seed(91)
    if case == "config_rows":
        shape, n = (256, 4, 128256), 128
        indices = torch.randperm(256, generator=g)[:n]
    else:
        shape, n = (40, 3, 1001), 30
        indices = torch.randint(0, 40, (n,), generator=g)
    source = torch.randn(*shape, generator=g).to(BF16).to(dev)
    indicator = torch.zeros(shape[0], dtype=torch.uint16)
    indicator[::2] = 0x40
    indicator = indicator.to(dev)
    idx = indices.to(I32).to(dev)
    theirs = torch.zeros_like(source)
    ours = torch.zeros_like(source)
    ref.indexed_copy(source, theirs, idx, indicator)
    indexed_copy(source, ours, idx, indicator)
    torch.cuda.synchronize()
    differ = int((theirs.view(torch.int16) != ours.view(torch.int16)).sum())
    report(f"indexed_copy {case}", rows=n, elements_differ=differ, rows_copied=int((ours != 0).flatten(1).any(1).sum()))
    assert differ == 0
    assert bool((ours != 0).any())


# ----------------------------------------------------------------------------------------
# slot population: SamplingBuffers.allocate / update at the full vocabulary
# ----------------------------------------------------------------------------------------


def _ref_state(b) -> dict:
    """The device-side fields of the reference's SamplingBuffers, cloned."""
    rep, w = b.repetition, b.weights
    plain = lambda t: torch.Tensor(t).as_subclass(torch.Tensor).clone()  # noqa: E731
    return dict(
        flags=plain(b.flags.packed), temperature=plain(b.temperature), top_p=plain(b.top_p), min_p=plain(b.min_p),
        top_k=plain(b.top_k), top_logprobs=plain(b.top_logprobs), multiplicative=plain(rep.multiplicative),
        frequency=plain(rep.frequency), presence=plain(rep.presence), context=plain(rep.counts.context),
        decode=plain(rep.counts.decode), bias=plain(b.bias), grammar=plain(b.grammar).view(torch.int32),
        gumbel_target=plain(w.gumbel.target), gumbel_draft=plain(w.gumbel.draft), uniform=plain(w.uniform),
    )


def test_population_matches_reference(ref, dev):
    """The reference's own SamplingBuffers (core/buffer.py) and ours, on the B200 at the full
    vocabulary (48 slots, 4 steps, V = 128256), starting from the same state and given the same
    admissions (prompts up to 1.5 V tokens, logit biases, bitmasks, greedy drafts) and updates
    (dense count rows), with CUDA generators seeded alike: every field, the noise included, bit
    for bit after each call (bias rows only where the BIAS bit is set: the reference copies its
    pinned mirror's stale contents for the others). Bitmasks go only with identity-prefix
    positions, where the reference's slot-indexed reading of them agrees with ours."""
    from sonic_sampler.core.buffer import SamplingBuffers as RefBuffers  # noqa: E402 (reference, on sys.path)
    from tests.test_populate import assert_state, buffers_from_state

    B, T, V = 48, 4, 128256
    W = (V + 31) // 32
    torch.manual_seed(17)
    theirs = RefBuffers.default(B, T, V, device=dev)
    ours = buffers_from_state(_ref_state(theirs), device=dev)
    g = torch.Generator().manual_seed(18)

    def params(n):
        return dict(
            multiplicative=[float(x) for x in (torch.rand(n, generator=g) * 0.6 + 0.7)],
            frequency=[float(x) for x in (torch.rand(n, generator=g) - 0.5)],
            presence=[float(x) for x in (torch.rand(n, generator=g) * 0.4)],
            temperature=[float(x) for x in (torch.rand(n, generator=g) + 0.4)],
            top_k=[(128, 20, 1, 64)[int(i)] for i in torch.randint(0, 4, (n,), generator=g)],
            top_p=[float(x) for x in (torch.rand(n, generator=g) * 0.3 + 0.7)],
            min_p=[(0.0, 0.05)[int(i)] for i in torch.randint(0, 2, (n,), generator=g)],
            top_logprobs=[int(i) for i in torch.randint(0, 6, (n,), generator=g)],
            biases=[None if j % 3 == 1 else {int(t): float(torch.randn(1, generator=g)) * 2
                                             for t in torch.randperm(V, generator=g)[: 2 + j % 16].tolist()}
                    for j in range(n)],
            greedy_drafts=[bool(j % 2) for j in range(n)],
        )

    def masks(n, full):
        out = []
        for j in range(n):
            rows = T if (full and j % 4 == 0) else 1
            m = torch.randint(-2**31, 2**31 - 1, (rows, W), generator=g, dtype=torch.int64).to(torch.int32)
            out.append(None if j % 2 else (m[0] if rows == 1 else m))
        return out

    plan = [("allocate", torch.randperm(B, generator=g)[:20].tolist(), False),
            ("allocate", list(range(12)), True),
            ("update", torch.randperm(B, generator=g)[:16].tolist(), False),
            ("update", None, True)]
    for k, (kind, positions, grammar) in enumerate(plan):
        n = len(positions) if positions else B
        kw = params(n)
        if grammar:
            kw["bitmasks"] = masks(n, full=(kind == "update"))
        if kind == "allocate":
            kw["encodings"] = [torch.randint(0, V, (int(torch.randint(1, 3 * V // 2, (1,), generator=g)),), generator=g)
                               for _ in range(n)]
        else:
            kw["counts"] = [(torch.randint(0, 9, (V,), generator=g, dtype=torch.int32),
                             torch.randint(0, 5, (V,), generator=g, dtype=torch.int32)) for _ in range(n)]
            kw["target_gumbel"] = [None] * n
        kw["positions"] = positions
        seed = 2000 + 17 * k
        getattr(theirs, kind)(generator=torch.Generator(dev).manual_seed(seed), **kw)
        getattr(ours, kind)(generator=torch.Generator(dev).manual_seed(seed), **kw)
        torch.cuda.synchronize()
        want = _ref_state(theirs)
        assert_state(ours, want, f"population call {k} ({kind})")
        report(f"population call {k} ({kind})", slots=n, fields_equal=1)

