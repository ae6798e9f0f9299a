"""The CPU oracle against golden vectors produced by the reference's own kernels
(tests/golden/make_golden.py). Bit-exact on tokens, indices, counts, offsets and top-k
values; fp32 logprobs within 1e-5 absolute; probabilities within 1e-5 relative."""

from __future__ import annotations

import pytest
import torch

from golden_cases import F32, LOGPROB_ATOL, load, singular_kwargs, slots_of, to
from sonic_sampler_b200 import ops
from sonic_sampler_b200.interface.functional.multistep import prepare_multistep
from sonic_sampler_b200.interface.functional.singular import prepare_singular


@pytest.mark.parametrize("k", [32, 128])
def test_topk_bf16(oracle_lib, k):
    case = load("topk_bf16")
    x = case["inputs"]["logits"]
    rows, vocab = x.shape
    values = torch.full((rows * k,), float("-inf"), dtype=torch.bfloat16)
    indices = torch.full((rows * k,), -1, dtype=torch.int32)
    oracle_lib.bounded_topk(ops.topk_args(x, vocab_size=vocab, k=k, block_n=1024, values=values, indices=indices))
    assert torch.equal(indices, case["outputs"][f"indices_k{k}"])
    assert torch.equal(values.view(torch.int16), case["outputs"][f"values_k{k}"].view(torch.int16))


def test_topk_bitonic_strategy(oracle_lib):
    case = load("topk_bitonic")
    x = case["inputs"]["logits"]
    rows, vocab = x.shape
    k = case["meta"]["k"]
    values = torch.empty(rows * k, dtype=torch.bfloat16)
    indices = torch.empty(rows * k, dtype=torch.int32)
    oracle_lib.bounded_topk(ops.topk_args(x, vocab_size=vocab, k=k, block_n=1024, values=values, indices=indices))
    assert torch.equal(indices, case["outputs"]["indices"])
    assert torch.equal(values.view(torch.int16), case["outputs"]["values"].view(torch.int16))


def _stochastic_rows(inputs, rows):
    ind = inputs["indicators"]
    return [r for r, s in enumerate(slots_of(inputs, rows)) if not (int(ind[s]) & 0x40)]


def test_singular_mixed(oracle_lib):
    case = load("singular_mixed")
    kw = singular_kwargs(case, "cpu")
    meta, out = case["meta"], case["outputs"]
    sel, args = prepare_singular(update_counts=True, return_logprobs=True, max_top_logprobs=meta["max_top_logprobs"],
                                 logprobs_dtype=F32, **kw)
    oracle_lib.fused_singular(args)
    assert torch.equal(sel.tokens, out["tokens"])
    assert int(sel.tokens[5]) == 1029  # reference greedy tile rule on the planted tie
    assert torch.equal(kw["decode_counts"], out["decode_counts"])
    rows = sel.tokens.size(0)
    stoch = _stochastic_rows(kw, rows)
    assert stoch, "case must hold stochastic rows"
    lp = sel.logprobs
    torch.testing.assert_close(lp.selected[stoch], out["logprobs"][stoch], atol=LOGPROB_ATOL, rtol=0)
    slots = slots_of(kw, rows)
    for r in stoch:
        s = slots[r]
        if int(kw["indicators"][s]) & 0x400:
            z = min(int(kw["top_k_logprobs"][s]), meta["max_top_logprobs"])
            assert torch.equal(lp.top_k.tokens[r, :z], out["top_tokens"][r, :z])
            torch.testing.assert_close(lp.top_k.logprobs[r, :z], out["top_logprobs"][r, :z], atol=LOGPROB_ATOL, rtol=0)


def test_singular_drafting(oracle_lib):
    case = load("singular_drafting")
    kw = singular_kwargs(case, "cpu")
    meta, out = case["meta"], case["outputs"]
    probs = torch.zeros(kw["indicators"].numel(), meta["target_vocab"], dtype=F32)
    sel, args = prepare_singular(lookahead=meta["lookahead"], target_vocab=meta["target_vocab"],
                                 return_probabilities=True, draft_probabilities=probs, **kw)
    oracle_lib.fused_singular(args)
    assert torch.equal(sel.tokens, out["tokens"])
    assert torch.equal(probs != 0, out["probabilities"] != 0)
    torch.testing.assert_close(probs, out["probabilities"], rtol=1e-5, atol=1e-7)


def multistep_kwargs(case: dict, device) -> dict:
    kw = to(case["inputs"], device)
    kw.update(block_n=case["meta"]["block_n"], enable_pdl=False, lookahead=case["meta"]["lookahead"])
    return kw


def check_multistep(ver, kw, case, device="cpu"):
    out = case["outputs"]
    zcap = case["meta"]["max_top_logprobs"]
    assert torch.equal(ver.offsets.cpu(), out["offsets"])
    assert torch.equal(ver.tokens.cpu(), out["tokens"])
    assert torch.equal(kw["decode_counts"].cpu(), out["decode_counts"])
    cu = kw.get("cu_seqlens")
    gamma = case["meta"]["lookahead"]
    ind = kw["indicators"].cpu()
    batch = ver.offsets.size(0)
    slots = slots_of(kw, batch)
    sel = ver.logprobs.selected.cpu().reshape(-1)
    ref_sel = out["logprobs"].reshape(-1)
    top = ver.logprobs.top_k.logprobs.cpu().reshape(-1, zcap)
    ref_top = out["top_logprobs"].reshape(-1, zcap)
    toks = ver.logprobs.top_k.tokens.cpu().reshape(-1, zcap)
    ref_toks = out["top_tokens"].reshape(-1, zcap)
    checked = 0
    for b in range(batch):
        s = slots[b]
        if int(ind[s]) & 0x40:
            continue  # greedy requests write no logprobs
        margin = b * (gamma + 1) if cu is None else int(cu[b])
        acc = int(ver.offsets[b])
        rows = list(range(margin, margin + acc + 1))
        torch.testing.assert_close(sel[rows], ref_sel[rows], atol=LOGPROB_ATOL, rtol=0)
        if int(ind[s]) & 0x400:
            z = min(int(kw["top_k_logprobs"][s]), zcap)
            assert torch.equal(toks[rows, :z], ref_toks[rows, :z])
            a, r = top[rows, :z], ref_top[rows, :z]
            assert torch.equal(torch.isinf(a), torch.isinf(r))
            torch.testing.assert_close(a[~torch.isinf(a)], r[~torch.isinf(r)], atol=LOGPROB_ATOL, rtol=0)
        checked += 1
    return checked


@pytest.mark.parametrize("name", ["multistep_stochastic", "multistep_mixed", "multistep_varlen"])
def test_multistep(oracle_lib, name):
    case = load(name)
    kw = multistep_kwargs(case, "cpu")
    ver, args = prepare_multistep(max_top_logprobs=case["meta"]["max_top_logprobs"], update_counts=True,
                                  return_logprobs=True, logprobs_dtype=F32, **kw)
    oracle_lib.fused_multistep(args)
    assert check_multistep(ver, kw, case) > 0


@pytest.mark.parametrize("tag", ["small", "blocks"])
def test_indexed_copy(tag):
    """The oracle's noise staging against the reference kernel's own output (bit for bit)."""
    from oracle import oracle

    case = load("indexed_copy")
    i, o = case["inputs"][tag], case["outputs"][tag]
    target = i["target"].clone()
    oracle.indexed_copy(i["source"], target, i["indices"], i["indicator"])
    assert torch.equal(target.view(torch.int16), o["target"].view(torch.int16))
