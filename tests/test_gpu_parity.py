"""CUDA path against the CPU oracle (bit-exact: tokens, offsets, counts, candidate ids,
probabilities and logprobs, which share the oracle's fixed fp32 order) and against the
reference's golden vectors (tokens exact, fp32 logprobs within 1e-5).

All calls go through the public interface and the C ABI of libsonic_b200.so."""

from __future__ import annotations

import pytest
import torch

from golden_cases import F32, LOGPROB_ATOL, load, singular_kwargs, slots_of, to
from test_oracle_golden import check_multistep, multistep_kwargs

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16
I32 = torch.int32


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from sonic_sampler_b200 import _abi

    _abi.load_library()  # fails loudly when the extension is missing
    return torch.device("cuda", 0)


def bits(t):
    t = t.cpu()
    return t.view(torch.int16) if t.dtype == BF16 else (t.view(torch.int32) if t.dtype == F32 else t)


# ----------------------------------------------------------------------------------------
# golden cases (reference outputs) on the GPU
# ----------------------------------------------------------------------------------------


@pytest.mark.parametrize("k", [32, 128])
def test_golden_topk(dev, k):
    from sonic_sampler_b200.interface import UnshardedBoundedTopK

    case = load("topk_bf16")
    x = case["inputs"]["logits"].to(dev)
    rows, vocab = x.shape
    topk = UnshardedBoundedTopK.initialize(vocab, block_size=1024, batch_size=rows, k=k).clear()
    topk(x)
    torch.cuda.synchronize()
    assert torch.equal(topk.indices.reshape(-1)[: rows * k].cpu(), case["outputs"][f"indices_k{k}"])
    assert torch.equal(bits(topk.values.reshape(-1)[: rows * k]), bits(case["outputs"][f"values_k{k}"]))


def test_golden_topk_bitonic(dev):
    from sonic_sampler_b200.interface import UnshardedBoundedTopK

    case = load("topk_bitonic")
    x = case["inputs"]["logits"].to(dev)
    rows, vocab = x.shape
    topk = UnshardedBoundedTopK.initialize(vocab, block_size=1024, batch_size=rows, k=128).clear()
    topk(x)
    torch.cuda.synchronize()
    assert torch.equal(topk.indices.reshape(-1)[: rows * 128].cpu(), case["outputs"]["indices"])
    assert torch.equal(bits(topk.values.reshape(-1)[: rows * 128]), bits(case["outputs"]["values"]))


def _singular_both(case, dev, **extra):
    """Run the same singular call on the GPU and on the oracle; return both selections and
    the device/host kwargs (whose decode counts were updated in place)."""
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.singular import fused_singular, prepare_singular

    kd = singular_kwargs(case, dev)
    kh = singular_kwargs(case, "cpu")
    probs_d = probs_h = None
    if "target_vocab" in extra:
        probs_d = torch.zeros(kd["indicators"].numel(), extra["target_vocab"], dtype=F32, device=dev)
        probs_h = probs_d.cpu().clone()
    sel_d = fused_singular(draft_probabilities=probs_d, **extra, **kd)
    ref, args = prepare_singular(draft_probabilities=probs_h, **extra, **kh)
    oracle.fused_singular(args)
    torch.cuda.synchronize()
    return sel_d, ref, kd, kh, probs_d, probs_h


@pytest.mark.parametrize("lp_dtype", [F32, BF16])
def test_golden_singular_mixed(dev, lp_dtype):
    case = load("singular_mixed")
    meta, out = case["meta"], case["outputs"]
    sel, ref, kd, kh, _, _ = _singular_both(case, dev, update_counts=True, return_logprobs=True,
                                            max_top_logprobs=meta["max_top_logprobs"], logprobs_dtype=lp_dtype)
    assert torch.equal(sel.tokens.cpu(), out["tokens"])
    assert torch.equal(sel.tokens.cpu(), ref.tokens)
    assert torch.equal(kd["decode_counts"].cpu(), out["decode_counts"])
    rows = sel.tokens.size(0)
    slots = slots_of(kh, rows)
    stoch = [r for r in range(rows) if not (int(kh["indicators"][slots[r]]) & 0x40)]
    assert torch.equal(bits(sel.logprobs.selected[stoch]), bits(ref.logprobs.selected[stoch]))
    if lp_dtype == F32:
        torch.testing.assert_close(sel.logprobs.selected.cpu()[stoch], out["logprobs"][stoch], atol=LOGPROB_ATOL, rtol=0)
    for r in stoch:
        s = slots[r]
        if int(kh["indicators"][s]) & 0x400:
            z = min(int(kh["top_k_logprobs"][s]), meta["max_top_logprobs"])
            assert torch.equal(sel.logprobs.top_k.tokens[r, :z].cpu(), out["top_tokens"][r, :z])
            assert torch.equal(bits(sel.logprobs.top_k.logprobs[r, :z]), bits(ref.logprobs.top_k.logprobs[r, :z]))


def test_golden_singular_drafting(dev):
    case = load("singular_drafting")
    meta, out = case["meta"], case["outputs"]
    sel, ref, _, _, pd, ph = _singular_both(case, dev, lookahead=meta["lookahead"], target_vocab=meta["target_vocab"],
                                            return_probabilities=True)
    assert torch.equal(sel.tokens.cpu(), out["tokens"])
    assert torch.equal(bits(pd), bits(ph))
    torch.testing.assert_close(pd.cpu(), out["probabilities"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("name", ["multistep_stochastic", "multistep_mixed", "multistep_varlen"])
def test_golden_multistep(dev, name):
    from oracle import oracle
    from sonic_sampler_b200.interface.functional.multistep import fused_multistep, prepare_multistep

    case = load(name)
    zcap = case["meta"]["max_top_logprobs"]
    kd = multistep_kwargs(case, dev)
    kh = multistep_kwargs(case, "cpu")
    common = dict(max_top_logprobs=zcap, update_counts=True, return_logprobs=True, logprobs_dtype=F32)
    values = torch.zeros(kd["logits"].reshape(-1, kd["logits"].size(-1)).size(0), 128, dtype=F32, device=dev)
    indices = torch.full_like(values, -1, dtype=I32)
    vh, ih = values.cpu().clone(), indices.cpu().clone()
    ver = fused_multistep(values=values, indices=indices, **common, **kd)
    ref, args = prepare_multistep(values=vh, indices=ih, **common, **kh)
    oracle.fused_multistep(args)
    torch.cuda.synchronize()
    assert check_multistep(ver, kd, case) > 0  # against the reference
    assert torch.equal(ver.tokens.cpu(), ref.tokens)
    assert torch.equal(ver.offsets.cpu(), ref.offsets)
    assert torch.equal(kd["decode_counts"].cpu(), kh["decode_counts"])
    # candidate buffers: identical where the oracle wrote them
    written = ih != -1
    assert torch.equal(indices.cpu()[written], ih[written])
    assert torch.equal(bits(values)[written], bits(vh)[written])
