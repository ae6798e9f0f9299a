"""The bounded-wait error path, on the GPU, without a fault.

Every wait of the ring-streaming kernels gives up after a bounded number of polls. A CTA whose
wait gave up leaves the streaming loop, lets its in-flight bulk copies land, records
SONIC_DEVICE_ERR_WAIT in the workspace's error word and marks its row (or multistep request)
failed, so the row writes none of its outputs. The diagnostic flag SONIC_FLAG_DEBUG_STALL_RING
makes every CTA's first wait one on a barrier that nothing completes, with a short limit: the
wait runs out, no GPU fault or hang is involved, and the call must return with its outputs
untouched, the error readable through sonic_workspace_error, and the workspace still valid for
the next call (checked against the CPU oracle)."""

from __future__ import annotations

import ctypes

import pytest
import torch

from sonic_sampler_b200 import workloads

pytestmark = pytest.mark.gpu

SENTINEL = -7


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from sonic_sampler_b200 import _abi

    _abi.load_library()
    return torch.device("cuda", 0)


def _singular_kwargs(b, processors: bool) -> dict:
    kw = dict(indicators=b.flags.target, temperature=b.temperature, top_k=b.top_k, top_p=b.top_p, min_p=b.min_p,
              top_k_logprobs=b.top_logprobs, gumbel_noise=b.weights.gumbel.target[:, 0], return_logprobs=True)
    if processors:
        kw.update(grammar=b.grammar[:, 0], context_counts=b.repetition.counts.context,
                  decode_counts=b.repetition.counts.decode, repetition_penalties=b.repetition.multiplicative,
                  frequency_penalties=b.repetition.frequency, presence_penalties=b.repetition.presence,
                  logit_bias=b.bias)
    return kw


def _launch(entry: str, args) -> None:
    from sonic_sampler_b200 import _abi

    lib = _abi.load_library()
    stream = torch.cuda.current_stream().cuda_stream
    _abi.check(getattr(lib, entry)(ctypes.byref(args), ctypes.c_void_p(stream)), lib)


@pytest.mark.parametrize("processors", [True, False], ids=["singular_kernel", "logits_only_kernel"])
def test_singular_wait_timeout_writes_nothing_and_is_reported(dev, processors):
    from oracle import oracle
    from sonic_sampler_b200 import _abi, ops
    from sonic_sampler_b200.interface.functional.singular import fused_singular, prepare_singular

    # config 2's shape: its column splits span several ring chunks in both kernels
    w = workloads.config2(dev, seed=21)
    kw = _singular_kwargs(w["buffers"], processors)
    ws = ops.new_workspace(ops.singular_workspace_bytes(64, 128256), dev)
    sel, args = prepare_singular(w["logits"], block_n=4096, scratchpad=ws, **kw)
    sel.tokens.fill_(SENTINEL)
    sel.logprobs.selected.fill_(float(SENTINEL))
    args.flags |= _abi.FLAG_DEBUG_STALL_RING
    _launch("sonic_fused_singular", args)
    torch.cuda.synchronize()
    assert bool((sel.tokens == SENTINEL).all()), "a row with a failed split wrote its token"
    assert bool((sel.logprobs.selected == SENTINEL).all())
    assert ops.workspace_error(ws) & _abi.DEVICE_ERR_WAIT
    assert ops.workspace_error(ws) == 0  # read clears it

    # the same workspace serves the next call: tickets were re-armed by the failed call
    good = fused_singular(w["logits"], block_n=4096, scratchpad=ws, **kw)
    hk = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
    ref, rargs = prepare_singular(w["logits"].cpu(), block_n=4096, **hk)
    oracle.fused_singular(rargs)
    torch.cuda.synchronize()
    assert torch.equal(good.tokens.cpu(), ref.tokens)
    assert ops.workspace_error(ws) == 0


def test_multistep_wait_timeout_writes_nothing_and_is_reported(dev):
    from oracle import oracle
    from sonic_sampler_b200 import _abi, ops
    from sonic_sampler_b200.interface.functional.multistep import fused_multistep, prepare_multistep

    c = workloads.config3(dev, seed=23, batch=4, gamma=3, vocab=32000, varlen=False)
    b = c["buffers"]
    kw = dict(grammar=b.grammar, context_counts=b.repetition.counts.context, decode_counts=b.repetition.counts.decode,
              repetition_penalties=b.repetition.multiplicative, frequency_penalties=b.repetition.frequency,
              presence_penalties=b.repetition.presence, logit_bias=b.bias, temperature=b.temperature, top_k=b.top_k,
              top_p=b.top_p, min_p=b.min_p, top_k_logprobs=b.top_logprobs, gumbel_noise=b.weights.gumbel.target,
              uniform_noise=b.weights.uniform, lookahead=c["gamma"], draft_probabilities=c["probabilities"],
              block_n=2048, return_logprobs=True)
    ws = ops.new_workspace(ops.multistep_workspace_bytes(4, c["gamma"], 32000), dev)
    tokens = c["tokens"].clone()
    ver, args = prepare_multistep(c["logits"], b.flags.target, tokens, scratchpad=ws, **kw)
    ver.offsets.fill_(SENTINEL)
    args.flags |= _abi.FLAG_DEBUG_STALL_RING
    _launch("sonic_fused_multistep", args)
    torch.cuda.synchronize()
    assert bool((ver.offsets == SENTINEL).all())
    assert torch.equal(ver.tokens, c["tokens"])  # drafted tokens untouched
    assert ops.workspace_error(ws) & _abi.DEVICE_ERR_WAIT

    good = fused_multistep(c["logits"], b.flags.target, c["tokens"].clone(), scratchpad=ws, **kw)
    hk = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
    ref, rargs = prepare_multistep(c["logits"].cpu(), b.flags.target.cpu(), c["tokens"].cpu().clone(), **hk)
    oracle.fused_multistep(rargs)
    torch.cuda.synchronize()
    assert torch.equal(good.offsets.cpu(), ref.offsets)
    assert torch.equal(good.tokens.cpu(), ref.tokens)
    assert ops.workspace_error(ws) == 0


def test_multistep_logits_only_wait_timeout(dev):
    """The same for multistep rows on the logits-only kernel (no grammar, counts or bias)."""
    from oracle import oracle
    from sonic_sampler_b200 import _abi, ops
    from sonic_sampler_b200.interface.functional.multistep import fused_multistep, prepare_multistep

    batch, gamma, vocab = 8, 3, 128256
    x = workloads.peaked_logits(batch * (gamma + 1), vocab, sigma=3.0, peaks=4, lift=12.0, device=dev,
                                seed=24).view(batch, gamma + 1, vocab)
    tokens = x.float().argmax(-1).to(torch.int32).contiguous()
    ind = torch.tensor([0x60, 0x1A0] * (batch // 2), dtype=torch.int32).to(torch.uint16).to(dev)
    kw = dict(temperature=torch.full((batch,), 0.8, dtype=torch.bfloat16, device=dev),
              top_k=torch.full((batch,), 40, dtype=torch.int32, device=dev),
              top_p=torch.full((batch,), 0.9, dtype=torch.bfloat16, device=dev),
              gumbel_noise=workloads.log_exponential((batch, gamma + 1, vocab), dev, 25),
              uniform_noise=torch.full((batch, gamma + 1), 0.5, dtype=torch.bfloat16, device=dev),
              lookahead=gamma, block_n=4096)
    ws = ops.new_workspace(ops.multistep_workspace_bytes(batch, gamma, vocab), dev)
    ver, args = prepare_multistep(x, ind, tokens.clone(), scratchpad=ws, **kw)
    ver.offsets.fill_(SENTINEL)
    args.flags |= _abi.FLAG_DEBUG_STALL_RING
    _launch("sonic_fused_multistep", args)
    torch.cuda.synchronize()
    assert bool((ver.offsets == SENTINEL).all())
    assert ops.workspace_error(ws) & _abi.DEVICE_ERR_WAIT

    good = fused_multistep(x, ind, tokens.clone(), scratchpad=ws, **kw)
    hk = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}
    ref, rargs = prepare_multistep(x.cpu(), ind.cpu(), tokens.cpu().clone(), **hk)
    oracle.fused_multistep(rargs)
    torch.cuda.synchronize()
    assert torch.equal(good.offsets.cpu(), ref.offsets)
    assert torch.equal(good.tokens.cpu(), ref.tokens)
    assert ops.workspace_error(ws) == 0


def test_static_entry_reports_into_the_library_word(dev):
    from sonic_sampler_b200 import _abi, ops
    from sonic_sampler_b200.interface.functional.singular import prepare_singular

    w = workloads.config2(dev, seed=22, batch=8, vocab=32000)
    kw = _singular_kwargs(w["buffers"], True)
    ops.workspace_error(None, dev)  # start from a clean library word
    sel, args = prepare_singular(w["logits"], block_n=2048, **kw)
    sel.tokens.fill_(SENTINEL)
    args.flags |= _abi.FLAG_DEBUG_STALL_RING
    _launch("sonic_fused_singular_static", args)
    torch.cuda.synchronize()
    assert bool((sel.tokens == SENTINEL).all())
    assert ops.workspace_error(None, dev) & _abi.DEVICE_ERR_WAIT
    # a clean call afterwards writes every token and leaves the word clear
    args.flags &= ~_abi.FLAG_DEBUG_STALL_RING
    _launch("sonic_fused_singular_static", args)
    torch.cuda.synchronize()
    assert bool((sel.tokens != SENTINEL).all())
    assert ops.workspace_error(None, dev) == 0
