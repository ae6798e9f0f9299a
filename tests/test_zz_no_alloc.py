"""sonic_fused_singular_static, the singular entry point that allocates nothing, against
sonic_fused_singular with a caller workspace. Both are called through the C ABI.

Some hosts cannot give this library device memory: an engine that has already handed all
free HBM to its KV cache, a cgo or JNI binding with no handle to the framework's caching
allocator, or a decode loop that cannot afford a cudaMalloc that may synchronise the
device. The static entry point runs the same kernel on a 4 MiB scratch array compiled into
the library and clears its tickets itself, so two calls in a row must both reproduce the
workspace entry point's output exactly (tokens bit for bit, logprobs within the 1e-5 bound
of the other GPU tests; here they are bit-identical, as the kernel is the same).

The file name sorts last so that a run stopping at its first failure has already run every
other test."""

from __future__ import annotations

import ctypes

import pytest
import torch

from sonic_sampler_b200 import workloads

pytestmark = pytest.mark.gpu

LOGPROB_ATOL = 1e-5


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
        gumbel_noise=b.weights.gumbel.target[:, 0], return_logprobs=True,
    )
    kw.update(extra)
    return kw


def _call(entry: str, logits, kw, dev):
    """One call of `entry` through the C ABI on the current stream; returns the selection
    and the argument struct (which keeps its tensors alive)."""
    from sonic_sampler_b200 import _abi
    from sonic_sampler_b200.interface.functional.singular import prepare_singular

    sel, args = prepare_singular(logits, **kw)
    lib = _abi.load_library()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _abi.check(getattr(lib, entry)(ctypes.byref(args), ctypes.c_void_p(stream)), lib)
    return sel, args


def _cases(dev):
    """(name, logits, kwargs, stochastic-row mask, top-logprob count)."""
    c2 = workloads.config2(dev, seed=11)  # B=64, V=128256, every processor, stochastic rows
    mixed_buffers = workloads.sampling_buffers(24, 1, 32000, dev, 5, workloads.config2_params(24, 6),
                                               top_logprobs=8)
    # every third row greedy: both kinds of selection share the scratch in one call
    ind = mixed_buffers.flags.target.cpu().to(torch.int32)
    ind[::3] |= 0x40
    mixed_buffers.flags.packed[:, 0] = ind.to(torch.uint16).to(dev)
    mixed = workloads.peaked_logits(24, 32000, sigma=3.0, peaks=4, lift=12.0, device=dev, seed=5)
    stoch = (ind & 0x40) == 0
    return [
        ("config2", c2["logits"], _kwargs(c2["buffers"]), torch.ones(64, dtype=torch.bool), 0),
        ("mixed", mixed, _kwargs(mixed_buffers, max_top_logprobs=8), stoch, 8),
    ]


def test_static_scratch_matches_workspace_entry(dev):
    for name, logits, kw, stoch, z in _cases(dev):
        ref, ref_args = _call("sonic_fused_singular", logits, kw, dev)
        runs = [_call("sonic_fused_singular_static", logits, kw, dev) for _ in range(2)]
        torch.cuda.synchronize()
        # greedy rows write a token only; compare what each call writes
        ref_lp = ref.logprobs.selected.cpu()[stoch]
        for i, (sel, _) in enumerate(runs):
            assert torch.equal(sel.tokens, ref.tokens), f"{name}: call {i + 1} tokens differ"
            torch.testing.assert_close(sel.logprobs.selected.cpu()[stoch], ref_lp, atol=LOGPROB_ATOL, rtol=0,
                                       equal_nan=True, msg=f"{name}: call {i + 1} logprobs differ")
            if z:
                assert torch.equal(sel.logprobs.top_k.tokens.cpu()[stoch, :z], ref.logprobs.top_k.tokens.cpu()[stoch, :z])
                torch.testing.assert_close(sel.logprobs.top_k.logprobs.cpu()[stoch, :z],
                                           ref.logprobs.top_k.logprobs.cpu()[stoch, :z], atol=LOGPROB_ATOL, rtol=0)
        del ref_args


def test_static_scratch_rejects_oversize(dev):
    from sonic_sampler_b200 import _abi
    from sonic_sampler_b200.ops import SingularArgs

    lib = _abi.load_library()
    a = SingularArgs()
    a.rows, a.vocab_size, a.block_n = 4096, 128256, 4096  # 8 MiB of candidate lists
    # arguments pass every check; the pointers are never dereferenced (the size check fails first)
    a.params.indicators = a.tokens = a.gumbel = a.logits = 1 << 20
    assert lib.sonic_fused_singular_workspace_size(ctypes.byref(a)) > 4 << 20
    status = lib.sonic_fused_singular_static(ctypes.byref(a), ctypes.c_void_p(0))
    assert status == _abi.SONIC_ERR_WORKSPACE
    assert b"static scratch" in lib.sonic_last_error()
