"""Slot population, host side (no GPU): SamplingBuffers.allocate / update pack their calls
exactly as on the GPU, the oracle applies the packed call in place of the kernel, and the
noise is refreshed by the same code as on the GPU; the buffers must then equal the
reference's own SamplingBuffers after the same call sequence (tests/golden/populate.pt)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from sonic_sampler_b200.core import population as pop
from sonic_sampler_b200.core.buffers import (
    Flags,
    GumbelNoise,
    RepetitionPenalties,
    SamplingBuffers,
    StochasticWeights,
    TokenCounts,
)
from sonic_sampler_b200.core.flags import Indicator, ScopedIndicators

GOLDEN = Path(__file__).resolve().parent / "golden" / "populate.pt"
BIAS_BIT = int(Indicator.BIAS)


def buffers_from_state(st: dict, device="cpu") -> SamplingBuffers:
    mv = lambda t: t.clone().to(device)  # noqa: E731
    packed = st["flags"].T.contiguous().clone().to(device).T
    return SamplingBuffers(
        grammar=mv(st["grammar"]).view(torch.uint32),
        repetition=RepetitionPenalties(
            counts=TokenCounts(context=mv(st["context"]), decode=mv(st["decode"])),
            frequency=mv(st["frequency"]), presence=mv(st["presence"]), multiplicative=mv(st["multiplicative"])),
        bias=mv(st["bias"]), temperature=mv(st["temperature"]), top_k=mv(st["top_k"]), top_p=mv(st["top_p"]),
        min_p=mv(st["min_p"]), top_logprobs=mv(st["top_logprobs"]),
        weights=StochasticWeights(uniform=mv(st["uniform"]),
                                  gumbel=GumbelNoise(target=mv(st["gumbel_target"]), draft=mv(st["gumbel_draft"]))),
        flags=Flags(packed=packed, target_host=[int(v) for v in st["flags"][:, 0]],
                    draft_host=[int(v) for v in st["flags"][:, 1]]),
    )


def dest_of(buf: SamplingBuffers) -> dict:
    rep = buf.repetition
    return dict(temperature=buf.temperature, top_p=buf.top_p, min_p=buf.min_p, top_k=buf.top_k,
                top_logprobs=buf.top_logprobs, multiplicative=rep.multiplicative, frequency=rep.frequency,
                presence=rep.presence, flags_target=buf.flags.target, flags_draft=buf.flags.draft,
                context=rep.counts.context, decode=rep.counts.decode, bias=buf.bias, grammar=buf.grammar)


def with_oracle_launch(buf: SamplingBuffers) -> SamplingBuffers:
    """The oracle applies each packed call where the GPU path launches the kernel."""
    dest = dest_of(buf)

    def launch(batch, scoped, positions, stream):
        oracle.populate_slots(batch, dest)
        if scoped is not None:
            buf.flags.update_host(scoped, positions)

    buf._launch = launch
    return buf


def bits(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


def assert_state(buf: SamplingBuffers, want: dict, tag: str) -> None:
    got = dest_of(buf)
    assert torch.equal(buf.flags.packed, want["flags"]), tag
    for name in ("temperature", "top_p", "min_p", "top_k", "top_logprobs", "multiplicative", "frequency", "presence",
                 "context", "decode"):
        assert torch.equal(bits(got[name]), bits(want[name])), (tag, name)
    assert torch.equal(got["grammar"].view(torch.int32), want["grammar"]), (tag, "grammar")
    # bias rows are read only under the BIAS indicator bit; elsewhere the reference copies
    # whatever its pinned mirror last held, and this implementation writes zeros
    on = (want["flags"][:, 0].to(torch.int32) & BIAS_BIT) != 0
    assert torch.equal(bits(got["bias"][on]), bits(want["bias"][on])), (tag, "bias")
    if "gumbel_target" in want:
        assert torch.equal(bits(buf.weights.gumbel.target), bits(want["gumbel_target"])), (tag, "gumbel target")
        assert torch.equal(bits(buf.weights.gumbel.draft), bits(want["gumbel_draft"])), (tag, "gumbel draft")
        assert torch.equal(bits(buf.weights.uniform), bits(want["uniform"])), (tag, "uniform")


def replay(buf: SamplingBuffers, calls: list, outputs: list, tag: str, generator_device="cpu") -> None:
    for k, (call, want) in enumerate(zip(calls, outputs)):
        gen = torch.Generator(generator_device).manual_seed(call["generator_seed"])
        getattr(buf, call["kind"])(generator=gen, **call["kwargs"])
        assert_state(buf, want, f"{tag} call {k}")


@pytest.fixture(scope="module")
def golden():
    return torch.load(GOLDEN, weights_only=False)


@pytest.mark.parametrize("tag", ["small", "ranges"])
def test_allocate_update_match_reference(golden, tag):
    inp = golden["inputs"][tag]
    buf = with_oracle_launch(buffers_from_state(inp["initial"]))
    replay(buf, inp["calls"], golden["outputs"][tag], tag)


def test_bias_rows_of_unbiased_slots_are_zero(golden):
    inp = golden["inputs"]["small"]
    buf = with_oracle_launch(buffers_from_state(inp["initial"]))
    replay(buf, inp["calls"], golden["outputs"]["small"], "small")
    off = (buf.flags.packed[:, 0].to(torch.int32) & BIAS_BIT) == 0
    assert off.any() and not buf.bias[off].any()


def test_bf16_rounding_matches_torch_tensor():
    vals = [0.1, 1.0 / 3.0, 1.00390625, 1.0 + 2 ** -9, -2.5e-39, 3.0e38, 0.0]
    got = pop.bf16_bits(vals)
    want = torch.tensor(vals, dtype=torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, want)


def test_packing_sections_and_blob_roundtrip():
    batch = pop.new_batch([3, 0], num_slots=4, vocab_size=100)
    scoped = ScopedIndicators.from_params(2, temperature=[0.5, 1.0], top_k=[1, 30])
    pop.pack_scalars(batch, [0.5, 1.0], [1.0, 0.9], [0.0, 0.1], [1.0, 1.2], [0.0, 0.3], [0.0, 0.1], [1, 30], [0, 2],
                     scoped.target, scoped.draft)
    pop.pack_histogram(batch, [torch.tensor([1, 1, 99]), torch.tensor([], dtype=torch.int64)])
    pop.pack_bias(batch, [{5: 1.0}, None])
    pop.pack_grammar(batch, [None, torch.zeros(4, dtype=torch.int32)], timesteps=2, step=0)
    assert batch.parts == pop.SCALARS | pop.HISTOGRAM | pop.BIAS | pop.GRAMMAR
    assert batch.token_offsets.tolist() == [0, 3, 3] and batch.bias_offsets.tolist() == [0, 1, 1]
    assert batch.grammar_rows.tolist() == [-1, 0] and batch.grammar_step == 0
    offsets, size = pop.blob_layout(batch)
    assert all(o % 16 == 0 for o in offsets.values())
    blob = np.zeros(size, dtype=np.uint8)
    pop.write_blob(batch, blob)
    for name, arr in batch.sections():
        o = offsets[name]
        assert np.array_equal(blob[o:o + arr.nbytes].view(arr.dtype), arr.reshape(-1)), name


def test_packing_rejects_what_the_reference_rejects():
    batch = pop.new_batch([0], num_slots=2, vocab_size=10)
    with pytest.raises(RuntimeError):
        pop.pack_histogram(batch, [torch.tensor([10])])  # scatter_add_ index out of bounds
    with pytest.raises(ValueError):
        pop.pack_bias(batch, [{-1: 1.0}])
    with pytest.raises(IndexError):
        pop.new_batch([2], num_slots=2, vocab_size=10)
    with pytest.raises(ValueError):
        pop.new_batch([1, 1], num_slots=2, vocab_size=10)
    with pytest.raises(ValueError):
        ScopedIndicators.from_params(1, top_k=[129])
    with pytest.raises(ValueError):
        pop.pack_grammar(batch, [torch.zeros(3, dtype=torch.int32)], timesteps=2, step=0)  # W = 1 word


def test_population_needs_cuda_buffers():
    buf = SamplingBuffers.default(2, 1, 64)
    with pytest.raises(ValueError, match="CUDA"):
        buf.allocate([torch.tensor([1])], [1.0], [0.0], [0.0], [None], [1.0], [128], [1.0], [0.0], [0], [0])


def test_indicator_bits_match_indicator_from_params():
    """The batch path's integer resolution equals Indicator.from_params (core/flags.py:150-184)."""
    import random

    from sonic_sampler_b200.core.flags import _indicator_bits

    rng = random.Random(1)
    for _ in range(5000):
        args = (rng.random() < .5, rng.choice([1.0, 0.9, 1.2]), rng.choice([0.0, 0.3]), rng.choice([0.0, -0.1]),
                rng.random() < .5, rng.choice([1.0, 0.0, 0.7]), rng.choice([1, 2, 20, 127, 128]),
                rng.choice([1.0, 0.0, 0.9, 1.5]), rng.choice([0.0, 0.05, 1.0]), rng.choice([0, 3, 128, 129]),
                rng.random() < .5)
        assert _indicator_bits(*args) == int(Indicator.from_params(*args)), args
