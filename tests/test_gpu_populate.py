"""Slot population on the GPU: SamplingBuffers.allocate / update / step_grammar through
`sonic_populate_slots`, against the reference's recorded buffers (tests/golden/populate.pt)
and, at full vocabulary size, against the oracle applied to the same packed calls."""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from sonic_sampler_b200.core.buffers import SamplingBuffers
from tests.test_populate import BIAS_BIT, assert_state, bits, buffers_from_state, dest_of

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def golden():
    return torch.load("tests/golden/populate.pt", weights_only=False)


def without_noise(state: dict) -> dict:
    return {k: v for k, v in state.items() if k not in ("gumbel_target", "gumbel_draft", "uniform")}


@pytest.mark.parametrize("tag", ["small", "ranges"])
def test_gpu_population_matches_reference(golden, tag):
    """The reference's own call sequence through the kernel; the noise comes from a CUDA
    generator here, so only the populated fields are compared."""
    inp = golden["inputs"][tag]
    buf = buffers_from_state(inp["initial"], device=DEV)
    for k, (call, want) in enumerate(zip(inp["calls"], golden["outputs"][tag])):
        gen = torch.Generator(DEV).manual_seed(call["generator_seed"])
        getattr(buf, call["kind"])(generator=gen, **call["kwargs"])
        torch.cuda.synchronize()
        host = buffers_from_state({**{n: t.cpu() for n, t in snapshot(buf).items()}}, device="cpu")
        assert_state(host, without_noise(want), f"{tag} call {k}")


def snapshot(buf: SamplingBuffers) -> dict:
    d = dest_of(buf)
    w = buf.weights
    return dict(flags=buf.flags.packed, temperature=d["temperature"], top_p=d["top_p"], min_p=d["min_p"],
                top_k=d["top_k"], top_logprobs=d["top_logprobs"], multiplicative=d["multiplicative"],
                frequency=d["frequency"], presence=d["presence"], context=d["context"], decode=d["decode"],
                bias=d["bias"], grammar=d["grammar"].view(torch.int32), gumbel_target=w.gumbel.target,
                gumbel_draft=w.gumbel.draft, uniform=w.uniform)


def recording(buf: SamplingBuffers, log: list) -> SamplingBuffers:
    """Keep every packed call the GPU path launches, for the oracle."""
    launch = buf._launch

    def wrapped(batch, scoped, positions, stream):
        log.append(batch)
        launch(batch, scoped, positions, stream)

    buf._launch = wrapped
    return buf


def random_params(n: int, g: torch.Generator, V: int) -> dict:
    return dict(
        multiplicative=[float(x) for x in torch.rand(n, generator=g) + 0.5],
        frequency=[float(x) for x in torch.rand(n, generator=g) - 0.5],
        presence=[float(x) for x in torch.rand(n, generator=g)],
        biases=[None if j % 4 == 3 else {int(t): float(torch.randn(1, generator=g))
                                          for t in torch.randperm(V, generator=g)[:64]} for j in range(n)],
        temperature=[float(x) for x in torch.rand(n, generator=g) + 0.3],
        top_k=[int(x) for x in torch.randint(1, 129, (n,), generator=g)],
        top_p=[float(x) for x in torch.rand(n, generator=g) * 0.5 + 0.5],
        min_p=[float(x) for x in torch.rand(n, generator=g) * 0.1],
        top_logprobs=[int(x) for x in torch.randint(0, 8, (n,), generator=g)],
    )


def test_gpu_population_full_vocabulary_matches_oracle():
    """B=64 slots, T=4, V=128256: admission of 40 slots with prompts of up to 6000 tokens, bias
    entries and step-0 bitmasks; an update of 30 slots from device-resident dense counts with
    per-step and broadcast bitmasks; a grammar-only step. Bit-exact against the oracle."""
    B, T, V = 64, 4, 128256
    W = (V + 31) // 32
    g = torch.Generator().manual_seed(77)
    buf = SamplingBuffers.default(B, T, V, device=DEV)
    ref = buffers_from_state({n: t.cpu() for n, t in snapshot(buf).items()})
    log: list = []
    recording(buf, log)

    pos = torch.randperm(B, generator=g)[:40].tolist()
    kw = random_params(40, g, V)
    enc = [torch.randint(0, V, (int(torch.randint(0, 6000, (1,), generator=g)),), generator=g) for _ in pos]
    masks = [torch.randint(-2**31, 2**31 - 1, (W,), generator=g, dtype=torch.int64).to(torch.int32)
             if j % 2 == 0 else None for j in range(40)]
    buf.allocate(enc, positions=pos, bitmasks=masks, generator=torch.Generator(DEV).manual_seed(1), **kw)

    pos2 = torch.randperm(B, generator=g)[:30].tolist()
    kw2 = random_params(30, g, V)
    counts = [(torch.randint(0, 50, (V,), generator=g, dtype=torch.int32).to(DEV),
               torch.randint(0, 5, (V,), generator=g, dtype=torch.int32).to(DEV)) for _ in pos2]
    masks2 = [torch.randint(-2**31, 2**31 - 1, (T, W) if j % 3 == 0 else (W,), generator=g,
                            dtype=torch.int64).to(torch.int32) if j % 3 != 2 else None for j in range(30)]
    buf.update(counts, [None] * 30, positions=pos2, bitmasks=masks2, generator=torch.Generator(DEV).manual_seed(2),
               **kw2)
    masks3 = [torch.randint(-2**31, 2**31 - 1, (W,), generator=g, dtype=torch.int64).to(torch.int32) for _ in range(3)]
    buf.step_grammar(masks3, positions=[5, 9, 63], timestep=2)
    torch.cuda.synchronize()

    assert len(log) == 3
    dest = dest_of(ref)
    for batch in log:
        oracle.populate_slots(batch, dest)
    got = {n: t.cpu() for n, t in snapshot(buf).items()}
    want = snapshot(ref)
    for name in ("flags", "temperature", "top_p", "min_p", "top_k", "top_logprobs", "multiplicative", "frequency",
                 "presence", "context", "decode", "bias", "grammar"):
        assert torch.equal(bits(got[name]), bits(want[name])), name
    assert int(got["context"].sum()) == sum(int(e.numel()) for e, p in zip(enc, pos) if p not in pos2) + \
        sum(int(c.sum()) for (c, _), p in zip(counts, pos2))


def test_gpu_population_unaligned_rows():
    """Rows whose starts are not 16-byte aligned (V = 1003 with row strides of 1003) take the
    element-wise paths; still bit-exact."""
    B, T, V = 5, 2, 1003
    buf = SamplingBuffers.default(B, T, V, device=DEV)
    ref = buffers_from_state({n: t.cpu() for n, t in snapshot(buf).items()})
    log: list = []
    recording(buf, log)
    g = torch.Generator().manual_seed(3)
    kw = random_params(3, g, V)
    enc = [torch.randint(0, V, (500,), generator=g) for _ in range(3)]
    buf.allocate(enc, positions=[1, 4, 2], **kw)
    torch.cuda.synchronize()
    dest = dest_of(ref)
    for batch in log:
        oracle.populate_slots(batch, dest)
    got = {n: t.cpu() for n, t in snapshot(buf).items()}
    want = snapshot(ref)
    for name in ("context", "decode", "bias", "flags", "temperature"):
        assert torch.equal(bits(got[name]), bits(want[name])), name
    on = (got["flags"][:, 0].to(torch.int32) & BIAS_BIT) != 0
    assert on.any()


def test_gpu_step_weights_stages_draft_noise():
    """step_weights (core/buffer.py:1054-1096): the draft noise of slots whose draft indicator is
    stochastic moves into their target noise, then the stochastic slots' noise is refreshed
    (the draft rows of stochastically drafted slots, the target rows otherwise)."""
    B, T, V = 6, 3, 4096
    buf = SamplingBuffers.default(B, T, V, device=DEV)
    g = torch.Generator().manual_seed(11)
    kw = random_params(4, g, V)
    kw["top_k"] = [1, 30, 30, 30]  # slot 0 greedy
    buf.allocate([torch.randint(0, V, (100,), generator=g) for _ in range(4)], positions=[0, 2, 3, 5],
                 greedy_drafts=[False, False, True, False], **kw)
    torch.cuda.synchronize()
    before_t = buf.weights.gumbel.target.clone()
    before_d = buf.weights.gumbel.draft.clone()
    positions = [0, 2, 3, 5]
    buf.step_weights(positions, indices=torch.tensor(positions, device=DEV), generator=torch.Generator(DEV).manual_seed(5))
    torch.cuda.synchronize()
    t, d = buf.weights.gumbel.target, buf.weights.gumbel.draft
    # slot 2: stochastic draft -> target = old draft, draft refreshed
    assert torch.equal(t[2], before_d[2]) and not torch.equal(d[2], before_d[2])
    # slot 3: greedy draft -> no staging; target refreshed, draft untouched
    assert not torch.equal(t[3], before_t[3]) and torch.equal(d[3], before_d[3])
    # slot 0: greedy target -> untouched; slots 1 and 4 not in the call -> untouched
    for s in (0, 1, 4):
        assert torch.equal(t[s], before_t[s]) and torch.equal(d[s], before_d[s])
