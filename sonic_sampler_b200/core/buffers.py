"""Request-state buffers read by the sampler (layout of reference core/buffer.py:784-817).

The interface classes only read the attribute paths listed below, so the reference's own
`SamplingBuffers` object works unchanged (duck typing); this lighter container has the
same paths, dtypes and shapes for users and tests that do not carry the reference:

    flags.target / flags.draft       u16 [B]   (views of packed [B, 2], stride (1, B))
    flags.all_greedy                 host bool
    grammar                          u32 [B, T, ceil(V/32)]
    repetition.counts.context        i32 [B, V]
    repetition.counts.decode         i32 [B, V]
    repetition.multiplicative / frequency / presence    bf16 [B]
    bias                             bf16 [B, V]
    temperature / top_p / min_p      bf16 [B]
    top_k / top_logprobs             i32 [B]
    weights.uniform                  bf16 [B, T]
    weights.gumbel.target / draft    bf16 [B, T, V]  (log of Exp(1) draws)

Host population (`allocate`, `update`, `step_grammar`, `step_weights`) keeps the reference's
signatures; everything but the noise goes through one batched `sonic_populate_slots` launch
(core/population.py), and the noise is refreshed with the caller's generator in the
reference's order, so a seeded generator gives the reference's noise.
"""

from __future__ import annotations

from contextlib import nullcontext
from dataclasses import dataclass, field
from itertools import compress, repeat
from typing import Sequence

import torch
from torch import Tensor

from sonic_sampler_b200.core.flags import MAX_K, Indicator, ScopedIndicators

BF16 = torch.bfloat16
I32 = torch.int32
U16 = torch.uint16
U32 = torch.uint32
TINY = torch.finfo(BF16).tiny


def _on(stream):
    return torch.cuda.stream(stream) if stream is not None else nullcontext()


@dataclass
class Flags:
    packed: Tensor                # u16 [B, 2], stride (1, B)
    target_host: list[int] = field(default_factory=list)
    draft_host: list[int] = field(default_factory=list)

    @classmethod
    def from_values(cls, target: Sequence[int], draft: Sequence[int] | None = None, device=None) -> "Flags":
        draft = list(target) if draft is None else list(draft)
        packed = torch.tensor([list(map(int, target)), list(map(int, draft))], dtype=U16, device=device).T
        return cls(packed=packed, target_host=list(map(int, target)), draft_host=list(map(int, draft)))

    @property
    def target(self) -> Tensor:
        return self.packed[:, 0]

    @property
    def draft(self) -> Tensor:
        return self.packed[:, 1]

    def update_host(self, scoped: ScopedIndicators, positions: Sequence[int]) -> None:
        """Host copies of the indicators (reference ScopedIndicators.update, core/flags.py:418-432)."""
        for i, j in enumerate(positions):
            self.target_host[j] = int(scoped.target[i])
            self.draft_host[j] = int(scoped.draft[i])

    @property
    def all_greedy(self) -> bool:
        g = int(Indicator.GREEDY)
        return all(v & g for v in self.target_host) and all(v & g for v in self.draft_host)


@dataclass
class TokenCounts:
    context: Tensor
    decode: Tensor


@dataclass
class RepetitionPenalties:
    counts: TokenCounts
    frequency: Tensor
    presence: Tensor
    multiplicative: Tensor


@dataclass
class GumbelNoise:
    target: Tensor
    draft: Tensor

    def stage_weights(self, indices: Tensor, indicator: Tensor, stream: torch.cuda.Stream | None = None) -> "GumbelNoise":
        """Copy the draft noise of the slots at `indices` whose indicator is not greedy into the
        target noise (reference `core/buffer.py:151-157`), on `stream` when given."""
        from contextlib import nullcontext

        from sonic_sampler_b200.ops import indexed_copy

        with _on(stream):
            indexed_copy(self.draft, self.target, indices, indicator)
        return self

    def populate(self, row, generator: torch.Generator | None, prefill: bool = False, draft: bool = False) -> "GumbelNoise":
        """Fresh log(Exp(1)) noise in place (reference core/buffer.py:95-120): at prefill the
        target's step 0 (and the whole draft row when drafting is stochastic), else the draft
        (stochastic drafting) or the target row."""
        if prefill:
            tensors = (self.target[row, 0], self.draft[row]) if draft else (self.target[row, 0],)
        else:
            tensors = ((self.draft if draft else self.target)[row],)
        for w in tensors:
            w.exponential_(1.0, generator=generator).log_()
        return self

    def update(self, targets, positions=None, stream=None) -> "GumbelNoise":
        """Copy the given target noise rows in (reference core/buffer.py:122-149)."""
        if any(selectors := [t is not None for t in targets]):
            pairs = zip(positions, targets) if positions else enumerate(targets)
            with _on(stream):
                for i, t in compress(pairs, selectors):
                    self.target[i].copy_(t, non_blocking=True)
        return self


def resolve_updates(size: int, generator=None, selectors=None, positions=None, prefill=False):
    """(position, generator, (target, draft), prefill) of each noise refresh (reference
    core/buffer.py:166-192): one batch-wide refresh for a shared generator without positions or
    selectors, else one per slot."""
    shared = generator is None or isinstance(generator, torch.Generator)
    if shared and not positions and not selectors:
        if isinstance(prefill, bool):
            return [(None, generator, (True, True), prefill)]
        if isinstance(prefill, list) and not prefill:
            return [(None, generator, (True, True), False)]
    indices = positions or range(size)
    predicates = selectors or repeat((True, True))
    generators = generator if isinstance(generator, list) else repeat(generator)
    initials = prefill if isinstance(prefill, list) and prefill else repeat(bool(prefill))
    return zip(indices, generators, predicates, initials)


@dataclass
class StochasticWeights:
    uniform: Tensor
    gumbel: GumbelNoise

    def refresh(self, position, generator, prefill: bool, draft: bool) -> None:
        """Reference core/buffer.py:236-250."""
        row = slice(None) if position is None else position
        self.gumbel.populate(row=row, generator=generator, prefill=prefill, draft=draft)
        if not prefill:
            self.uniform[row].uniform_(TINY, 1.0, generator=generator)

    def update(self, generator=None, selectors=None, targets=None, positions=None, prefill=False, stream=None,
               event=None) -> "StochasticWeights":
        """Noise refresh between iterations (reference core/buffer.py:252-311)."""
        updates = resolve_updates(self.uniform.size(0), generator, selectors, positions, prefill)
        with _on(stream):
            for i, rng, (target, draft), initial in updates:
                if target:
                    self.refresh(position=i, generator=rng, prefill=initial, draft=draft)
            if targets and not prefill:
                self.gumbel.update(targets=targets, positions=positions, stream=stream)
            if event is not None:
                event.record(stream)
        return self

    def step(self, positions, scoped: ScopedIndicators, indicator: Tensor, indices: Tensor | None = None,
             generator=None, stream=None, event=None) -> None:
        """Stage the draft noise into the target and refresh (reference core/buffer.py:313-344)."""
        if indices is not None and scoped.has_stochastic_draft:
            self.gumbel.stage_weights(indices=indices, indicator=indicator, stream=stream)
        self.update(generator=generator, selectors=scoped.stochastic_selectors, positions=positions, stream=stream,
                    event=event)


@dataclass
class SamplingBuffers:
    grammar: Tensor
    repetition: RepetitionPenalties
    bias: Tensor
    temperature: Tensor
    top_k: Tensor
    top_p: Tensor
    min_p: Tensor
    top_logprobs: Tensor
    weights: StochasticWeights
    flags: Flags
    _stager: object = field(default=None, init=False, repr=False, compare=False)

    @property
    def device(self) -> torch.device:
        return self.bias.device

    @property
    def vocab_size(self) -> int:
        return self.bias.size(-1)

    @classmethod
    def default(cls, size: int, timesteps: int, vocab_size: int, device=None,
                generator: torch.Generator | None = None) -> "SamplingBuffers":
        """Neutral parameters (no processors), fresh noise (reference core/buffer.py:939-987)."""
        dev = torch.device(device) if device is not None else torch.device("cpu")
        words = (vocab_size + 31) // 32
        gumbel = torch.empty((2, size, timesteps, vocab_size), dtype=torch.float32, device=dev)
        gumbel.exponential_(1.0, generator=generator).log_()
        gumbel = gumbel.to(BF16)
        uniform = torch.empty((size, timesteps), dtype=torch.float32, device=dev)
        uniform.uniform_(torch.finfo(BF16).tiny, 1.0, generator=generator)
        return cls(
            grammar=torch.full((size, timesteps, words), -1, dtype=I32, device=dev).view(U32),
            repetition=RepetitionPenalties(
                counts=TokenCounts(context=torch.zeros((size, vocab_size), dtype=I32, device=dev),
                                   decode=torch.zeros((size, vocab_size), dtype=I32, device=dev)),
                frequency=torch.zeros(size, dtype=BF16, device=dev),
                presence=torch.zeros(size, dtype=BF16, device=dev),
                multiplicative=torch.ones(size, dtype=BF16, device=dev),
            ),
            bias=torch.zeros((size, vocab_size), dtype=BF16, device=dev),
            temperature=torch.ones(size, dtype=BF16, device=dev),
            top_k=torch.full((size,), MAX_K, dtype=I32, device=dev),
            top_p=torch.ones(size, dtype=BF16, device=dev),
            min_p=torch.zeros(size, dtype=BF16, device=dev),
            top_logprobs=torch.zeros(size, dtype=I32, device=dev),
            weights=StochasticWeights(uniform=uniform.to(BF16),
                                      gumbel=GumbelNoise(target=gumbel[0], draft=gumbel[1])),
            flags=Flags.from_values([0] * size, device=dev),
        )

    # ---- host population (reference core/buffer.py:1026-1352) ----

    def _population(self):
        from sonic_sampler_b200.core import population

        if self.device.type != "cuda":
            raise ValueError("slot population runs on CUDA buffers only (no CPU fallback)")
        if self._stager is None:
            self._stager = population.SlotStager(self.device)
        return population

    def _positions(self, positions, n: int) -> list[int]:
        if positions:
            return [int(p) for p in positions]
        if n != self.bias.size(0):
            raise ValueError(f"without positions the lists must cover all {self.bias.size(0)} slots")
        return list(range(n))

    def step_grammar(self, bitmasks, positions=None, timestep: int | None = None, stream=None, event=None):
        """Bitmask rows into the grammar buffer (reference core/buffer.py:1026-1052): step
        `timestep` of each slot, or every step. The list is aligned with `positions`."""
        if bitmasks and any(m is not None for m in bitmasks):
            pop = self._population()
            batch = pop.new_batch(self._positions(positions, len(bitmasks)), self.bias.size(0), self.vocab_size)
            pop.pack_grammar(batch, bitmasks, self.grammar.size(1), timestep)
            self._launch(batch, None, batch.positions.tolist(), stream)
            if event is not None:
                event.record(stream)
        return self

    def step_weights(self, positions, indices: Tensor | None = None, generator=None, stream=None, event=None):
        """Post-verification noise step of the slots at `positions` (reference core/buffer.py:1054-1096)."""
        target = [self.flags.target_host[p] for p in positions]
        draft = [self.flags.draft_host[p] for p in positions]
        scoped = ScopedIndicators(target, draft)
        if scoped.has_stochastic_target:
            self.weights.step(positions=positions, scoped=scoped, indicator=self.flags.draft, indices=indices,
                              generator=generator, stream=stream, event=event)
        return self

    def _scoped(self, n, indicators, multiplicative, frequency, presence, biases, temperature, top_k, top_p, min_p,
                top_logprobs, bitmasks, greedy_drafts) -> ScopedIndicators:
        if indicators is None:
            return ScopedIndicators.from_params(n, multiplicative, frequency, presence, biases, temperature, top_k,
                                                top_p, min_p, top_logprobs, bitmasks, greedy_drafts)
        if isinstance(indicators, ScopedIndicators):
            return indicators
        if hasattr(indicators, "target") and hasattr(indicators, "draft"):
            return ScopedIndicators(indicators.target, indicators.draft)
        return ScopedIndicators.from_pairs(indicators)

    def slot_batch(self, positions, scoped, multiplicative, frequency, presence, biases, temperature, top_k, top_p,
                   min_p, top_logprobs, bitmasks, step, counts=None, encodings=None):
        """Host side of one allocate (`encodings`, grammar `step` 0) or update (`counts`, every
        step): the packed SlotBatch of the call. Needs no GPU."""
        from sonic_sampler_b200.core import population as pop

        batch = pop.new_batch(positions, self.bias.size(0), self.vocab_size)
        pop.pack_scalars(batch, temperature, top_p, min_p, multiplicative, frequency, presence, top_k, top_logprobs,
                         scoped.target, scoped.draft)
        if encodings is not None:
            pop.pack_histogram(batch, encodings)
        else:
            pop.pack_dense_counts(batch, counts, self.device)
        pop.pack_bias(batch, biases)
        pop.pack_grammar(batch, bitmasks, self.grammar.size(1), step)
        return batch

    def _launch(self, batch, scoped, positions, stream) -> None:
        pop = self._population()
        pop.launch_populate(self, batch, self._stager, stream)
        if scoped is not None:
            self.flags.update_host(scoped, positions)

    def update(self, counts, target_gumbel, multiplicative, frequency, presence, biases, temperature, top_k, top_p,
               min_p, top_logprobs, positions=None, indicators=None, greedy_drafts=False, prefill=False,
               bitmasks=None, stream=None, generator=None):
        """Rewrite the parameters, counts, bias rows, grammar rows and indicators of the slots at
        `positions` (all slots, in order, without) and refresh their noise (reference
        core/buffer.py:1139-1237). Returns an event recorded on `stream` when one is given."""
        event = torch.cuda.Event() if stream is not None else None
        pos = self._positions(positions, len(counts))
        scoped = self._scoped(len(counts), indicators, multiplicative, frequency, presence, biases, temperature, top_k,
                              top_p, min_p, top_logprobs, bitmasks, greedy_drafts)
        batch = self.slot_batch(pos, scoped, multiplicative, frequency, presence, biases, temperature, top_k, top_p,
                                min_p, top_logprobs, bitmasks, None, counts=counts)
        self._launch(batch, scoped, pos, stream)
        self.refresh_noise(scoped, positions, generator, prefill, target_gumbel, stream)
        if event is not None:
            event.record(stream)
        return event

    def allocate(self, encodings, multiplicative, frequency, presence, biases, temperature, top_k, top_p, min_p,
                 top_logprobs, positions, indicators=None, greedy_drafts=False, bitmasks=None, stream=None,
                 generator=None):
        """Admit requests into the slots at `positions`: parameters, the prompt histogram as context
        counts, zero decode counts, bias rows, step-0 grammar rows, indicators and prefill noise
        (reference core/buffer.py:1239-1352). Returns an event recorded on `stream` when given."""
        event = torch.cuda.Event() if stream is not None else None
        pos = [int(p) for p in positions]
        scoped = self._scoped(len(encodings), indicators, multiplicative, frequency, presence, biases, temperature,
                              top_k, top_p, min_p, top_logprobs, bitmasks, greedy_drafts)
        batch = self.slot_batch(pos, scoped, multiplicative, frequency, presence, biases, temperature, top_k, top_p,
                                min_p, top_logprobs, bitmasks, 0, encodings=encodings)
        self._launch(batch, scoped, pos, stream)
        self.refresh_noise(scoped, pos, generator, True, None, stream)
        if event is not None:
            event.record(stream)
        return event

    def refresh_noise(self, scoped: ScopedIndicators, positions, generator, prefill, target_gumbel=None,
                      stream=None) -> None:
        """The noise part of allocate / update (core/buffer.py:1221-1232, 1335-1345): only when a
        slot's target is stochastic, with the caller's generator(s), in the reference's order."""
        if scoped.has_stochastic_target:
            self.weights.update(generator=generator, selectors=scoped.stochastic_selectors, targets=target_gumbel,
                                positions=positions, prefill=prefill, stream=stream)

    def to(self, device) -> "SamplingBuffers":
        """Deep copy onto `device` (the packed flags keep their [B, 2] stride (1, B) layout)."""
        mv = lambda t: t.to(device).clone()  # noqa: E731
        return SamplingBuffers(
            grammar=mv(self.grammar),
            repetition=RepetitionPenalties(
                counts=TokenCounts(context=mv(self.repetition.counts.context),
                                   decode=mv(self.repetition.counts.decode)),
                frequency=mv(self.repetition.frequency),
                presence=mv(self.repetition.presence),
                multiplicative=mv(self.repetition.multiplicative),
            ),
            bias=mv(self.bias),
            temperature=mv(self.temperature),
            top_k=mv(self.top_k),
            top_p=mv(self.top_p),
            min_p=mv(self.min_p),
            top_logprobs=mv(self.top_logprobs),
            weights=StochasticWeights(uniform=mv(self.weights.uniform),
                                      gumbel=GumbelNoise(target=mv(self.weights.gumbel.target),
                                                         draft=mv(self.weights.gumbel.draft))),
            flags=Flags(packed=self.flags.packed.T.contiguous().to(device).T,
                        target_host=list(self.flags.target_host), draft_host=list(self.flags.draft_host)),
        )
