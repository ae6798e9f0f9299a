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

Host population (pinned staging, per-slot updates) is the engine's business and out of
scope here.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Sequence

import torch
from torch import Tensor

from sonic_sampler_b200.core.flags import MAX_K, Indicator

BF16 = torch.bfloat16
I32 = torch.int32
U16 = torch.uint16
U32 = torch.uint32


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

        with (torch.cuda.stream(stream) if stream is not None else nullcontext()):
            indexed_copy(self.draft, self.target, indices, indicator)
        return self


@dataclass
class StochasticWeights:
    uniform: Tensor
    gumbel: GumbelNoise


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
