"""Per-request indicator bits (reference core/flags.py:58-221).

The sampler kernels read one u16 indicator per request slot. The bit layout is the
reference's contract with the inference engine, so it is kept as is.
"""

from __future__ import annotations

from enum import IntFlag, unique

import torch

MAX_K = 128


@unique
class Indicator(IntFlag):
    GRAMMAR = 0x1
    MULTIPLICATIVE = 0x2
    FREQUENCY = 0x4
    PRESENCE = 0x8
    BIAS = 0x10
    TEMPERATURE = 0x20
    GREEDY = 0x40
    TOP_K = 0x80
    TOP_P = 0x100
    MIN_P = 0x200
    TOP_K_LOGPROBS = 0x400
    STOCHASTIC_VERIFY_GREEDY_DRAFT = 0x800

    @classmethod
    def all(cls) -> "Indicator":
        return cls(0xFFF)

    @classmethod
    def stochastic(cls) -> "Indicator":
        return cls.TEMPERATURE | cls.TOP_K | cls.TOP_P | cls.MIN_P

    @classmethod
    def maximal(cls) -> "Indicator":
        return cls.all() ^ cls.GREEDY

    @classmethod
    def default(cls) -> "Indicator":
        return cls(0)

    @classmethod
    def repetition(cls) -> "Indicator":
        return cls.MULTIPLICATIVE | cls.FREQUENCY | cls.PRESENCE

    @classmethod
    def cumulative(cls) -> "Indicator":
        return cls.TOP_K | cls.TOP_P | cls.MIN_P

    @classmethod
    def from_params(
        cls,
        grammar: bool = False,
        multiplicative: float = 1.0,
        frequency: float = 0.0,
        presence: float = 0.0,
        logit_bias: bool = False,
        temperature: float = 1.0,
        top_k: int = MAX_K,
        top_p: float = 1.0,
        min_p: float = 0.0,
        top_k_logprobs: int = 0,
        greedy_draft: bool = False,
    ) -> "Indicator":
        """Same resolution as the reference (core/flags.py:150-184)."""
        greedy = top_k == 1
        bits = [
            grammar,
            multiplicative != 1.0,
            frequency != 0.0,
            presence != 0.0,
            logit_bias,
            temperature != 1.0,
            greedy,
            1 < top_k < MAX_K,
            not greedy and (0.0 < top_p < 1.0),
            not greedy and (0.0 < min_p < 1.0),
            not greedy and (0 < top_k_logprobs <= MAX_K),
            not greedy and greedy_draft,
        ]
        return cls(sum(int(b) << i for i, b in enumerate(bits)))

    def greedy(self) -> "Indicator":
        mask = Indicator.all() ^ Indicator.stochastic() ^ Indicator.TOP_K_LOGPROBS ^ Indicator.STOCHASTIC_VERIFY_GREEDY_DRAFT
        return (self & mask) | Indicator.GREEDY

    def disable(self, value: "Indicator") -> "Indicator":
        return self & (Indicator.all() ^ value)


def indicator_tensor(values, device=None) -> torch.Tensor:
    """u16 indicator vector from a list of Indicator / ints."""
    return torch.tensor([int(v) for v in values], dtype=torch.uint16, device=device)
