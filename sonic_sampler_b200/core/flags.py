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


_GREEDY = int(Indicator.GREEDY)


def _indicator_bits(grammar, multiplicative, frequency, presence, logit_bias, temperature, top_k, top_p, min_p,
                    top_k_logprobs, greedy_draft) -> int:
    """Indicator.from_params as a plain int (the per-slot hot loop of a batch admission)."""
    greedy = top_k == 1
    bits = (bool(grammar) | (multiplicative != 1.0) << 1 | (frequency != 0.0) << 2 | (presence != 0.0) << 3
            | bool(logit_bias) << 4 | (temperature != 1.0) << 5 | greedy << 6 | (1 < top_k < MAX_K) << 7)
    if not greedy:
        bits |= (0.0 < top_p < 1.0) << 8 | (0.0 < min_p < 1.0) << 9 | (0 < top_k_logprobs <= MAX_K) << 10
        bits |= bool(greedy_draft) << 11
    return int(bits)


class ScopedIndicators:
    """Target and draft indicators of a list of slots (reference core/flags.py:229-432)."""

    def __init__(self, target: list, draft: list):
        # plain ints with the Indicator bit values (Indicator is an int subclass)
        self.target = [int(v) for v in target]
        self.draft = [int(v) for v in draft]

    @classmethod
    def from_pairs(cls, pairs) -> "ScopedIndicators":
        pairs = list(pairs)
        return cls([t for t, _ in pairs], [d for _, d in pairs])

    @classmethod
    def from_params(cls, size: int, multiplicative=None, frequency=None, presence=None, biases=None,
                    temperature=None, top_k=None, top_p=None, min_p=None, top_logprobs=None, bitmasks=None,
                    greedy_drafts=False) -> "ScopedIndicators":
        """Same resolution as the reference (core/flags.py:310-362), defaults included: a missing
        or empty `temperature` list counts as 0.0 (which sets the temperature bit), and a bias
        dict or bitmask that is not None sets its bit even when empty."""
        if top_k and any(k > MAX_K for k in top_k):
            raise ValueError(f"`top_k` greater than {MAX_K} is not supported")
        fill = lambda v: [v] * size  # noqa: E731
        drafter = list(greedy_drafts) if isinstance(greedy_drafts, list) else fill(greedy_drafts)
        rows = zip(
            [m is not None for m in bitmasks] if bitmasks else fill(False),
            multiplicative or fill(1.0),
            frequency or fill(0.0),
            presence or fill(0.0),
            [b is not None for b in biases] if biases else fill(False),
            temperature or fill(0.0),
            top_k or fill(MAX_K),
            top_p or fill(1.0),
            min_p or fill(0.0),
            top_logprobs or fill(0),
            drafter,
        )
        target = [_indicator_bits(*r) for r in rows]
        greedy_mask = int(Indicator.all() ^ Indicator.stochastic() ^ Indicator.TOP_K_LOGPROBS
                          ^ Indicator.STOCHASTIC_VERIFY_GREEDY_DRAFT)
        no_top_z = int(Indicator.all() ^ Indicator.TOP_K_LOGPROBS)
        draft = [((t & greedy_mask) | int(Indicator.GREEDY)) if g else (t & no_top_z) for g, t in zip(drafter, target)]
        return cls(target, draft)

    @property
    def has_stochastic_target(self) -> bool:
        return any(not (v & _GREEDY) for v in self.target)

    @property
    def has_stochastic_draft(self) -> bool:
        return any(not (v & _GREEDY) for v in self.draft)

    @property
    def stochastic_selectors(self) -> list[tuple[bool, bool]]:
        return [(not (t & _GREEDY), not (d & _GREEDY)) for t, d in zip(self.target, self.draft)]

    def subset(self, indices) -> "ScopedIndicators":
        return ScopedIndicators([self.target[i] for i in indices], [self.draft[i] for i in indices])
