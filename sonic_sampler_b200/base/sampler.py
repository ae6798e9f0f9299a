"""Output containers of the sampler (reference base/sampler.py:35-199).

Same field names, shapes and dtypes as the reference: int32 tokens, bf16 logprobs.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Final

import torch
from torch import Tensor

DEFAULT_TOP_LOGPROBS: Final[int] = 5

I32 = torch.int32
BF16 = torch.bfloat16


@dataclass
class TopTargets:
    # top-k tokens with shape [B, Z] or [B, gamma + 1, Z]
    tokens: Tensor
    # their log-probabilities, same shape
    logprobs: Tensor

    @classmethod
    def empty_blocked(cls, batch_size: int, targets: int, timesteps: int = 1, device=None,
                      dtype: torch.dtype = BF16) -> "TopTargets | None":
        if targets > 0:
            shape = (batch_size, timesteps, targets) if timesteps > 1 else (batch_size, targets)
            return cls(tokens=torch.empty(shape, dtype=I32, device=device),
                       logprobs=torch.empty(shape, dtype=dtype, device=device))
        return None

    @classmethod
    def empty_varlen(cls, num_tokens: int, targets: int, device=None, dtype: torch.dtype = BF16) -> "TopTargets | None":
        if targets > 0:
            return cls(tokens=torch.empty(num_tokens, targets, dtype=I32, device=device),
                       logprobs=torch.empty(num_tokens, targets, dtype=dtype, device=device))
        return None


@dataclass
class LogProbabilities:
    # selected-token log-probabilities, [B, 1] or [B, gamma + 1]
    selected: Tensor
    top_k: TopTargets | None = None

    @classmethod
    def empty_blocked(cls, batch_size: int, timesteps: int = 1, top_k: int = 0, device=None,
                      dtype: torch.dtype = BF16) -> "LogProbabilities":
        return cls(selected=torch.empty(batch_size, timesteps, dtype=dtype, device=device),
                   top_k=TopTargets.empty_blocked(batch_size, top_k, timesteps, device=device, dtype=dtype))

    @classmethod
    def empty_varlen(cls, num_tokens: int, top_k: int = 0, device=None, dtype: torch.dtype = BF16) -> "LogProbabilities":
        return cls(selected=torch.empty(num_tokens, dtype=dtype, device=device),
                   top_k=TopTargets.empty_varlen(num_tokens, top_k, device=device, dtype=dtype))


@dataclass
class Selection:
    # selected next tokens, [B, 1] int32
    tokens: Tensor
    # candidate probabilities scattered into [slots, V_t] (drafting)
    probabilities: Tensor | None = None
    logprobs: LogProbabilities | None = None

    @classmethod
    def from_buffers(cls, tokens: Tensor, probabilities: Tensor | None = None, logprobs: bool = False,
                     top_logprobs: int = 0, dtype: torch.dtype = BF16) -> "Selection":
        lp = None
        if logprobs:
            lp = LogProbabilities.empty_blocked(tokens.size(0), top_k=top_logprobs, device=tokens.device, dtype=dtype)
        return cls(tokens=tokens, probabilities=probabilities, logprobs=lp)

    @classmethod
    def empty(cls, batch_size: int, vocab_size: int, device: torch.device, probs: bool = False,
              logprobs: bool = False, top_logprobs: int = 0) -> "Selection":
        tokens = torch.empty((batch_size, 1), dtype=I32, device=device)
        pb = torch.empty((batch_size, vocab_size), dtype=BF16, device=device) if probs else None
        lp = LogProbabilities.empty_blocked(batch_size, top_k=top_logprobs, device=device) if logprobs else None
        return cls(tokens=tokens, probabilities=pb, logprobs=lp)


@dataclass
class Verification:
    # drafted tokens with the accepted prefix + next token written in place, [B, gamma + 1]
    tokens: Tensor
    # accepted draft count per request, [B, 1] int32
    offsets: Tensor
    logprobs: LogProbabilities | None = None

    @classmethod
    def from_tokens(cls, tokens: Tensor, batch_size: int, timesteps: int, logprobs: bool = False,
                    varlen: bool = False, top_logprobs: int = 0, dtype: torch.dtype = BF16) -> "Verification":
        offsets = torch.empty(batch_size, 1, dtype=I32, device=tokens.device)
        lp = None
        if logprobs:
            if varlen:
                lp = LogProbabilities.empty_varlen(tokens.size(0), top_k=top_logprobs, device=tokens.device,
                                                   dtype=dtype)
            else:
                lp = LogProbabilities.empty_blocked(batch_size, timesteps=timesteps, top_k=top_logprobs,
                                                    device=tokens.device, dtype=dtype)
        return cls(tokens=tokens, offsets=offsets, logprobs=lp)
