"""Tiling resolution shared by the modular interface classes (reference interface/base.py:17-276).

Keeps the reference's constructor contract (same arguments, same ValueError messages) and
its `block_n` resolution. What each instance owns differs: instead of the reference's u32
tile scratchpad it owns one zero-filled workspace for the fused B200 kernel, sized at
initialization, so calls never allocate workspace memory.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from sonic_sampler_b200._abi import MAX_K
from sonic_sampler_b200.base.sampler import DEFAULT_TOP_LOGPROBS
from sonic_sampler_b200.interface.dispatch import (
    DispatchSummary,
    RuntimeConfig,
    Strategy,
    TwoStageWarpConfig,
    VocabBucket,
)

FP32 = torch.float32
BF16 = torch.bfloat16
I32 = torch.int32
U32 = torch.uint32


def cdiv(a: int, b: int) -> int:
    return -(-a // b)


@dataclass(frozen=True)
class Vocabulary:
    size: int
    blocks: int

    @classmethod
    def resolve(cls, size: int, block_n: int) -> "Vocabulary":
        return cls(size=size, blocks=cdiv(size, block_n))

    def evolve(self, block_n: int) -> "Vocabulary":
        return Vocabulary(size=self.size, blocks=cdiv(self.size, block_n))


@dataclass(frozen=True)
class TopKStrategy:
    """Reference top-k strategy knob (interface/base.py:63-118). Accepted for API parity; the
    B200 kernels always compute the exact top-128, which all reference strategies produce."""

    radix: bool = False
    sparse: bool = False
    scale: int = 4

    @classmethod
    def adaptive(cls, scale: int = 4) -> "TopKStrategy":
        return cls(radix=True, sparse=True, scale=scale)

    @classmethod
    def resolve(cls, config: RuntimeConfig) -> "TopKStrategy":
        return {"bitonic": cls(), "radix": cls(radix=True), "adaptive": cls.adaptive()}[config.strategy]

    @property
    def key(self) -> Strategy:
        if self.radix:
            return "adaptive" if self.sparse else "radix"
        return "bitonic"

    @property
    def is_adaptive(self) -> bool:
        return self.radix and self.sparse

    @property
    def is_alternating(self) -> bool:
        return not self.radix

    @property
    def inverse(self) -> float | None:
        return 1 / self.scale if self.is_adaptive else None


def resolve_dispatch(k: int, vocab_size: int, block_size: int | None, arch: int | None) -> tuple[VocabBucket | None, int]:
    if k > MAX_K:
        raise ValueError(f"maximum supported top-k value is {MAX_K}, got {k} instead")
    elif int.bit_count(k) > 1:
        raise ValueError(f"top-k value must be a power of 2, got {k} instead")
    elif block_size is None:
        if (dispatch := DispatchSummary.load(k=k, arch=arch)) is None:
            raise ValueError("unable to resolve dispatch summary for given top-k and architecture")
        elif (bucket := dispatch.get_vocab(vocab_size)) is None:
            raise ValueError("unable to match tuning configuration for given vocabulary size")
        return bucket, bucket.block_n
    return None, block_size


def default_device() -> torch.device:
    """Device of the owned buffers: the current CUDA device (the reference allocates on the
    default device, interface/base.py:224-231)."""
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


@dataclass
class TwoStageTiling:
    pdl: bool
    block_n: int
    vocabulary: Vocabulary
    # zero-filled workspace of the fused kernel (name kept from the reference)
    scratchpad: Tensor
    dispatch: VocabBucket | None

    @classmethod
    def resolve(cls, vocab_size: int, k: int = MAX_K, top_logprobs: int = DEFAULT_TOP_LOGPROBS,
                block_size: int | None = None, arch: int | None = None,
                ensure_multiblock: bool = True) -> tuple[VocabBucket | None, Vocabulary, int]:
        dispatch, block_n = resolve_dispatch(k, vocab_size, block_size, arch)
        vocabulary = Vocabulary.resolve(vocab_size, block_n)
        if ensure_multiblock and (blocks := vocabulary.blocks) <= 1:
            raise ValueError(f"total vocab blocks must be greater than 1, got {blocks} instead")
        elif top_logprobs < 0 or top_logprobs > MAX_K:
            raise ValueError(f"top logprobs must be within the interval [0, {MAX_K}]")
        if block_n & (block_n - 1) or not 256 <= block_n <= 65536:
            raise ValueError(f"block size must be a power of 2 in [256, 65536], got {block_n}")
        if vocab_size < MAX_K:
            raise ValueError(f"vocab size must be at least {MAX_K}, got {vocab_size}")
        return dispatch, vocabulary, block_n

    def device_error(self) -> int:
        """Read and clear the device error word of this object's workspace: 0 when every call
        since the last read completed, else SONIC_DEVICE_ERR_* bits (a bounded wait gave up and
        the affected rows wrote no outputs). Synchronises the current stream; an addition of
        this library (the reference has no device-side error path)."""
        from sonic_sampler_b200 import ops

        return ops.workspace_error(self.scratchpad)

    def tuning(self, size: int, strategy: TopKStrategy | None = None,
               tuning: TwoStageWarpConfig | None = None) -> tuple[TwoStageWarpConfig, TopKStrategy, int]:
        """Same resolution as the reference (interface/base.py:243-276)."""
        block_size = self.block_n
        k_strategy = strategy
        config = tuning
        if config is None and self.dispatch and (bucket := self.dispatch.get_batch(size)):
            if strategy:
                target = bucket.get(strategy.key)
                config, block_size = target.warp_config, target.block_n
            else:
                best = bucket.best
                config, k_strategy, block_size = best.warp_config, TopKStrategy.resolve(best), best.block_n
        return config or TwoStageWarpConfig.default(), k_strategy or TopKStrategy(), block_size
