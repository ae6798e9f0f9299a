"""Tile-size dispatch of the reference interface (reference interface/dispatch.py:65-268).

The B200 kernels pick their own launch shape, so the warp counts here have no effect on
them. The tile width `block_n` still matters for one observable: the reference's greedy
selection breaks ties between equal maxima by the smallest offset inside a `block_n` tile
(ops/prologue.py:117-138, ops/singular.py:71-131). To reproduce the reference bit for bit,
`block_n` is resolved exactly as the reference resolves it, from the same tuned table
(reference resources/dispatch/sm{90,100}_k128.toml, reproduced below as data:
vocab bucket -> batch bucket -> priority-ordered (strategy, block_n, first_warps,
second_warps)).
"""

from __future__ import annotations

from bisect import bisect_left
from dataclasses import dataclass
from typing import Literal

from sonic_sampler_b200._abi import MAX_K

Strategy = Literal["bitonic", "adaptive", "radix"]


def next_power_of_2(value: int) -> int:
    """Reference ops/base.py:27-31 (note: 0 maps to 0 and 1 to 1)."""
    return (1 << int.bit_length(value)) if int.bit_count(value) > 1 else value


@dataclass(frozen=True)
class TwoStageWarpConfig:
    first: int
    second: int

    @classmethod
    def default(cls) -> "TwoStageWarpConfig":
        return cls(first=16, second=8)


@dataclass(frozen=True)
class ThreeStageWarpConfig(TwoStageWarpConfig):
    third: int = 4

    @property
    def two_stage(self) -> TwoStageWarpConfig:
        return TwoStageWarpConfig(first=self.first, second=self.second)

    @classmethod
    def from_config(cls, config: TwoStageWarpConfig, third: int | None = None, gamma: int = 3) -> "ThreeStageWarpConfig":
        return cls(first=config.first, second=config.second, third=third or next_power_of_2(gamma + 1))

    @classmethod
    def default(cls, gamma: int = 3) -> "ThreeStageWarpConfig":  # type: ignore[override]
        return cls.from_config(TwoStageWarpConfig.default(), gamma=gamma)


@dataclass(frozen=True)
class RuntimeConfig:
    priority: int
    block_n: int
    strategy: Strategy
    first_warps: int
    second_warps: int

    @property
    def warp_config(self) -> TwoStageWarpConfig:
        return TwoStageWarpConfig(first=self.first_warps, second=self.second_warps)


@dataclass(frozen=True)
class BatchBucket:
    size: int
    config: tuple[RuntimeConfig, ...]

    @property
    def best(self) -> RuntimeConfig:
        return self.config[0]

    def get(self, strategy: Strategy) -> RuntimeConfig:
        for c in self.config:
            if c.strategy == strategy:
                return c
        raise KeyError(strategy)


def _bucket_get(buckets, size: int, margin: float = 0.5):
    """First bucket with size >= `size`, else the last one within +50 % (dispatch.py:130-142)."""
    sizes = [b.size for b in buckets]
    i = bisect_left(sizes, size)
    if i < len(buckets):
        return buckets[i]
    if buckets and size < buckets[-1].size * (1 + margin):
        return buckets[-1]
    return None


@dataclass(frozen=True)
class VocabBucket:
    size: int
    batch: tuple[BatchBucket, ...]

    @property
    def block_n(self) -> int:
        return min(c.block_n for b in self.batch for c in b.config)

    def get_batch(self, size: int) -> BatchBucket | None:
        return _bucket_get(self.batch, size)


_B = "bitonic"
_A = "adaptive"
_R = "radix"

# (vocab bucket, ((batch bucket, ((strategy, block_n, first_warps, second_warps), ...)), ...))
_SM100 = (
    (8192, ((1, ((_B, 1024, 4, 4), (_A, 1024, 8, 8), (_R, 1024, 4, 8))),
            (2, ((_B, 1024, 4, 4), (_A, 2048, 8, 4), (_R, 1024, 4, 8))),
            (4, ((_B, 1024, 4, 4), (_A, 2048, 8, 4), (_R, 1024, 4, 8))),
            (8, ((_B, 1024, 4, 4), (_A, 2048, 8, 4), (_R, 1024, 4, 8))),
            (16, ((_B, 1024, 4, 4), (_A, 2048, 8, 4), (_R, 1024, 4, 8))),
            (32, ((_B, 2048, 8, 4), (_A, 2048, 8, 4), (_R, 2048, 8, 4))))),
    (16384, ((1, ((_B, 1024, 4, 16), (_A, 2048, 8, 8), (_R, 2048, 8, 8))),
             (2, ((_B, 1024, 4, 16), (_A, 2048, 8, 8), (_R, 2048, 8, 8))),
             (4, ((_B, 1024, 4, 16), (_A, 2048, 8, 8), (_R, 2048, 8, 8))),
             (8, ((_B, 1024, 4, 16), (_A, 2048, 8, 8), (_R, 2048, 8, 8))),
             (16, ((_B, 2048, 8, 4), (_A, 2048, 8, 8), (_R, 2048, 8, 8))),
             (32, ((_B, 4096, 8, 4), (_A, 4096, 16, 4), (_R, 4096, 8, 4))))),
    (32768, ((1, ((_B, 2048, 8, 16), (_A, 4096, 16, 8), (_R, 2048, 8, 16))),
             (2, ((_B, 2048, 8, 16), (_A, 4096, 16, 8), (_R, 2048, 8, 16))),
             (4, ((_B, 2048, 8, 16), (_A, 4096, 16, 8), (_R, 2048, 8, 16))),
             (8, ((_B, 2048, 8, 16), (_A, 4096, 16, 8), (_R, 2048, 8, 16))),
             (16, ((_B, 4096, 8, 4), (_A, 4096, 16, 8), (_R, 4096, 8, 8))),
             (32, ((_A, 8192, 8, 4), (_B, 4096, 8, 4), (_R, 8192, 8, 4))))),
    (65536, ((1, ((_B, 4096, 8, 16), (_A, 4096, 16, 16), (_R, 4096, 8, 16))),
             (2, ((_B, 4096, 8, 16), (_A, 4096, 16, 16), (_R, 4096, 8, 16))),
             (4, ((_B, 4096, 8, 16), (_A, 4096, 16, 16), (_R, 4096, 8, 16))),
             (8, ((_B, 4096, 8, 16), (_A, 4096, 16, 16), (_R, 4096, 8, 16))),
             (16, ((_A, 8192, 8, 8), (_B, 4096, 8, 16), (_R, 8192, 8, 8))),
             (32, ((_B, 4096, 8, 16), (_A, 16384, 16, 4), (_R, 16384, 16, 4))))),
    (131072, ((1, ((_B, 4096, 8, 16), (_A, 8192, 8, 16), (_R, 4096, 8, 32))),
              (2, ((_B, 4096, 8, 16), (_A, 8192, 8, 16), (_R, 4096, 8, 32))),
              (4, ((_B, 4096, 8, 16), (_A, 8192, 8, 16), (_R, 4096, 8, 32))),
              (8, ((_A, 8192, 8, 16), (_B, 8192, 16, 16), (_R, 8192, 8, 16))),
              (16, ((_A, 16384, 16, 8), (_B, 4096, 8, 16), (_R, 16384, 16, 8))),
              (32, ((_B, 4096, 8, 16), (_A, 16384, 16, 8), (_R, 16384, 16, 8))))),
    (262144, ((1, ((_B, 4096, 8, 32), (_A, 8192, 8, 32), (_R, 8192, 8, 32))),
              (2, ((_B, 4096, 8, 32), (_A, 8192, 8, 32), (_R, 8192, 8, 32))),
              (4, ((_B, 8192, 16, 16), (_A, 8192, 8, 32), (_R, 8192, 8, 32))),
              (8, ((_A, 16384, 16, 16), (_B, 16384, 32, 16), (_R, 16384, 16, 16))),
              (16, ((_B, 4096, 8, 32), (_A, 16384, 16, 16), (_R, 16384, 16, 16))),
              (32, ((_B, 4096, 8, 32), (_A, 8192, 8, 32), (_R, 16384, 16, 16))))),
)

# sm90 differs from sm100 only in these buckets
_SM90_DIFF = {
    (65536, 32): ((_A, 16384, 16, 4), (_B, 4096, 8, 16), (_R, 16384, 16, 4)),
    (262144, 4): ((_A, 8192, 8, 32), (_B, 8192, 16, 16), (_R, 8192, 8, 32)),
    (262144, 16): ((_A, 16384, 16, 16), (_B, 4096, 8, 32), (_R, 16384, 16, 16)),
    (262144, 32): ((_A, 8192, 8, 32), (_B, 4096, 8, 32), (_R, 16384, 16, 16)),
}


def _table(rows, diff=None) -> tuple[VocabBucket, ...]:
    out = []
    for vsize, batches in rows:
        bb = []
        for bsize, cfgs in batches:
            cfgs = (diff or {}).get((vsize, bsize), cfgs)
            bb.append(BatchBucket(bsize, tuple(RuntimeConfig(i, bn, s, f, w) for i, (s, bn, f, w) in enumerate(cfgs))))
        out.append(VocabBucket(vsize, tuple(bb)))
    return tuple(out)


_TABLES = {100: _table(_SM100), 90: _table(_SM100, _SM90_DIFF)}


@dataclass(frozen=True)
class DispatchSummary:
    k: int
    vocab: tuple[VocabBucket, ...]

    def get_vocab(self, size: int) -> VocabBucket | None:
        return _bucket_get(self.vocab, size)

    @classmethod
    def load(cls, k: int = MAX_K, arch: int | None = None) -> "DispatchSummary | None":
        if arch is None:
            arch = current_arch()
        if k != MAX_K or arch not in _TABLES:
            return None
        return cls(k=k, vocab=_TABLES[arch])


def current_arch() -> int:
    import torch

    if torch.cuda.is_available():
        major, minor = torch.cuda.get_device_capability()
        return major * 10 + minor
    return 100
