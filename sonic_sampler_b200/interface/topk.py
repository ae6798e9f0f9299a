"""`UnshardedBoundedTopK` (reference interface/topk.py:38-161): exact top-k per row, values
descending, ties to the lowest column.

Kept from the reference on purpose: the values buffer is bf16 [batch_size, 128] and row r's
k results sit at flat offset r*k of the buffers (reference ops/topk/unpack.py:374-377 stores
with max_k = k), so for k < 128 read them as `values.view(-1)[:rows*k].view(rows, k)`.
fp32 logits (which the reference rejects) are accepted: the selection then runs on fp32
values and returns them in an fp32 buffer of the same layout.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from sonic_sampler_b200 import ops
from sonic_sampler_b200._abi import FLAG_PDL, MAX_K
from sonic_sampler_b200.interface.base import TopKStrategy, TwoStageTiling, default_device
from sonic_sampler_b200.interface.dispatch import TwoStageWarpConfig
from sonic_sampler_b200.interface.functional.base import collapse_2d

BF16 = torch.bfloat16
I32 = torch.int32


@dataclass
class UnshardedBoundedTopK(TwoStageTiling):
    k: int = MAX_K
    values: Tensor | None = None
    indices: Tensor | None = None
    values_f32: Tensor | None = None

    @classmethod
    def initialize(cls, vocab_size: int, block_size: int | None = None, batch_size: int = 32, k: int = MAX_K,
                   pdl: bool = True, arch: int | None = None) -> "UnshardedBoundedTopK":
        dispatch, vocabulary, block_n = cls.resolve(vocab_size=vocab_size, k=MAX_K, block_size=block_size,
                                                    arch=arch, ensure_multiblock=True)
        if k > MAX_K:
            raise ValueError(f"maximum supported top-k value is {MAX_K}, got {k} instead")
        if int.bit_count(k) > 1:
            raise ValueError(f"top-k value must be a power of 2, got {k} instead")
        device = default_device()
        workspace = ops.new_workspace(ops.topk_workspace_bytes(batch_size, vocab_size), device)
        return cls(pdl=pdl, block_n=block_n, vocabulary=vocabulary, scratchpad=workspace, dispatch=dispatch, k=k,
                   values=torch.empty(batch_size, MAX_K, dtype=BF16, device=device),
                   indices=torch.empty(batch_size, MAX_K, dtype=I32, device=device))

    def clear(self) -> "UnshardedBoundedTopK":
        """Reset the output buffers between consecutive correctness checks (the workspace
        already returns to its zero state after every call)."""
        self.values.fill_(-float("inf"))
        self.indices.fill_(-1)
        if self.values_f32 is not None:
            self.values_f32.fill_(-float("inf"))
        return self

    def __call__(self, logits: Tensor, *, strategy: TopKStrategy | None = None,
                 tuning: TwoStageWarpConfig | None = None) -> tuple[Tensor, Tensor]:
        ops._require_cuda(logits)
        *batch_step, _ = logits.shape
        flat = collapse_2d(logits)
        n_rows = flat.size(0)
        _, _, block_n = self.tuning(n_rows, strategy, tuning)
        if n_rows > self.values.size(0):
            raise ValueError(f"{n_rows} rows exceed the initialized batch size {self.values.size(0)}")
        need = ops.topk_workspace_bytes(n_rows, self.vocabulary.size)
        if self.scratchpad.numel() < need:
            self.scratchpad = ops.new_workspace(need, self.scratchpad.device)
        values = self.values
        if flat.dtype == torch.float32:
            if self.values_f32 is None:
                self.values_f32 = torch.empty(self.values.shape, dtype=torch.float32, device=self.values.device)
            values = self.values_f32
        args = ops.topk_args(flat, vocab_size=self.vocabulary.size, k=self.k, block_n=block_n, values=values,
                             indices=self.indices, flags=FLAG_PDL if self.pdl else 0, workspace=self.scratchpad)
        ops.launch_topk(args, flat.device)
        return values[:n_rows].unflatten(0, batch_step), self.indices[:n_rows].unflatten(0, batch_step)
