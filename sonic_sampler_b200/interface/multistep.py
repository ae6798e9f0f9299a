"""`UnshardedFusedMultistep` (reference interface/multistep.py:27-161): target verification
of gamma drafted tokens, same methods, arguments and defaults as the reference."""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from sonic_sampler_b200 import ops
from sonic_sampler_b200._abi import MAX_K
from sonic_sampler_b200.base.sampler import DEFAULT_TOP_LOGPROBS, Verification
from sonic_sampler_b200.interface.base import TopKStrategy, TwoStageTiling, default_device
from sonic_sampler_b200.interface.dispatch import ThreeStageWarpConfig
from sonic_sampler_b200.interface.functional.base import collapse_2d
from sonic_sampler_b200.interface.functional.multistep import fused_multistep


@dataclass
class UnshardedFusedMultistep(TwoStageTiling):
    lookahead: int = 1
    max_top_logprobs: int = DEFAULT_TOP_LOGPROBS
    # fp32 [B * (gamma + 1), 128] candidate probabilities and int32 candidate ids
    values: Tensor | None = None
    indices: Tensor | None = None

    @classmethod
    def initialize(cls, vocab_size: int, lookahead: int, batch_size: int = 32, pdl: bool = True,
                   block_size: int | None = None, arch: int | None = None,
                   max_top_logprobs: int = DEFAULT_TOP_LOGPROBS) -> "UnshardedFusedMultistep":
        dispatch, vocabulary, block_n = cls.resolve(vocab_size=vocab_size, k=MAX_K, top_logprobs=max_top_logprobs,
                                                    block_size=block_size, arch=arch, ensure_multiblock=True)
        rows = batch_size * (lookahead + 1)
        device = default_device()
        workspace = ops.new_workspace(ops.multistep_workspace_bytes(batch_size, lookahead, vocab_size, rows), device)
        return cls(pdl=pdl, block_n=block_n, vocabulary=vocabulary, scratchpad=workspace, dispatch=dispatch,
                   lookahead=lookahead, max_top_logprobs=max_top_logprobs,
                   values=torch.empty(rows, MAX_K, dtype=torch.float32, device=device),
                   indices=torch.empty(rows, MAX_K, dtype=torch.int32, device=device))

    def tuning(self, size: int, strategy: TopKStrategy | None = None,  # type: ignore[override]
               tuning: ThreeStageWarpConfig | None = None) -> tuple[ThreeStageWarpConfig, TopKStrategy, int]:
        config, k_strategy, block_n = super().tuning(size, strategy, tuning and tuning.two_stage)
        config = ThreeStageWarpConfig.from_config(config=config, third=tuning and tuning.third, gamma=self.lookahead)
        return config, k_strategy, block_n

    def __call__(self, logits: Tensor, tokens: Tensor, buffers, probabilities: Tensor | None = None,
                 slot_mapping: Tensor | None = None, update_counts: bool = False, logprobs: bool = False,
                 in_place: bool = False, strategy: TopKStrategy | None = None,
                 tuning: ThreeStageWarpConfig | None = None) -> Verification:
        counts = (penalties := buffers.repetition).counts
        rows = collapse_2d(logits).size(0)
        config, k_strategy, _ = self.tuning(rows, strategy, tuning)
        need = ops.multistep_workspace_bytes(rows // (self.lookahead + 1), self.lookahead, logits.size(-1), rows)
        if self.scratchpad.numel() < need:
            self.scratchpad = ops.new_workspace(need, self.scratchpad.device)
        values, indices = self.values, self.indices
        if values is None or values.size(0) < rows:
            values = self.values = logits.new_empty((rows, MAX_K), dtype=torch.float32)
            indices = self.indices = logits.new_empty((rows, MAX_K), dtype=torch.int32)
        return fused_multistep(
            logits=logits,
            indicators=buffers.flags.target,
            drafted_tokens=tokens,
            lookahead=self.lookahead,
            max_top_logprobs=self.max_top_logprobs,
            enable_pdl=self.pdl,
            update_counts=update_counts,
            return_logprobs=logprobs,
            # the reference passes the untuned block size here (interface/multistep.py:127,138)
            block_n=self.block_n,
            scratchpad=self.scratchpad,
            values=values,
            indices=indices,
            draft_probabilities=probabilities,
            slot_mapping=slot_mapping,
            grammar=buffers.grammar,
            context_counts=counts.context,
            decode_counts=counts.decode,
            repetition_penalties=penalties.multiplicative,
            frequency_penalties=penalties.frequency,
            presence_penalties=penalties.presence,
            logit_bias=buffers.bias,
            temperature=buffers.temperature,
            top_k=buffers.top_k,
            top_p=buffers.top_p,
            min_p=buffers.min_p,
            top_k_logprobs=buffers.top_logprobs,
            gumbel_noise=(weights := buffers.weights).gumbel.target,
            uniform_noise=weights.uniform,
            output_tokens=tokens if in_place else None,
            topk_strategy=k_strategy,
            warp_config=config,
        )
