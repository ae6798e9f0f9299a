"""`UnshardedFusedSingular` (reference interface/singular.py:41-194): autoregressive decode
and drafting steps, same methods, arguments and defaults as the reference."""

from __future__ import annotations

from dataclasses import dataclass

from torch import Tensor

from sonic_sampler_b200 import ops
from sonic_sampler_b200._abi import MAX_K
from sonic_sampler_b200.base.sampler import DEFAULT_TOP_LOGPROBS, Selection
from sonic_sampler_b200.interface.base import TopKStrategy, TwoStageTiling, default_device
from sonic_sampler_b200.interface.dispatch import TwoStageWarpConfig
from sonic_sampler_b200.interface.functional.singular import fused_singular


def resolve_tokens(tokens: Tensor | None, timestep: int, in_place: bool) -> tuple[Tensor | None, Tensor | None]:
    output = drafted = None
    if tokens is not None:
        if in_place:
            output = tokens[:, timestep, None]
        if timestep:
            drafted = tokens
    return output, drafted


@dataclass
class UnshardedFusedSingular(TwoStageTiling):
    lookahead: int = 0
    max_top_logprobs: int = DEFAULT_TOP_LOGPROBS
    batch_size: int = 32

    @classmethod
    def initialize(cls, vocab_size: int, batch_size: int = 32, lookahead: int = 0, pdl: bool = True,
                   block_size: int | None = None, arch: int | None = None,
                   max_top_logprobs: int = DEFAULT_TOP_LOGPROBS) -> "UnshardedFusedSingular":
        dispatch, vocabulary, block_n = cls.resolve(vocab_size=vocab_size, k=MAX_K, top_logprobs=max_top_logprobs,
                                                    block_size=block_size, arch=arch, ensure_multiblock=True)
        rows = batch_size * (lookahead + 1)
        device = default_device()
        workspace = ops.new_workspace(ops.singular_workspace_bytes(rows, vocab_size), device)
        return cls(pdl=pdl, block_n=block_n, vocabulary=vocabulary, scratchpad=workspace, dispatch=dispatch,
                   lookahead=lookahead, max_top_logprobs=max_top_logprobs, batch_size=rows)

    def _workspace(self, rows: int, vocab: int) -> Tensor:
        need = ops.singular_workspace_bytes(rows, vocab)
        if self.scratchpad.numel() < need:
            self.scratchpad = ops.new_workspace(need, self.scratchpad.device)
        return self.scratchpad

    def autoregressive(self, logits: Tensor, buffers, prefill: bool = False, update_counts: bool = False,
                       logprobs: bool = False, slot_mapping: Tensor | None = None,
                       strategy: TopKStrategy | None = None,
                       tuning: TwoStageWarpConfig | None = None) -> Selection:
        counts = (penalties := buffers.repetition).counts
        config, k_strategy, block_n = self.tuning(logits.size(0), strategy, tuning)
        return fused_singular(
            logits=logits,
            indicators=buffers.flags.target,
            max_top_logprobs=self.max_top_logprobs,
            enable_pdl=self.pdl,
            is_prefill=prefill,
            update_counts=update_counts,
            return_logprobs=logprobs,
            block_n=block_n,
            scratchpad=self._workspace(logits.size(0), logits.size(1)),
            slot_mapping=slot_mapping,
            grammar=buffers.grammar[:, 0],
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
            gumbel_noise=buffers.weights.gumbel.target[:, 0],
            topk_strategy=k_strategy,
            warp_config=config,
        )

    def drafting(self, logits: Tensor, buffers, timestep: int = 0, tokens: Tensor | None = None,
                 probabilities: Tensor | None = None, slot_mapping: Tensor | None = None,
                 d2t_mapping: Tensor | None = None, target_vocab: int | None = None, in_place: bool = False,
                 strategy: TopKStrategy | None = None, tuning: TwoStageWarpConfig | None = None) -> Selection:
        counts = (penalties := buffers.repetition).counts
        config, k_strategy, block_n = self.tuning(logits.size(0), strategy, tuning)
        output_tokens, drafted_tokens = resolve_tokens(tokens, timestep, in_place)
        return_probabilities = not buffers.flags.all_greedy
        return fused_singular(
            logits=logits,
            indicators=buffers.flags.draft,
            lookahead=self.lookahead,
            target_vocab=target_vocab,
            enable_pdl=self.pdl,
            return_probabilities=return_probabilities,
            block_n=block_n,
            scratchpad=self._workspace(logits.size(0), logits.size(1)),
            slot_mapping=slot_mapping,
            d2t_mapping=d2t_mapping,
            grammar=buffers.grammar[:, timestep],
            context_counts=counts.context,
            decode_counts=counts.decode,
            drafted_tokens=drafted_tokens,
            repetition_penalties=penalties.multiplicative,
            frequency_penalties=penalties.frequency,
            presence_penalties=penalties.presence,
            logit_bias=buffers.bias,
            temperature=buffers.temperature,
            top_k=buffers.top_k,
            top_p=buffers.top_p,
            min_p=buffers.min_p,
            top_k_logprobs=buffers.top_logprobs,
            gumbel_noise=buffers.weights.gumbel.draft[:, timestep],
            output_tokens=output_tokens,
            draft_probabilities=probabilities,
            topk_strategy=k_strategy,
            warp_config=config,
        )
