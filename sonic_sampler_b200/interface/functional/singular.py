"""`fused_singular`: one-token selection per row (reference interface/functional/singular.py:75-322).

Same keyword set and defaults as the reference; the two Triton launches become one launch
of the fused B200 kernel through the C ABI (`sonic_fused_singular`). Two additions, both
off by default: `philox_seed` / `philox_offset` select counter-based in-kernel Gumbel noise
instead of the `gumbel_noise` buffer.
"""

from __future__ import annotations

import torch
from torch import Tensor

from sonic_sampler_b200 import ops
from sonic_sampler_b200._abi import (
    FLAG_LOGPROBS,
    FLAG_PDL,
    FLAG_PHILOX,
    FLAG_PREFILL,
    FLAG_PROBABILITIES,
    FLAG_UPDATE_COUNTS,
)
from sonic_sampler_b200.base.sampler import DEFAULT_TOP_LOGPROBS, Selection
from sonic_sampler_b200.interface.base import TopKStrategy
from sonic_sampler_b200.interface.dispatch import TwoStageWarpConfig
from sonic_sampler_b200.interface.functional.base import (
    I32,
    resolve_workspace,
    validate_count_update,
)


def resolve_gumbel(noise: Tensor | None, logits: Tensor) -> Tensor:
    if (weights := noise) is None:
        weights = torch.empty_like(logits).exponential_(1.0).log_()
    return weights


def resolve_tokens(buffer: Tensor | None, batch_size: int, source: Tensor) -> Tensor:
    if (tokens := buffer) is None:
        tokens = source.new_empty(batch_size, 1, dtype=I32)
    return tokens


def resolve_probabilities(precondition: bool, source: Tensor, batch_size: int, vocab_size: int | None = None,
                          buffer: Tensor | None = None) -> Tensor | None:
    if (probabilities := buffer) is None and precondition:
        probabilities = source.new_zeros((batch_size, vocab_size or source.size(1)))
    return probabilities


def prepare_singular(
    # Required.
    logits: Tensor,
    indicators: Tensor,
    # Model & Engine Specific(s).
    local_vocab: int | None = None,
    shard_size: int | None = None,
    world_size: int = 1,
    local_rank: int = 0,
    lookahead: int = 0,
    target_vocab: int | None = None,
    max_top_logprobs: int = DEFAULT_TOP_LOGPROBS,
    # Conditional(s).
    enable_pdl: bool = True,
    is_prefill: bool = False,
    update_counts: bool = False,
    return_logprobs: bool = False,
    return_probabilities: bool = False,
    # Kernel Specific(s).
    block_n: int = 4_096,
    # Buffer(s).
    scratchpad: Tensor | None = None,
    # Logit Manipulator(s).
    slot_mapping: Tensor | None = None,
    d2t_mapping: Tensor | None = None,
    grammar: Tensor | None = None,
    context_counts: Tensor | None = None,
    decode_counts: Tensor | None = None,
    drafted_tokens: Tensor | None = None,
    repetition_penalties: Tensor | None = None,
    frequency_penalties: Tensor | None = None,
    presence_penalties: Tensor | None = None,
    logit_bias: Tensor | None = None,
    temperature: Tensor | None = None,
    top_k: Tensor | None = None,
    top_p: Tensor | None = None,
    min_p: Tensor | None = None,
    # Selection Parameter(s).
    top_k_logprobs: Tensor | None = None,
    gumbel_noise: Tensor | None = None,
    # Output Buffer(s).
    output_tokens: Tensor | None = None,
    draft_probabilities: Tensor | None = None,
    # Top-K Strategy & Tuning Configuration (accepted; no effect on the B200 kernel).
    topk_strategy: TopKStrategy | None = None,
    warp_config: TwoStageWarpConfig | None = None,
    # Counter-based noise (B200 addition).
    philox_seed: int | None = None,
    philox_offset: int = 0,
    # dtype of the logprob outputs: bf16 like the reference, or fp32 (B200 addition).
    logprobs_dtype: torch.dtype = torch.bfloat16,
) -> tuple[Selection, "ops.SingularArgs"]:
    """Resolve defaults, outputs and C-ABI arguments of `fused_singular` without launching.
    Works for host tensors too (no workspace is attached then)."""
    validate_count_update(update_counts, decode_counts)
    if world_size > 1 and gumbel_noise is None and philox_seed is None:
        raise ValueError("vocab-sharded sampling needs the full-vocabulary `gumbel_noise` (the same on every "
                         "rank) or `philox_seed`")

    batch_size, vocab_size = logits.shape
    vocab_size = min(vocab_size, local_vocab or vocab_size)
    shard_size = shard_size or vocab_size
    shard_offset = local_rank * shard_size

    philox = philox_seed is not None
    gumbel_weights = None if philox else resolve_gumbel(gumbel_noise, logits)
    final_tokens = resolve_tokens(output_tokens, batch_size, logits)
    probabilities = resolve_probabilities(return_probabilities, logits, indicators.size(0), target_vocab,
                                          draft_probabilities)
    selection = Selection.from_buffers(tokens=final_tokens, probabilities=probabilities,
                                       logprobs=return_logprobs, top_logprobs=max_top_logprobs,
                                       dtype=logprobs_dtype)
    token_logprobs = top_logprobs = top_tokens = None
    if sl := selection.logprobs:
        token_logprobs = sl.selected
        if st := sl.top_k:
            top_logprobs, top_tokens = st.logprobs, st.tokens

    flags = (
        (FLAG_PDL if enable_pdl else 0)
        | (FLAG_PREFILL if is_prefill else 0)
        | (FLAG_UPDATE_COUNTS if update_counts else 0)
        | (FLAG_LOGPROBS if return_logprobs else 0)
        | (FLAG_PROBABILITIES if return_probabilities else 0)
        | (FLAG_PHILOX if philox else 0)
    )
    # the reference reads bias with the counts' row stride when counts are given
    # (functional/singular.py:207 + ops/prologue.py:441)
    stride_c = next((t.stride(0) for t in (decode_counts, logit_bias) if t is not None), None)
    params = ops.sampling_params(
        indicators, slot_mapping=slot_mapping, grammar=grammar, context_counts=context_counts,
        decode_counts=decode_counts, counts_stride=stride_c, repetition_penalties=repetition_penalties,
        frequency_penalties=frequency_penalties, presence_penalties=presence_penalties, logit_bias=logit_bias,
        bias_stride=stride_c, temperature=temperature, top_k=top_k, top_p=top_p, min_p=min_p,
        top_k_logprobs=top_k_logprobs,
    )
    workspace = None
    if logits.device.type == "cuda":
        workspace = resolve_workspace(scratchpad, ops.singular_workspace_bytes(batch_size, vocab_size), logits.device)
    args = ops.singular_args(
        logits, params, vocab_size=vocab_size, block_n=block_n, tokens=final_tokens, flags=flags,
        lookahead=lookahead, shard_offset=shard_offset, max_top_logprobs=max_top_logprobs,
        target_vocab=(target_vocab or 0), d2t=d2t_mapping,
        drafted_tokens=drafted_tokens, gumbel=gumbel_weights, philox_seed=philox_seed or 0,
        philox_offset=philox_offset, logprobs=token_logprobs, top_logprob_values=top_logprobs,
        top_logprob_tokens=top_tokens, probabilities=probabilities, workspace=workspace,
    )
    return selection, args


def fused_singular(logits: Tensor, indicators: Tensor, process_group=None, **kwargs) -> Selection:
    """Same keywords as the reference's `fused_singular` (see `prepare_singular`).

    With `world_size > 1` the vocabulary is sharded: this rank's `logits` hold the columns
    [local_rank * shard_size, local_rank * shard_size + logits.size(1)), while buffers, noise
    and outputs cover the whole vocabulary and are the same on every rank. Each rank extracts
    its 128 best candidates per row, one all-gather over `process_group` (default: the world
    group) exchanges them, and every rank merges and selects identically."""
    ops._require_cuda(logits)
    selection, args = prepare_singular(logits, indicators, **kwargs)
    world = int(kwargs.get("world_size", 1))
    if world <= 1:
        ops.launch_singular(args, logits.device)
        return selection
    dev = logits.device
    vocab_sharded_exchange(args, logits.size(0), world, int(kwargs.get("shard_size") or logits.size(1)), dev,
                           extract=lambda a, keys: ops.launch_shard_candidates(a, keys, dev),
                           merge=lambda a, gathered, w: ops.launch_merge_candidates(a, gathered, w, dev),
                           process_group=process_group)
    return selection


def vocab_sharded_exchange(args, rows: int, world: int, shard: int, device, extract, merge,
                           process_group=None) -> None:
    """The exchange of the vocab-sharded path, identical on every rank: `extract(args, keys)`
    writes this rank's [rows, 128] candidate keys (global columns), one all-gather over
    `process_group` collects the `world` lists, and `merge(args, gathered, world)` merges and
    selects over the whole vocabulary. The product passes the CUDA steps
    (sonic_shard_candidates / sonic_merge_candidates); the multi-rank CPU tests pass the
    oracle's restatement of the same steps."""
    import torch.distributed as dist

    keys = torch.empty(rows, 128, dtype=torch.int64, device=device)
    extract(args, keys)
    # rank-major [world * rows, 128] (the layout every backend's all-gather writes)
    gathered = torch.empty(world * rows, 128, dtype=torch.int64, device=device)
    dist.all_gather_into_tensor(gathered, keys, group=process_group)
    args.vocab_size = shard * world  # candidates carry global columns below this bound
    merge(args, gathered.view(world, rows, 128), world)
