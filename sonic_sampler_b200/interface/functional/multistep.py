"""`fused_multistep`: speculative verification of gamma drafted tokens per request
(reference interface/functional/multistep.py:175-461).

Same keyword set, shape handling and ValueErrors as the reference; the three Triton
launches become the fused B200 kernels of `sonic_fused_multistep`, which also read each
request's count and bias rows once instead of once per timestep.

One addition, off by default: `philox_seed` / `philox_offset` draw the acceptance uniforms
and the rejection step's Gumbel noise in-kernel from counter-based Philox (step s of the
call uses counter offset `philox_offset + s`), so no noise buffer is read or refreshed.
"""

from __future__ import annotations

import torch
from torch import Tensor

from sonic_sampler_b200 import ops
from sonic_sampler_b200._abi import FLAG_LOGPROBS, FLAG_PDL, FLAG_PHILOX, FLAG_UPDATE_COUNTS, MAX_K
from sonic_sampler_b200.base.sampler import DEFAULT_TOP_LOGPROBS, Verification
from sonic_sampler_b200.interface.base import TopKStrategy
from sonic_sampler_b200.interface.dispatch import ThreeStageWarpConfig
from sonic_sampler_b200.interface.functional.base import (
    I32,
    collapse_2d,
    resolve_workspace,
    validate_count_update,
)

BF16 = torch.bfloat16
FP32 = torch.float32
TINY: float = torch.finfo(BF16).tiny


def resolve_batch_vocab(logits: Tensor, cu_seqlens: Tensor | None, lookahead: int | None) -> tuple[bool, int, int, int]:
    """Same shape rules and messages as the reference (functional/multistep.py:50-106)."""
    varlen = cu_seqlens is not None
    if logits.ndim == 2:
        n_rows, vocab_size = logits.shape
        if varlen:
            if not lookahead:
                raise ValueError("maximum lookahead must be defined for varlen logits")
            return varlen, cu_seqlens.size(0) - 1, lookahead, vocab_size
        if not lookahead:
            raise ValueError("found 2-D logits with zero lookahead")
        batch_size, margin = divmod(n_rows, lookahead + 1)
        if margin:
            raise ValueError("not varlen but total rows not a multiple of lookahead + 1")
        return varlen, batch_size, lookahead, vocab_size
    if logits.ndim == 3:
        if varlen:
            raise ValueError("expected varlen but logits has a fixed timestep dimension")
        batch_size, timesteps, vocab_size = logits.shape
        return varlen, batch_size, timesteps - 1, vocab_size
    raise ValueError(f"unsupported logits shape: {tuple(logits.shape)}")


def resolve_unpack_buffers(logits: Tensor, values: Tensor | None, indices: Tensor | None) -> tuple[Tensor, Tensor]:
    n_rows = collapse_2d(logits).size(0)
    if values is None:
        values = logits.new_empty((n_rows, MAX_K), dtype=FP32)
    if indices is None:
        indices = logits.new_empty((n_rows, MAX_K), dtype=I32)
    return values, indices


def resolve_gumbel(noise: Tensor | None, logits: Tensor, batch_size: int, timesteps: int) -> Tensor:
    if noise is None:
        noise = logits.new_empty((batch_size, timesteps, logits.size(-1))).exponential_(1.0).log_()
    return noise


def resolve_uniform(noise: Tensor | None, logits: Tensor, batch_size: int, lookahead: int) -> Tensor:
    if noise is None:
        noise = logits.new_empty((batch_size, lookahead)).uniform_(TINY, 1)
    return noise


def resolve_tokens(drafted: Tensor, output: Tensor | None) -> Tensor:
    return output if output is not None else drafted.clone()


def prepare_multistep(
    # Required.
    logits: Tensor,
    indicators: Tensor,
    drafted_tokens: Tensor,
    # Model & Engine Specific(s).
    local_vocab: int | None = None,
    shard_size: int | None = None,
    world_size: int = 1,
    local_rank: int = 0,
    lookahead: int | None = None,
    max_top_logprobs: int = DEFAULT_TOP_LOGPROBS,
    # Conditional(s).
    enable_pdl: bool = True,
    update_counts: bool = False,
    return_logprobs: bool = False,
    # Kernel Specific(s).
    block_n: int = 4_096,
    # Buffer(s).
    scratchpad: Tensor | None = None,
    values: Tensor | None = None,
    indices: Tensor | None = None,
    # Support(s).
    draft_probabilities: Tensor | None = None,
    # Logit Manipulator(s).
    slot_mapping: Tensor | None = None,
    cu_seqlens: Tensor | None = None,
    grammar: Tensor | None = None,
    context_counts: Tensor | None = None,
    decode_counts: Tensor | None = None,
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
    uniform_noise: Tensor | None = None,
    # Counter-based in-kernel noise (B200 addition; see module docstring).
    philox_seed: int | None = None,
    philox_offset: int = 0,
    # Output Buffer(s).
    output_tokens: Tensor | None = None,
    # Top-K Strategy & Tuning Configuration (accepted; no effect on the B200 kernel).
    topk_strategy: TopKStrategy | None = None,
    warp_config: ThreeStageWarpConfig | None = None,
    # dtype of the logprob outputs: bf16 like the reference, or fp32 (B200 addition).
    logprobs_dtype: torch.dtype = BF16,
) -> tuple[Verification, "ops.MultistepArgs"]:
    """Resolve defaults, outputs and C-ABI arguments of `fused_multistep` without launching.
    Works for host tensors too (no workspace is attached then)."""
    validate_count_update(update_counts, decode_counts)
    if world_size > 1:
        raise ValueError("vocab-sharded multistep verification is not supported; shard requests by rows")

    varlen, batch_size, gamma, vocab_size = resolve_batch_vocab(logits, cu_seqlens, lookahead)
    vocab_size = min(vocab_size, local_vocab or vocab_size)
    shard_size = shard_size or vocab_size
    shard_offset = local_rank * shard_size

    flat_logits = collapse_2d(logits)
    values_buffer, indices_buffer = resolve_unpack_buffers(logits, values, indices)
    philox = philox_seed is not None
    # with Philox noise no buffer is read, so none is drawn either (the reference's default
    # draws fresh [B, gamma+1, V] and [B, gamma] buffers on every call)
    gumbel_weights = None if philox else resolve_gumbel(gumbel_noise, logits, batch_size, gamma + 1)
    uniform_weights = None if philox else resolve_uniform(uniform_noise, logits, batch_size, gamma)

    verification = Verification.from_tokens(
        tokens=resolve_tokens(drafted_tokens, output_tokens), batch_size=batch_size, timesteps=gamma + 1,
        logprobs=return_logprobs, varlen=varlen, top_logprobs=max_top_logprobs, dtype=logprobs_dtype,
    )
    token_logprobs = top_logprobs = top_tokens = None
    if vl := verification.logprobs:
        token_logprobs = vl.selected
        if vt := vl.top_k:
            top_logprobs, top_tokens = vt.logprobs, vt.tokens

    flags = (
        (FLAG_PDL if enable_pdl else 0)
        | (FLAG_UPDATE_COUNTS if update_counts else 0)
        | (FLAG_LOGPROBS if return_logprobs else 0)
        | (FLAG_PHILOX if philox else 0)
    )
    # counts and bias rows are read with the noise row stride (functional/multistep.py:316);
    # without a noise buffer, with their own row stride
    if gumbel_weights is not None:
        stride_c = collapse_2d(gumbel_weights).stride(0)
    else:
        rows_c = [t for t in (decode_counts, context_counts, logit_bias, draft_probabilities) if t is not None]
        stride_c = collapse_2d(rows_c[0]).stride(0) if rows_c else vocab_size
    params = ops.sampling_params(
        indicators, slot_mapping=slot_mapping, grammar=grammar,
        grammar_stride=None if grammar is None else collapse_2d(grammar).stride(0),
        context_counts=context_counts, decode_counts=decode_counts, counts_stride=stride_c,
        repetition_penalties=repetition_penalties, frequency_penalties=frequency_penalties,
        presence_penalties=presence_penalties, logit_bias=logit_bias, bias_stride=stride_c,
        temperature=temperature, top_k=top_k, top_p=top_p, min_p=min_p, top_k_logprobs=top_k_logprobs,
    )
    workspace = None
    if logits.device.type == "cuda":
        workspace = resolve_workspace(
            scratchpad, ops.multistep_workspace_bytes(batch_size, gamma, vocab_size, flat_logits.size(0)), logits.device)
    args = ops.multistep_args(
        flat_logits, params, batch_size=batch_size, lookahead=gamma, vocab_size=vocab_size, block_n=block_n,
        drafted_tokens=drafted_tokens, tokens=verification.tokens, offsets=verification.offsets,
        uniform=uniform_weights, gumbel=gumbel_weights, gumbel_step_stride=stride_c, flags=flags,
        cu_seqlens=cu_seqlens, shard_offset=shard_offset, max_top_logprobs=max_top_logprobs,
        draft_probs=draft_probabilities,
        # the reference steps through q with the same row stride (verify.py:140-142, 220)
        draft_step_stride=stride_c,
        values=values_buffer, indices=indices_buffer, logprobs=token_logprobs,
        top_logprob_values=top_logprobs, top_logprob_tokens=top_tokens, workspace=workspace,
        philox_seed=philox_seed or 0, philox_offset=philox_offset,
    )
    return verification, args


def fused_multistep(logits: Tensor, indicators: Tensor, drafted_tokens: Tensor, **kwargs) -> Verification:
    """Same keywords as the reference's `fused_multistep` (see `prepare_multistep`)."""
    ops._require_cuda(logits)
    verification, args = prepare_multistep(logits, indicators, drafted_tokens, **kwargs)
    ops.launch_multistep(args, logits.device)
    return verification
