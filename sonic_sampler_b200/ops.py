"""Marshalling from PyTorch tensors to the C ABI (include/sonic_b200.h).

The `*_args` builders only read tensor metadata (data pointers, strides, dtypes), so the
same builder describes device tensors for the CUDA library and host tensors for the CPU
checker used by the tests. `launch_*` run the CUDA library on the current stream of the
tensors' device. Dtype / layout contracts follow the reference's SamplingBuffers
(core/buffer.py:784-817); a tensor that breaks them raises ValueError before any launch.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from sonic_sampler_b200 import _abi
from sonic_sampler_b200._abi import (
    DT_BF16,
    DT_F32,
    DT_I32,
    DT_I64,
    MultistepArgs,
    SamplingParams,
    SingularArgs,
    TopKArgs,
)

BF16 = torch.bfloat16
F32 = torch.float32
I32 = torch.int32
I64 = torch.int64

_INDEX_DTYPES = {I32: DT_I32, I64: DT_I64}
_FLOAT_DTYPES = {BF16: DT_BF16, F32: DT_F32}


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _keep(args, *tensors) -> None:
    """Hold references to the tensors an argument struct points at, for as long as the struct
    lives (the struct itself only stores raw addresses)."""
    prev = getattr(args, "_tensors", ())
    args._tensors = prev + tuple(t for t in tensors if isinstance(t, Tensor))


def _require(cond: bool, message: str) -> None:
    if not cond:
        raise ValueError(message)


def _vector(t: Tensor | None, name: str, dtypes: tuple[torch.dtype, ...]) -> int | None:
    if t is None:
        return None
    _require(t.dtype in dtypes, f"`{name}` must have dtype in {dtypes}, got {t.dtype}")
    _require(t.dim() == 1 and (t.numel() <= 1 or t.stride(0) == 1), f"`{name}` must be a contiguous vector")
    return t.data_ptr()


def _rows(t: Tensor | None, name: str, dtypes: tuple[torch.dtype, ...]) -> tuple[int | None, int]:
    """(pointer, row stride) of a tensor whose last dimension is unit-stride."""
    if t is None:
        return None, 0
    _require(t.dtype in dtypes, f"`{name}` must have dtype in {dtypes}, got {t.dtype}")
    _require(t.dim() >= 1 and (t.size(-1) <= 1 or t.stride(-1) == 1), f"`{name}` must have a unit inner stride")
    return t.data_ptr(), (t.stride(0) if t.dim() >= 2 else 0)


def index_dtype(t: Tensor | None, name: str) -> int:
    if t is None:
        return DT_I32
    _require(t.dtype in _INDEX_DTYPES, f"`{name}` must be int32 or int64, got {t.dtype}")
    return _INDEX_DTYPES[t.dtype]


def sampling_params(
    indicators: Tensor,
    slot_mapping: Tensor | None = None,
    grammar: Tensor | None = None,
    grammar_stride: int | None = None,
    context_counts: Tensor | None = None,
    decode_counts: Tensor | None = None,
    counts_stride: int | None = None,
    repetition_penalties: Tensor | None = None,
    frequency_penalties: Tensor | None = None,
    presence_penalties: Tensor | None = None,
    logit_bias: Tensor | None = None,
    bias_stride: int | None = None,
    temperature: Tensor | None = None,
    top_k: Tensor | None = None,
    top_p: Tensor | None = None,
    min_p: Tensor | None = None,
    top_k_logprobs: Tensor | None = None,
) -> SamplingParams:
    p = SamplingParams()
    p.indicators = _vector(indicators, "indicators", (torch.uint16, torch.int16))
    _require(p.indicators is not None, "`indicators` is required")
    p.num_slots = indicators.numel()
    if slot_mapping is not None:
        p.slot_mapping = _vector(slot_mapping, "slot_mapping", (I32, I64))
        p.slot_dtype = index_dtype(slot_mapping, "slot_mapping")
    if grammar is not None:
        _require(grammar.dtype in (torch.uint32, I32), "`grammar` must be uint32 or int32")
        _require(grammar.stride(-1) == 1, "`grammar` must have a unit inner stride")
        p.grammar = grammar.data_ptr()
        p.grammar_stride = grammar_stride if grammar_stride is not None else grammar.stride(0)
    ctx_ptr, ctx_stride = _rows(context_counts, "context_counts", (I32,))
    dec_ptr, dec_stride = _rows(decode_counts, "decode_counts", (I32,))
    p.context_counts = ctx_ptr
    p.decode_counts = dec_ptr
    p.counts_stride = counts_stride if counts_stride is not None else (dec_stride or ctx_stride)
    p.repetition = _vector(repetition_penalties, "repetition_penalties", (BF16,))
    p.frequency = _vector(frequency_penalties, "frequency_penalties", (BF16,))
    p.presence = _vector(presence_penalties, "presence_penalties", (BF16,))
    b_ptr, b_stride = _rows(logit_bias, "logit_bias", (BF16,))
    p.bias = b_ptr
    p.bias_stride = bias_stride if bias_stride is not None else b_stride
    p.temperature = _vector(temperature, "temperature", (BF16,))
    p.top_k = _vector(top_k, "top_k", (I32,))
    p.top_p = _vector(top_p, "top_p", (BF16,))
    p.min_p = _vector(min_p, "min_p", (BF16,))
    p.top_logprobs = _vector(top_k_logprobs, "top_k_logprobs", (I32,))
    _keep(p, indicators, slot_mapping, grammar, context_counts, decode_counts, repetition_penalties,
          frequency_penalties, presence_penalties, logit_bias, temperature, top_k, top_p, min_p, top_k_logprobs)
    return p


def singular_args(
    logits: Tensor,
    params: SamplingParams,
    *,
    vocab_size: int,
    block_n: int,
    tokens: Tensor,
    flags: int,
    lookahead: int = 0,
    shard_offset: int = 0,
    max_top_logprobs: int = 0,
    target_vocab: int = 0,
    d2t: Tensor | None = None,
    drafted_tokens: Tensor | None = None,
    gumbel: Tensor | None = None,
    philox_seed: int = 0,
    philox_offset: int = 0,
    logprobs: Tensor | None = None,
    top_logprob_values: Tensor | None = None,
    top_logprob_tokens: Tensor | None = None,
    probabilities: Tensor | None = None,
    workspace: Tensor | None = None,
) -> SingularArgs:
    a = SingularArgs()
    _require(logits.dim() == 2, "logits must be 2-D [rows, vocab]")
    a.rows = logits.size(0)
    a.vocab_size = vocab_size
    a.block_n = block_n
    a.lookahead = lookahead
    a.shard_offset = shard_offset
    a.max_top_logprobs = max_top_logprobs
    a.target_vocab = target_vocab
    a.flags = flags
    a.logits, a.logits_stride = _rows(logits, "logits", (BF16,))
    a.logits_dtype = DT_BF16
    a.params = params
    if d2t is not None:
        a.d2t = _vector(d2t, "d2t_mapping", (I32, I64))
        a.d2t_dtype = index_dtype(d2t, "d2t_mapping")
    a.drafted_tokens, a.drafted_stride = _rows(drafted_tokens, "drafted_tokens", (I32,))
    a.gumbel, a.gumbel_stride = _rows(gumbel, "gumbel_noise", (BF16,))
    a.philox_seed = philox_seed & 0xFFFFFFFFFFFFFFFF
    a.philox_offset = philox_offset & 0xFFFFFFFFFFFFFFFF
    a.tokens, a.tokens_stride = _rows(tokens, "output_tokens", (I32,))
    if tokens.dim() == 1:
        a.tokens_stride = tokens.stride(0)
    if logprobs is not None:
        _require(logprobs.dtype in _FLOAT_DTYPES, "logprobs output must be bf16 or fp32")
        a.logprobs, a.logprobs_stride = logprobs.data_ptr(), logprobs.stride(0)
        a.logprobs_dtype = _FLOAT_DTYPES[logprobs.dtype]
    if top_logprob_values is not None:
        _require(top_logprob_values.stride() == top_logprob_tokens.stride(), "top-k logprob outputs must share strides")
        _require(logprobs is not None and top_logprob_values.dtype == logprobs.dtype,
                 "top-k logprobs must share the selected logprobs' dtype")
        a.top_logprob_values, a.top_stride = _rows(top_logprob_values, "top_logprobs", (BF16, F32))
        a.top_logprob_tokens, _ = _rows(top_logprob_tokens, "top_tokens", (I32,))
    if probabilities is not None:
        a.probabilities, a.probabilities_stride = _rows(probabilities, "probabilities", (BF16, F32))
        a.probabilities_dtype = _FLOAT_DTYPES[probabilities.dtype]
    if workspace is not None:
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel() * workspace.element_size()
    _keep(a, logits, tokens, d2t, drafted_tokens, gumbel, logprobs, top_logprob_values, top_logprob_tokens,
          probabilities, workspace, *getattr(params, "_tensors", ()))
    return a


def multistep_args(
    logits: Tensor,
    params: SamplingParams,
    *,
    batch_size: int,
    lookahead: int,
    vocab_size: int,
    block_n: int,
    drafted_tokens: Tensor,
    tokens: Tensor,
    offsets: Tensor,
    uniform: Tensor | None,
    gumbel: Tensor | None,
    gumbel_step_stride: int,
    flags: int,
    cu_seqlens: Tensor | None = None,
    shard_offset: int = 0,
    max_top_logprobs: int = 0,
    draft_probs: Tensor | None = None,
    draft_step_stride: int = 0,
    values: Tensor | None = None,
    indices: Tensor | None = None,
    logprobs: Tensor | None = None,
    top_logprob_values: Tensor | None = None,
    top_logprob_tokens: Tensor | None = None,
    workspace: Tensor | None = None,
    philox_seed: int = 0,
    philox_offset: int = 0,
) -> MultistepArgs:
    a = MultistepArgs()
    _require(logits.dim() == 2, "logits must be collapsed to 2-D [rows, vocab]")
    a.batch_size = batch_size
    a.lookahead = lookahead
    a.vocab_size = vocab_size
    a.block_n = block_n
    a.shard_offset = shard_offset
    a.max_top_logprobs = max_top_logprobs
    a.flags = flags
    a.total_rows = logits.size(0)
    a.logits, a.logits_stride = _rows(logits, "logits", (BF16,))
    a.logits_dtype = DT_BF16
    if cu_seqlens is not None:
        a.cu_seqlens = _vector(cu_seqlens, "cu_seqlens", (I32,))
    a.params = params
    _require(drafted_tokens.dtype == I32 and drafted_tokens.is_contiguous(), "drafted tokens must be contiguous int32")
    a.drafted_tokens = drafted_tokens.data_ptr()
    if draft_probs is not None:
        _require(draft_probs.dtype in _FLOAT_DTYPES, "draft probabilities must be fp32 or bf16")
        _require(draft_probs.stride(-1) == 1, "draft probabilities must have a unit inner stride")
        a.draft_probs = draft_probs.data_ptr()
        a.draft_dtype = _FLOAT_DTYPES[draft_probs.dtype]
        a.draft_stride = draft_probs.stride(0)
        a.draft_step_stride = draft_step_stride
    if uniform is not None:
        a.uniform, a.uniform_stride = _rows(uniform, "uniform_noise", (BF16,))
    if gumbel is not None:
        a.gumbel, a.gumbel_stride = _rows(gumbel, "gumbel_noise", (BF16,))
    a.gumbel_step_stride = gumbel_step_stride
    a.philox_seed = philox_seed & 0xFFFFFFFFFFFFFFFF
    a.philox_offset = philox_offset & 0xFFFFFFFFFFFFFFFF
    if values is not None:
        _require(values.dtype == F32 and values.is_contiguous(), "values buffer must be contiguous fp32")
        a.values = values.data_ptr()
    if indices is not None:
        _require(indices.dtype == I32 and indices.is_contiguous(), "indices buffer must be contiguous int32")
        a.indices = indices.data_ptr()
    _require(tokens.dtype == I32 and tokens.is_contiguous(), "output tokens must be contiguous int32")
    a.tokens = tokens.data_ptr()
    _require(offsets.dtype == I32 and offsets.is_contiguous(), "offsets must be contiguous int32")
    a.offsets = offsets.data_ptr()
    if logprobs is not None:
        _require(logprobs.dtype in _FLOAT_DTYPES and logprobs.is_contiguous(), "logprobs output must be contiguous bf16/fp32")
        a.logprobs = logprobs.data_ptr()
        a.logprobs_dtype = _FLOAT_DTYPES[logprobs.dtype]
    if top_logprob_values is not None:
        _require(logprobs is not None and top_logprob_values.dtype == logprobs.dtype,
                 "top-k logprobs must share the selected logprobs' dtype")
        a.top_logprob_values, a.top_stride = _rows(top_logprob_values.flatten(0, -2), "top_logprobs", (BF16, F32))
        a.top_logprob_tokens, _ = _rows(top_logprob_tokens.flatten(0, -2), "top_tokens", (I32,))
    if workspace is not None:
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel() * workspace.element_size()
    _keep(a, logits, cu_seqlens, drafted_tokens, tokens, offsets, uniform, gumbel, draft_probs, values, indices,
          logprobs, top_logprob_values, top_logprob_tokens, workspace, *getattr(params, "_tensors", ()))
    return a


def topk_args(
    logits: Tensor,
    *,
    vocab_size: int,
    k: int,
    block_n: int,
    values: Tensor,
    indices: Tensor,
    flags: int = 0,
    workspace: Tensor | None = None,
) -> TopKArgs:
    a = TopKArgs()
    _require(logits.dim() == 2, "logits must be 2-D [rows, vocab]")
    a.rows = logits.size(0)
    a.vocab_size = vocab_size
    a.k = k
    a.block_n = block_n
    a.flags = flags
    a.logits, a.logits_stride = _rows(logits, "logits", (BF16, F32))
    a.logits_dtype = _FLOAT_DTYPES[logits.dtype]
    _require(values.dtype in _FLOAT_DTYPES and values.is_contiguous(), "values buffer must be contiguous bf16/fp32")
    a.values = values.data_ptr()
    a.values_dtype = _FLOAT_DTYPES[values.dtype]
    _require(indices.dtype in _INDEX_DTYPES and indices.is_contiguous(), "indices buffer must be contiguous int32/int64")
    a.indices = indices.data_ptr()
    a.indices_dtype = _INDEX_DTYPES[indices.dtype]
    if workspace is not None:
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel() * workspace.element_size()
    _keep(a, logits, values, indices, workspace)
    return a


# ---------------------------------------------------------------------------------------
# workspace + launch
# ---------------------------------------------------------------------------------------


def singular_workspace_bytes(rows: int, vocab_size: int) -> int:
    a = SingularArgs()
    a.rows, a.vocab_size = rows, vocab_size
    return int(_abi.load_library().sonic_fused_singular_workspace_size(ctypes.byref(a)))


def multistep_workspace_bytes(batch_size: int, lookahead: int, vocab_size: int, total_rows: int = 0) -> int:
    a = MultistepArgs()
    a.batch_size, a.lookahead, a.vocab_size, a.total_rows = batch_size, lookahead, vocab_size, total_rows
    return int(_abi.load_library().sonic_fused_multistep_workspace_size(ctypes.byref(a)))


def topk_workspace_bytes(rows: int, vocab_size: int) -> int:
    a = TopKArgs()
    a.rows, a.vocab_size = rows, vocab_size
    return int(_abi.load_library().sonic_bounded_topk_workspace_size(ctypes.byref(a)))


def new_workspace(nbytes: int, device: torch.device) -> Tensor:
    """Zero-filled workspace (the kernels keep their tickets at zero between calls).

    The zero fill runs on the current stream. Outside graph capture the call waits for it,
    so that a later call on any other stream finds the tickets at zero."""
    ws = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
    if ws.is_cuda and not torch.cuda.is_current_stream_capturing():
        torch.cuda.current_stream(ws.device).synchronize()
    return ws


def workspace_error(workspace: Tensor | None, device: torch.device | None = None) -> int:
    """Read and clear the device error word (DEVICE_ERR_* bits) that earlier calls left in
    `workspace`, or with None the library's own word (static-scratch and noise-staging
    calls). Synchronises the current stream of `device`."""
    dev = workspace.device if workspace is not None else (device or torch.device("cuda", torch.cuda.current_device()))
    lib = _abi.load_library()
    out = ctypes.c_uint32(0)
    with torch.cuda.device(dev):
        _abi.check(lib.sonic_workspace_error(_ptr(workspace), ctypes.byref(out), _stream(dev)), lib)
    return int(out.value)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: Tensor) -> None:
    if t.device.type != "cuda":
        raise ValueError("the fused sampler runs on CUDA tensors only (no CPU fallback)")


def launch_singular(args: SingularArgs, device: torch.device) -> None:
    lib = _abi.load_library()
    with torch.cuda.device(device):
        _abi.check(lib.sonic_fused_singular(ctypes.byref(args), ctypes.c_void_p(_stream(device))), lib)


def launch_shard_candidates(args: SingularArgs, keys: Tensor, device: torch.device) -> None:
    """Vocab-sharded step 1: this rank's top-128 candidate keys per row into `keys` [rows, 128] int64."""
    _require(keys.dtype == torch.int64 and keys.is_contiguous() and keys.numel() >= args.rows * 128,
             "keys must be a contiguous int64 tensor of rows x 128")
    lib = _abi.load_library()
    with torch.cuda.device(device):
        _abi.check(lib.sonic_shard_candidates(ctypes.byref(args), ctypes.c_void_p(keys.data_ptr()),
                                              ctypes.c_void_p(_stream(device))), lib)


def launch_merge_candidates(args: SingularArgs, gathered: Tensor, world: int, device: torch.device) -> None:
    """Vocab-sharded step 3: merge `gathered` [world, rows, 128] int64 keys and select."""
    _require(gathered.dtype == torch.int64 and gathered.is_contiguous() and gathered.numel() >= world * args.rows * 128,
             "gathered must be a contiguous int64 tensor of world x rows x 128")
    lib = _abi.load_library()
    with torch.cuda.device(device):
        _abi.check(lib.sonic_merge_candidates(ctypes.byref(args), ctypes.c_void_p(gathered.data_ptr()), int(world),
                                              ctypes.c_void_p(_stream(device))), lib)


def launch_multistep(args: MultistepArgs, device: torch.device) -> None:
    lib = _abi.load_library()
    with torch.cuda.device(device):
        _abi.check(lib.sonic_fused_multistep(ctypes.byref(args), ctypes.c_void_p(_stream(device))), lib)


def launch_topk(args: TopKArgs, device: torch.device) -> None:
    lib = _abi.load_library()
    with torch.cuda.device(device):
        _abi.check(lib.sonic_bounded_topk(ctypes.byref(args), ctypes.c_void_p(_stream(device))), lib)


def indexed_copy(source: Tensor, target: Tensor, indices: Tensor, indicator: Tensor) -> None:
    """Fused `index_select` of `source` rows at `indices` and `index_copy_` into `target`, only
    for rows whose `indicator` lacks the greedy bit 0x40 (reference `ops/copy.py:86-109`).

    `source` and `target` have the same shape, dtype and row stride, with each row contiguous
    (the reference copies `source.flatten(1).size(1)` elements per row at `source.stride(0)`
    for both). `indices` is int32 or int64, `indicator` uint16 per row. Runs on the current
    stream of the tensors' device; indices outside the rows are skipped."""
    _require(source.is_cuda and target.is_cuda and indices.is_cuda and indicator.is_cuda,
             "source, target, indices and indicator must be CUDA tensors")
    _require(source.shape == target.shape and source.dtype == target.dtype, "source and target must match in shape and dtype")
    _require(source.dim() >= 1 and source.stride(0) == target.stride(0), "source and target must share the row stride")
    rows = source.size(0)
    if rows == 0 or indices.numel() == 0:
        return
    _require(source[0].is_contiguous() and target[0].is_contiguous(), "rows must be contiguous")
    _require(indicator.dtype == torch.uint16 and indicator.is_contiguous() and indicator.numel() >= rows,
             "indicator must be a contiguous uint16 tensor with an entry per row")
    _require(indices.dim() == 1 and indices.is_contiguous(), "indices must be a contiguous vector")
    cols = source[0].numel()
    lib = _abi.load_library()
    with torch.cuda.device(source.device):
        _abi.check(lib.sonic_indexed_copy(
            ctypes.c_void_p(source.data_ptr()), ctypes.c_void_p(target.data_ptr()), rows, source.stride(0), cols,
            source.element_size(), ctypes.c_void_p(indices.data_ptr()), index_dtype(indices, "indices"),
            indices.numel(), ctypes.c_void_p(indicator.data_ptr()), ctypes.c_void_p(_stream(source.device))), lib)
