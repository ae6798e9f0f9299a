"""Batched population of request slots: the device side of the reference's
`SamplingBuffers.allocate / update / step_grammar` (core/buffer.py:1026-1052, 1139-1352).

The reference fills a slot through pinned host mirrors and about a dozen `copy_` calls per
slot: the scalars (PinnedRelay.populate + transfer, RepetitionPenalties.populate +
transfer, Flags.update), a dense V-long bias row (PinnedRelay.update_bias), a dense V-long
prompt histogram built on the host (TokenCounts.populate + allocate) or two dense count
rows (TokenCounts.update), and the grammar rows (step_grammar). Here every slot of a call
is packed into one staging blob of sparse inputs (prompt token ids, bias entries, bitmask
words), copied to the device with one `cudaMemcpyAsync` from pinned memory, and written by
one `sonic_populate_slots` launch.

The `pack_*` functions are host-only (numpy); `SlotStager` and `launch_populate` need CUDA.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np
import torch
from torch import Tensor

from sonic_sampler_b200 import _abi

BF16 = torch.bfloat16

SCALARS = _abi.POPULATE_SCALARS
HISTOGRAM = _abi.POPULATE_HISTOGRAM
DENSE_COUNTS = _abi.POPULATE_DENSE_COUNTS
BIAS = _abi.POPULATE_BIAS
GRAMMAR = _abi.POPULATE_GRAMMAR

_ALIGN = 16


def bf16_bits(values: Sequence[float]) -> np.ndarray:
    """bf16 bit patterns of Python floats, rounded exactly as the reference's
    `torch.tensor(values, dtype=BF16)` (core/buffer.py:568, 750)."""
    if len(values) == 0:
        return np.zeros(0, dtype=np.uint16)
    return torch.tensor(list(values), dtype=BF16).view(torch.int16).numpy().view(np.uint16).copy()


@dataclass
class SlotBatch:
    """Host-side inputs of one `sonic_populate_slots` call (arrays of the C ABI's
    SonicPopulateArgs, see include/sonic_b200.h)."""

    count: int
    vocab_size: int
    parts: int
    positions: np.ndarray                      # i32 [count]
    grammar_step: int = -1
    values_bf16: np.ndarray | None = None      # u16 [count, 6]
    values_i32: np.ndarray | None = None       # i32 [count, 2]
    indicators: np.ndarray | None = None       # u16 [count, 2]
    token_offsets: np.ndarray | None = None    # i64 [count + 1]
    tokens: np.ndarray | None = None           # i32 [n]
    bias_offsets: np.ndarray | None = None     # i64 [count + 1]
    bias_tokens: np.ndarray | None = None      # i32 [m]
    bias_values: np.ndarray | None = None      # u16 [m]
    grammar_rows: np.ndarray | None = None     # i32 [count], -1: no bitmask
    grammar_steps: np.ndarray | None = None    # i32 [count]
    grammar_words: np.ndarray | None = None    # u32 [rows, ceil(V / 32)]
    dense_context: np.ndarray | Tensor | None = None  # i32 [count, V] (host array or device tensor)
    dense_decode: np.ndarray | Tensor | None = None
    keep: list = field(default_factory=list)   # device tensors the launch reads

    def sections(self) -> list[tuple[str, np.ndarray]]:
        """The host arrays that travel in the staging blob, in blob order."""
        names = ("positions", "values_bf16", "values_i32", "indicators", "token_offsets", "tokens", "bias_offsets",
                 "bias_tokens", "bias_values", "grammar_rows", "grammar_steps", "grammar_words", "dense_context",
                 "dense_decode")
        out = []
        for name in names:
            v = getattr(self, name)
            if isinstance(v, np.ndarray):
                out.append((name, np.ascontiguousarray(v)))
        return out


def _check_positions(positions: Sequence[int], num_slots: int) -> np.ndarray:
    pos = np.asarray(list(positions), dtype=np.int64)
    if pos.size and (pos.min() < 0 or pos.max() >= num_slots):
        raise IndexError(f"positions must lie in [0, {num_slots})")
    if len(set(pos.tolist())) != pos.size:
        raise ValueError("positions must be distinct")
    return pos.astype(np.int32)


def pack_scalars(batch: SlotBatch, temperature, top_p, min_p, multiplicative, frequency, presence, top_k, top_logprobs,
                 target, draft) -> None:
    """Per-slot scalars (PinnedRelay.populate core/buffer.py:738-764, RepetitionPenalties.populate
    :562-582, Flags.update core/flags.py:543-572)."""
    n = batch.count
    cols = [temperature, top_p, min_p, multiplicative, frequency, presence]
    if any(len(c) != n for c in cols + [top_k, top_logprobs, target, draft]):
        raise ValueError("every per-slot parameter list must have one entry per position")
    batch.values_bf16 = np.stack([bf16_bits(c) for c in cols], axis=1) if n else np.zeros((0, 6), np.uint16)
    batch.values_i32 = np.asarray([list(map(int, top_k)), list(map(int, top_logprobs))], dtype=np.int64).T.astype(np.int32)
    batch.indicators = np.asarray([list(map(int, target)), list(map(int, draft))], dtype=np.int64).T.astype(np.uint16)
    batch.parts |= SCALARS


def pack_histogram(batch: SlotBatch, encodings: Sequence[Tensor]) -> None:
    """Prompt token ids whose histogram becomes the context counts (TokenCounts.populate +
    allocate, core/buffer.py:422-457). The reference's `scatter_add_` raises on ids outside
    the vocabulary; so does this."""
    if len(encodings) != batch.count:
        raise ValueError("encodings must have one entry per position")
    V = batch.vocab_size
    flat = [e.detach().reshape(-1).cpu() if isinstance(e, Tensor) else torch.as_tensor(np.asarray(e)).reshape(-1)
            for e in encodings]
    lengths = np.fromiter((t.numel() for t in flat), dtype=np.int64, count=len(flat))
    ids = torch.cat(flat).to(torch.int64) if flat else torch.zeros(0, dtype=torch.int64)
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= V):
        raise RuntimeError(f"token id out of bounds for a vocabulary of {V}")
    batch.token_offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    batch.tokens = ids.to(torch.int32).numpy()
    batch.parts |= HISTOGRAM


def pack_dense_counts(batch: SlotBatch, counts: Sequence[tuple[Tensor, Tensor]], device: torch.device) -> None:
    """Dense (context, decode) rows copied as they are (TokenCounts.update core/buffer.py:395-420).
    Host rows travel in the staging blob; when any row is on the device the rows are stacked
    there instead."""
    if len(counts) != batch.count:
        raise ValueError("counts must have one (context, decode) pair per position")
    V = batch.vocab_size
    for c, d in counts:
        if c.numel() != V or d.numel() != V:
            raise ValueError(f"count rows must hold vocab_size ({V}) entries")
    if any(t.is_cuda for pair in counts for t in pair):
        ctx = torch.stack([c.reshape(-1).to(device=device, dtype=torch.int32) for c, _ in counts])
        dec = torch.stack([d.reshape(-1).to(device=device, dtype=torch.int32) for _, d in counts])
        batch.dense_context, batch.dense_decode = ctx, dec
        batch.keep += [ctx, dec]
    else:
        batch.dense_context = np.stack([c.reshape(-1).numpy().astype(np.int32) for c, _ in counts]) \
            if counts else np.zeros((0, V), np.int32)
        batch.dense_decode = np.stack([d.reshape(-1).numpy().astype(np.int32) for _, d in counts]) \
            if counts else np.zeros((0, V), np.int32)
    batch.parts |= DENSE_COUNTS


def pack_bias(batch: SlotBatch, biases: Sequence[dict[int, float] | None] | None) -> None:
    """Bias rows: zero, then the slot's {token: value} entries (PinnedRelay.update_bias +
    transfer, core/buffer.py:707-736, 1098-1135). Token ids must lie in the vocabulary."""
    n, V = batch.count, batch.vocab_size
    biases = list(biases) if biases else [None] * n
    if len(biases) != n:
        raise ValueError("biases must have one entry per position")
    maps = [m if m else {} for m in biases]
    lengths = np.fromiter((len(m) for m in maps), dtype=np.int64, count=n)
    total = int(lengths.sum())
    toks = np.fromiter((t for m in maps for t in m.keys()), dtype=np.int64, count=total)
    vals = [float(v) for m in maps for v in m.values()]
    if total and (toks.min() < 0 or toks.max() >= V):
        bad = toks[(toks < 0) | (toks >= V)][0]
        raise ValueError(f"logit bias token {bad} outside the vocabulary of {V}")
    batch.bias_offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    batch.bias_tokens = toks.astype(np.int32)
    batch.bias_values = bf16_bits(vals)
    batch.parts |= BIAS


def pack_grammar(batch: SlotBatch, bitmasks: Sequence[Tensor | None] | None, timesteps: int, step: int | None) -> None:
    """Grammar bitmask words (step_grammar, core/buffer.py:1026-1052): with `step` the mask goes
    to that step of the slot (admission writes step 0); without, to every step, from one row
    (broadcast, as `copy_` does) or from one row a step. The list is aligned with the
    positions, like every other per-slot list."""
    if not bitmasks or not any(m is not None for m in bitmasks):
        return
    if len(bitmasks) != batch.count:
        raise ValueError("bitmasks must have one entry per position")
    W = (batch.vocab_size + 31) // 32
    rows, nsteps, blocks = [], [], []
    next_row = 0
    for m in bitmasks:
        if m is None:
            rows.append(-1)
            nsteps.append(0)
            continue
        t = m if isinstance(m, Tensor) else torch.as_tensor(np.asarray(m))
        if t.element_size() != 4:
            raise ValueError("grammar bitmasks are 32-bit words")
        t = t.detach().reshape(-1, t.shape[-1]) if t.dim() > 1 else t.detach().reshape(1, -1)
        if t.shape[-1] != W or (t.shape[0] != 1 and (step is not None or t.shape[0] != timesteps)):
            raise ValueError(f"a bitmask must have shape [{W}]" + ("" if step is not None else f" or [{timesteps}, {W}]"))
        rows.append(next_row)
        nsteps.append(t.shape[0])
        blocks.append(t.view(torch.int32) if t.dtype != torch.int32 else t)
        next_row += t.shape[0]
    batch.grammar_rows = np.asarray(rows, dtype=np.int32)
    batch.grammar_steps = np.asarray(nsteps, dtype=np.int32)
    batch.grammar_words = torch.cat(blocks).cpu().numpy().view(np.uint32)
    batch.grammar_step = -1 if step is None else int(step)
    batch.parts |= GRAMMAR


def new_batch(positions: Sequence[int], num_slots: int, vocab_size: int) -> SlotBatch:
    pos = _check_positions(positions, num_slots)
    return SlotBatch(count=int(pos.size), vocab_size=int(vocab_size), parts=0, positions=pos)


def blob_layout(batch: SlotBatch) -> tuple[dict[str, int], int]:
    """Byte offset of every host section in the staging blob (16-byte aligned) and its size."""
    offsets, at = {}, 0
    for name, arr in batch.sections():
        offsets[name] = at
        at += (arr.nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
    return offsets, max(at, _ALIGN)


def write_blob(batch: SlotBatch, out: np.ndarray) -> dict[str, int]:
    """Write the host sections into `out` (uint8, at least the blob size); returns the offsets."""
    offsets, size = blob_layout(batch)
    if out.nbytes < size:
        raise ValueError("staging buffer too small")
    for name, arr in batch.sections():
        o = offsets[name]
        out[o:o + arr.nbytes] = arr.reshape(-1).view(np.uint8)
    return offsets


class SlotStager:
    """Pinned host and device staging buffers of one device, grown on demand.

    Before the pinned bytes are rewritten, the host waits for the previous call's H2D copy
    to have read them; a call's launch stream waits for the previous call's kernel before
    the device bytes are overwritten."""

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self.host: Tensor | None = None
        self.dev: Tensor | None = None
        self.copied: torch.cuda.Event | None = None
        self.consumed: torch.cuda.Event | None = None
        self.keep: list = []

    def stage(self, batch: SlotBatch, stream: torch.cuda.Stream) -> tuple[int, dict[str, int]]:
        """Pack `batch` into pinned memory and queue its copy on `stream`; returns the device base
        address and the section offsets."""
        _, size = blob_layout(batch)
        if self.copied is not None:
            self.copied.synchronize()
        if self.host is None or self.host.numel() < size:
            cap = 1 << max(16, (size - 1).bit_length())
            if self.consumed is not None:
                self.consumed.synchronize()
            self.host = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
            self.dev = torch.empty(cap, dtype=torch.uint8, device=self.device)
        offsets = write_blob(batch, self.host.numpy())
        if self.consumed is not None:
            stream.wait_event(self.consumed)
        with torch.cuda.stream(stream):
            self.dev[:size].copy_(self.host[:size], non_blocking=True)
            self.copied = torch.cuda.Event()
            self.copied.record(stream)
        return self.dev.data_ptr(), offsets

    def done(self, batch: SlotBatch, stream: torch.cuda.Stream) -> None:
        self.consumed = torch.cuda.Event()
        self.consumed.record(stream)
        self.keep = list(batch.keep)


def _vp(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def populate_args(buffers, batch: SlotBatch, base: int, offsets: dict[str, int]) -> _abi.PopulateArgs:
    """The C-ABI arguments of `batch` staged at device address `base` (section offsets
    `offsets`), written into `buffers`."""
    p = _abi.PopulateArgs()
    p.count = batch.count
    p.num_slots = buffers.bias.size(0)
    p.vocab_size = batch.vocab_size
    p.parts = batch.parts
    p.grammar_step = batch.grammar_step
    for name in offsets:
        setattr(p, name, base + offsets[name])
    for name in ("dense_context", "dense_decode"):
        v = getattr(batch, name)
        if isinstance(v, Tensor):
            setattr(p, name, v.data_ptr())
    rep = buffers.repetition
    for name, t in (("temperature", buffers.temperature), ("top_p", buffers.top_p), ("min_p", buffers.min_p),
                    ("top_k", buffers.top_k), ("top_logprobs", buffers.top_logprobs),
                    ("multiplicative", rep.multiplicative), ("frequency", rep.frequency),
                    ("presence", rep.presence), ("flags_target", buffers.flags.target),
                    ("flags_draft", buffers.flags.draft)):
        if t.dim() != 1 or t.stride(0) != 1:
            raise ValueError(f"`{name}` must be a contiguous vector")
        setattr(p, name, t.data_ptr())
    ctx, dec = rep.counts.context, rep.counts.decode
    if ctx.stride(1) != 1 or dec.stride(1) != 1 or ctx.stride(0) != dec.stride(0):
        raise ValueError("context and decode counts must be row-major with one row stride")
    p.context_counts, p.decode_counts, p.counts_stride = ctx.data_ptr(), dec.data_ptr(), ctx.stride(0)
    if buffers.bias.stride(1) != 1:
        raise ValueError("bias rows must be contiguous")
    p.bias, p.bias_stride = buffers.bias.data_ptr(), buffers.bias.stride(0)
    g = buffers.grammar
    if g.dim() != 3 or g.stride(2) != 1:
        raise ValueError("grammar must be [slots, timesteps, words] with contiguous words")
    p.grammar, p.timesteps = g.data_ptr(), g.size(1)
    p.grammar_slot_stride, p.grammar_step_stride = g.stride(0), g.stride(1)
    return p


def run_populate(args: _abi.PopulateArgs, device: torch.device, stream: torch.cuda.Stream) -> None:
    lib = _abi.load_library()
    with torch.cuda.device(device):
        _abi.check(lib.sonic_populate_slots(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream)), lib)


def launch_populate(buffers, batch: SlotBatch, stager: SlotStager, stream: torch.cuda.Stream | None = None) -> None:
    """Stage `batch` and write it into `buffers` (a SamplingBuffers on a CUDA device) on `stream`
    (default: the current stream)."""
    dev = buffers.device
    if dev.type != "cuda":
        raise ValueError("slot population runs on CUDA buffers only (no CPU fallback)")
    if batch.count == 0 or batch.parts == 0:
        return
    stream = stream or torch.cuda.current_stream(dev)
    base, off = stager.stage(batch, stream)
    run_populate(populate_args(buffers, batch, base, off), dev, stream)
    stager.done(batch, stream)
