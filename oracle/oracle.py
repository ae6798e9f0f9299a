"""ORACLE -- test infrastructure only.

ctypes front end of the CPU restatement in sonic_oracle.c. Only tests/, __graft_entry__.smoke()
and bench.py's cpu_baseline leg use it, always as the checker next to the CUDA path, never
as the thing measured or shipped. It takes the same argument structs as the C ABI
(include/sonic_b200.h), built from HOST tensors.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "build" / "libsonic_oracle.so"

_LIB = None


def build(force: bool = False) -> Path:
    srcs = [ORACLE_DIR / "sonic_oracle.c", ORACLE_DIR.parent / "include" / "sonic_b200.h"]
    if force or not LIB_PATH.is_file() or any(p.stat().st_mtime > LIB_PATH.stat().st_mtime for p in srcs):
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "-B" if force else "build/libsonic_oracle.so"],
                       check=True)
    return LIB_PATH


def load() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        from sonic_sampler_b200._abi import MultistepArgs, SingularArgs, TopKArgs

        build()
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, argt in (
            ("oracle_fused_singular", SingularArgs),
            ("oracle_fused_multistep", MultistepArgs),
            ("oracle_bounded_topk", TopKArgs),
        ):
            fn = getattr(lib, name)
            fn.argtypes = [ctypes.POINTER(argt)]
            fn.restype = ctypes.c_int32
        for name in ("ox_exp", "ox_log"):
            fn = getattr(lib, name)
            fn.argtypes = [ctypes.c_float]
            fn.restype = ctypes.c_float
        lib.oracle_shard_candidates.argtypes = [ctypes.POINTER(SingularArgs), ctypes.c_void_p]
        lib.oracle_shard_candidates.restype = ctypes.c_int32
        lib.oracle_merge_candidates.argtypes = [ctypes.POINTER(SingularArgs), ctypes.c_void_p, ctypes.c_int32]
        lib.oracle_merge_candidates.restype = ctypes.c_int32
        lib.ox_philox_log_exponential.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64]
        lib.ox_philox_log_exponential.restype = ctypes.c_float
        _LIB = lib
    return _LIB


def _run(fn, args) -> None:
    status = fn(ctypes.byref(args))
    if status != 0:
        raise RuntimeError(f"oracle returned status {status}")


def fused_singular(args) -> None:
    _run(load().oracle_fused_singular, args)


def fused_multistep(args) -> None:
    _run(load().oracle_fused_multistep, args)


def bounded_topk(args) -> None:
    _run(load().oracle_bounded_topk, args)


def shard_candidates(args, keys) -> None:
    """Vocab-sharded step 1 of one rank: `keys` (contiguous uint64-sized int64 tensor
    [rows, 128]) receives each row's 128 best keys of this shard, global columns."""
    status = load().oracle_shard_candidates(ctypes.byref(args), keys.data_ptr())
    if status != 0:
        raise RuntimeError(f"oracle returned status {status}")


def merge_candidates(args, gathered, world: int) -> None:
    """Vocab-sharded step 3: merge gathered [world, rows, 128] keys and select."""
    status = load().oracle_merge_candidates(ctypes.byref(args), gathered.data_ptr(), world)
    if status != 0:
        raise RuntimeError(f"oracle returned status {status}")


def exp(x: float) -> float:
    return load().ox_exp(x)


def log(x: float) -> float:
    return load().ox_log(x)


def philox_log_exponential(seed: int, offset: int, slot: int, token: int) -> float:
    return load().ox_philox_log_exponential(seed, offset, slot, token)


def indexed_copy(source, target, indices, indicator) -> None:
    """CPU restatement of the reference's noise staging (ops/copy.py:21-55
    `indexed_copy_kernel`, launched by `indexed_copy` at :86-109): program (i, block) reads row
    j = indices[i] and, unless indicator[j] has the greedy bit 0x40, copies that row's
    flattened columns of `source` into the same offsets of `target`. Host tensors; `target`
    is updated in place."""
    src = source.reshape(source.size(0), -1)
    dst = target.view(target.size(0), -1)
    for i in range(indices.numel()):
        j = int(indices[i])
        if not (int(indicator[j]) & 0x40):
            dst[j].copy_(src[j])


def populate_slots(batch, dest: dict) -> None:
    """CPU restatement of slot population from a packed call (the arrays of
    sonic_populate_slots; `batch` is a core.population.SlotBatch). `dest` holds host tensors
    named like the SamplingBuffers fields: temperature, top_p, min_p, top_k, top_logprobs,
    multiplicative, frequency, presence, flags_target, flags_draft, context, decode, bias,
    grammar [slots, T, W]. Updated in place, slot by slot, in the reference's terms:

    - scalars and indicators: PinnedRelay.populate + transfer (core/buffer.py:738-764,
      1098-1135), RepetitionPenalties.populate + transfer (:562-604), Flags.update
      (core/flags.py:543-572);
    - prompt histogram: pinned row zeroed and `scatter_add_` of ones at the prompt ids, copied to
      the context counts; decode counts zeroed (TokenCounts.populate + allocate, :422-457);
      dense counts copied (TokenCounts.update, :395-420);
    - bias: row zeroed, then `scatter_` of the slot's values at its token ids
      (PinnedRelay.update_bias, :707-736);
    - grammar: `copy_` of the bitmask into step `grammar_step`, or into every step of the slot
      (step_grammar, :1026-1052)."""
    import torch

    from sonic_sampler_b200.core import population as P

    V = batch.vocab_size
    bf = lambda a: torch.from_numpy(a.astype("int16")).view(torch.bfloat16)  # noqa: E731
    for i in range(batch.count):
        s = int(batch.positions[i])
        if batch.parts & P.SCALARS:
            f = bf(batch.values_bf16[i])
            dest["temperature"][s], dest["top_p"][s], dest["min_p"][s] = f[0], f[1], f[2]
            dest["multiplicative"][s], dest["frequency"][s], dest["presence"][s] = f[3], f[4], f[5]
            dest["top_k"][s] = int(batch.values_i32[i, 0])
            dest["top_logprobs"][s] = int(batch.values_i32[i, 1])
            dest["flags_target"][s] = int(batch.indicators[i, 0])
            dest["flags_draft"][s] = int(batch.indicators[i, 1])
        if batch.parts & P.HISTOGRAM:
            toks = torch.from_numpy(batch.tokens[batch.token_offsets[i]:batch.token_offsets[i + 1]].astype("int64"))
            row = torch.zeros(V, dtype=torch.int32)
            row.scatter_add_(0, toks, torch.ones_like(toks, dtype=torch.int32))
            dest["context"][s, :V] = row
            dest["decode"][s, :V] = 0
        elif batch.parts & P.DENSE_COUNTS:
            dc, dd = batch.dense_context, batch.dense_decode
            dc = dc.cpu().numpy() if isinstance(dc, torch.Tensor) else dc
            dd = dd.cpu().numpy() if isinstance(dd, torch.Tensor) else dd
            dest["context"][s, :V] = torch.from_numpy(dc[i].copy())
            dest["decode"][s, :V] = torch.from_numpy(dd[i].copy())
        if batch.parts & P.BIAS:
            row = torch.zeros(V, dtype=torch.bfloat16)
            if batch.bias_offsets is not None:
                b0, b1 = int(batch.bias_offsets[i]), int(batch.bias_offsets[i + 1])
                row.scatter_(0, torch.from_numpy(batch.bias_tokens[b0:b1].astype("int64")),
                             bf(batch.bias_values[b0:b1]))
            dest["bias"][s, :V] = row
        if batch.parts & P.GRAMMAR and int(batch.grammar_rows[i]) >= 0:
            r0, n = int(batch.grammar_rows[i]), int(batch.grammar_steps[i])
            g = dest["grammar"].view(torch.int32)
            steps = [batch.grammar_step] if batch.grammar_step >= 0 else range(g.size(1))
            for k, t in enumerate(steps):
                g[s, t] = torch.from_numpy(batch.grammar_words[r0 + (k if n > 1 else 0)].view("int32").copy())
