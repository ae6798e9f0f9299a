"""ctypes mirror of include/sonic_b200.h and the loader of the in-tree CUDA library.

The C ABI is the drop-in boundary: every GPU call of this package goes through
`libsonic_b200.so` with raw device pointers, strides and an explicit CUDA stream. There is
no CPU or PyTorch fallback; when the library is missing the import of the calling module
fails with a message that says how to build it.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

ABI_VERSION = 4
MAX_K = 128
MAX_LOOKAHEAD = 15

# status codes
SONIC_OK = 0
SONIC_ERR_INVALID_ARGUMENT = 1
SONIC_ERR_UNSUPPORTED = 2
SONIC_ERR_WORKSPACE = 3
SONIC_ERR_CUDA = 4

# dtype tags
DT_BF16 = 0
DT_F32 = 1
DT_I32 = 2
DT_I64 = 3

# call flags
FLAG_PDL = 1 << 0
FLAG_PREFILL = 1 << 1
FLAG_UPDATE_COUNTS = 1 << 2
FLAG_LOGPROBS = 1 << 3
FLAG_PROBABILITIES = 1 << 4
FLAG_PHILOX = 1 << 5
# diagnostics: every ring wait of the call first runs out (tests of the bounded-wait error path)
FLAG_DEBUG_STALL_RING = 1 << 15

# bits of a workspace's device error word (sonic_workspace_error)
DEVICE_ERR_WAIT = 1 << 0

# parts of sonic_populate_slots
POPULATE_SCALARS = 0x1
POPULATE_HISTOGRAM = 0x2
POPULATE_DENSE_COUNTS = 0x4
POPULATE_BIAS = 0x8
POPULATE_GRAMMAR = 0x10

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64


class SamplingParams(ctypes.Structure):
    _fields_ = [
        ("indicators", _vp),
        ("slot_mapping", _vp),
        ("slot_dtype", _i32),
        ("num_slots", _i32),
        ("grammar", _vp),
        ("grammar_stride", _i64),
        ("context_counts", _vp),
        ("decode_counts", _vp),
        ("counts_stride", _i64),
        ("repetition", _vp),
        ("frequency", _vp),
        ("presence", _vp),
        ("bias", _vp),
        ("bias_stride", _i64),
        ("temperature", _vp),
        ("top_k", _vp),
        ("top_p", _vp),
        ("min_p", _vp),
        ("top_logprobs", _vp),
    ]


class SingularArgs(ctypes.Structure):
    _fields_ = [
        ("rows", _i32),
        ("vocab_size", _i32),
        ("block_n", _i32),
        ("lookahead", _i32),
        ("shard_offset", _i32),
        ("max_top_logprobs", _i32),
        ("target_vocab", _i32),
        ("flags", _u32),
        ("logits", _vp),
        ("logits_dtype", _i32),
        ("logits_stride", _i64),
        ("params", SamplingParams),
        ("d2t", _vp),
        ("d2t_dtype", _i32),
        ("drafted_tokens", _vp),
        ("drafted_stride", _i64),
        ("gumbel", _vp),
        ("gumbel_stride", _i64),
        ("philox_seed", _u64),
        ("philox_offset", _u64),
        ("tokens", _vp),
        ("tokens_stride", _i64),
        ("logprobs", _vp),
        ("logprobs_stride", _i64),
        ("logprobs_dtype", _i32),
        ("top_logprob_values", _vp),
        ("top_logprob_tokens", _vp),
        ("top_stride", _i64),
        ("probabilities", _vp),
        ("probabilities_dtype", _i32),
        ("probabilities_stride", _i64),
        ("workspace", _vp),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class MultistepArgs(ctypes.Structure):
    _fields_ = [
        ("batch_size", _i32),
        ("lookahead", _i32),
        ("vocab_size", _i32),
        ("block_n", _i32),
        ("shard_offset", _i32),
        ("max_top_logprobs", _i32),
        ("flags", _u32),
        ("total_rows", _i32),
        ("logits", _vp),
        ("logits_dtype", _i32),
        ("logits_stride", _i64),
        ("cu_seqlens", _vp),
        ("params", SamplingParams),
        ("drafted_tokens", _vp),
        ("draft_probs", _vp),
        ("draft_dtype", _i32),
        ("draft_stride", _i64),
        ("draft_step_stride", _i64),
        ("uniform", _vp),
        ("uniform_stride", _i64),
        ("gumbel", _vp),
        ("gumbel_stride", _i64),
        ("gumbel_step_stride", _i64),
        ("values", _vp),
        ("indices", _vp),
        ("tokens", _vp),
        ("offsets", _vp),
        ("logprobs", _vp),
        ("logprobs_dtype", _i32),
        ("top_logprob_values", _vp),
        ("top_logprob_tokens", _vp),
        ("top_stride", _i64),
        ("workspace", _vp),
        ("workspace_bytes", ctypes.c_size_t),
        ("philox_seed", ctypes.c_uint64),
        ("philox_offset", ctypes.c_uint64),
    ]


class TopKArgs(ctypes.Structure):
    _fields_ = [
        ("rows", _i32),
        ("vocab_size", _i32),
        ("k", _i32),
        ("block_n", _i32),
        ("flags", _u32),
        ("logits", _vp),
        ("logits_dtype", _i32),
        ("logits_stride", _i64),
        ("values", _vp),
        ("values_dtype", _i32),
        ("indices", _vp),
        ("indices_dtype", _i32),
        ("workspace", _vp),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class PopulateArgs(ctypes.Structure):
    _fields_ = [
        ("count", _i32),
        ("num_slots", _i32),
        ("vocab_size", _i64),
        ("parts", _u32),
        ("timesteps", _i32),
        ("grammar_step", _i32),
        ("_pad0", _i32),
        ("positions", _vp),
        ("values_bf16", _vp),
        ("values_i32", _vp),
        ("indicators", _vp),
        ("token_offsets", _vp),
        ("tokens", _vp),
        ("dense_context", _vp),
        ("dense_decode", _vp),
        ("bias_offsets", _vp),
        ("bias_tokens", _vp),
        ("bias_values", _vp),
        ("grammar_rows", _vp),
        ("grammar_steps", _vp),
        ("grammar_words", _vp),
        ("temperature", _vp),
        ("top_p", _vp),
        ("min_p", _vp),
        ("top_k", _vp),
        ("top_logprobs", _vp),
        ("multiplicative", _vp),
        ("frequency", _vp),
        ("presence", _vp),
        ("flags_target", _vp),
        ("flags_draft", _vp),
        ("context_counts", _vp),
        ("decode_counts", _vp),
        ("counts_stride", _i64),
        ("bias", _vp),
        ("bias_stride", _i64),
        ("grammar", _vp),
        ("grammar_slot_stride", _i64),
        ("grammar_step_stride", _i64),
    ]


#: every symbol include/sonic_b200.h declares
EXPORTED_SYMBOLS = (
    "sonic_fused_singular_workspace_size",
    "sonic_fused_multistep_workspace_size",
    "sonic_bounded_topk_workspace_size",
    "sonic_fused_singular",
    "sonic_fused_multistep",
    "sonic_bounded_topk",
    "sonic_fused_singular_static",
    "sonic_workspace_error",
    "sonic_shard_candidates",
    "sonic_merge_candidates",
    "sonic_indexed_copy",
    "sonic_populate_slots",
    "sonic_abi_version",
    "sonic_last_error",
)

PACKAGE_DIR = Path(__file__).resolve().parent
LIB_PATH = PACKAGE_DIR / "_lib" / "libsonic_b200.so"


def _declare(lib: ctypes.CDLL) -> ctypes.CDLL:
    for name, argt in (
        ("sonic_fused_singular_workspace_size", SingularArgs),
        ("sonic_fused_multistep_workspace_size", MultistepArgs),
        ("sonic_bounded_topk_workspace_size", TopKArgs),
    ):
        fn = getattr(lib, name)
        fn.argtypes = [ctypes.POINTER(argt)]
        fn.restype = ctypes.c_size_t
    for name, argt in (
        ("sonic_fused_singular", SingularArgs),
        ("sonic_fused_multistep", MultistepArgs),
        ("sonic_bounded_topk", TopKArgs),
        ("sonic_fused_singular_static", SingularArgs),
    ):
        fn = getattr(lib, name)
        fn.argtypes = [ctypes.POINTER(argt), _vp]
        fn.restype = _i32
    lib.sonic_workspace_error.argtypes = [_vp, ctypes.POINTER(ctypes.c_uint32), _vp]
    lib.sonic_workspace_error.restype = _i32
    lib.sonic_shard_candidates.argtypes = [ctypes.POINTER(SingularArgs), _vp, _vp]
    lib.sonic_shard_candidates.restype = _i32
    lib.sonic_merge_candidates.argtypes = [ctypes.POINTER(SingularArgs), _vp, _i32, _vp]
    lib.sonic_merge_candidates.restype = _i32
    lib.sonic_indexed_copy.argtypes = [_vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _i32, _vp, _i32, _i32,
                                       _vp, _vp]
    lib.sonic_indexed_copy.restype = _i32
    lib.sonic_populate_slots.argtypes = [ctypes.POINTER(PopulateArgs), _vp]
    lib.sonic_populate_slots.restype = _i32
    lib.sonic_abi_version.argtypes = []
    lib.sonic_abi_version.restype = _i32
    lib.sonic_last_error.argtypes = []
    lib.sonic_last_error.restype = ctypes.c_char_p
    return lib


_LIB: ctypes.CDLL | None = None


def load_library(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the CUDA library. Raises RuntimeError when it is not built."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    # SONIC_B200_LIBRARY selects another build of the same ABI (the phase-stamp variant)
    target = Path(path) if path is not None else Path(os.environ.get("SONIC_B200_LIBRARY", LIB_PATH))
    if not target.is_file():
        raise RuntimeError(
            f"{target} is missing: build the CUDA extension first "
            "(python -m sonic_sampler_b200.build, or __graft_entry__.build())"
        )
    lib = _declare(ctypes.CDLL(str(target)))
    if lib.sonic_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{target} has ABI {lib.sonic_abi_version()}, expected {ABI_VERSION}")
    if path is None:
        _LIB = lib
    return lib


class SonicError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"sonic status {status}: {message}")
        self.status = status


def check(status: int, lib: ctypes.CDLL) -> None:
    if status != SONIC_OK:
        message = lib.sonic_last_error().decode(errors="replace")
        if status == SONIC_ERR_INVALID_ARGUMENT:
            raise ValueError(message)
        raise SonicError(status, message)
