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
