"""Run the reference's Triton kernels on the CPU through Triton's interpreter.

Used only by make_golden.py, in a container that has the reference sources. It changes
nothing in the reference; it adjusts Triton's interpreter (and rebinds three names inside
the already-imported reference modules) so that bf16 behaves as a real 16-bit float type:

1. bf16 tensors become `ml_dtypes.bfloat16` numpy arrays (arithmetic in fp32, rounded to
   bf16 after each operation) instead of raw uint16, and bf16 <-> fp32 casts round to
   nearest even;
2. `fast_expf` / `fast_logf` (libdevice, absent from the interpreter) are rebound to
   `tl.exp` / `tl.log`, i.e. numpy's exp / log;
3. the reference's `to_scalar` builtin is rebound to a one-element `tl.sum`.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

if "SONIC_REFERENCE_SRC" not in os.environ:
    raise RuntimeError("set SONIC_REFERENCE_SRC to the reference checkout's src/ directory "
                       "(the sonic_sampler package of tachyontrails/sonic-sampler)")
REFERENCE_SRC = Path(os.environ["SONIC_REFERENCE_SRC"])
sys.path.insert(0, str(Path(__file__).resolve().parent / "_shim"))
sys.path.insert(0, str(REFERENCE_SRC))

import ml_dtypes  # noqa: E402
import numpy as np  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402
import triton.runtime.interpreter as interp  # noqa: E402

_BF16_NP = np.dtype(ml_dtypes.bfloat16)
_original_np_dtype = interp._get_np_dtype
_original_convert = interp._convert_float


def _np_dtype(t):
    scalar = t.element_ty if isinstance(t, tl.block_type) else t
    return _BF16_NP if scalar == tl.bfloat16 else _original_np_dtype(t)


def _convert(x, src, dst, rounding_mode):
    if {src, dst} <= {tl.bfloat16, tl.float32}:
        s = _BF16_NP if src == tl.bfloat16 else np.dtype(np.float32)
        d = _BF16_NP if dst == tl.bfloat16 else np.dtype(np.float32)
        return np.frombuffer(x.tobytes(), dtype=s).astype(d).reshape(x.shape)
    return _original_convert(x, src, dst, rounding_mode)


interp._get_np_dtype = _np_dtype
interp._convert_float = _convert
interp.InterpreterBuilder.get_bf16 = lambda self, v: interp.TensorHandle(np.array([v], dtype=_BF16_NP), tl.bfloat16)


@triton.jit
def _exp(x):
    return tl.exp(x)


@triton.jit
def _log(x):
    return tl.log(x)


@triton.jit
def _scalar(x):
    return tl.sum(x, axis=0)


import sonic_sampler.ops.base as _ref_base  # noqa: E402
import sonic_sampler.ops.multistep as _ref_multistep  # noqa: E402
import sonic_sampler.ops.singular as _ref_singular  # noqa: E402
import sonic_sampler.ops.verify as _ref_verify  # noqa: E402

for _module in (_ref_base, _ref_singular, _ref_multistep, _ref_verify):
    if hasattr(_module, "fast_expf"):
        _module.fast_expf = _exp
    if hasattr(_module, "fast_logf"):
        _module.fast_logf = _log
_ref_singular.to_scalar = _scalar
