"""The reference's own Triton implementation, run on the GPU, as a parity checker and as
timing context. Test and benchmark infrastructure only: no product path imports it.

The reference (tachyontrails/sonic-sampler 1.0.0) is pip-installed unmodified into
`baseline/_ref` at the repository root:

    python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
        --no-deps --target baseline/_ref <a copy of the reference checkout>

That folder is git-ignored but travels to the GPU box with the working tree. The one
dependency the image lacks, `cytoolz`, is stood in for by `tests/golden/_shim` (the only
function the reference imports from it, `thread_first`). Triton compiles the reference's
kernels for the local GPU on first use, exactly as in a deployment of the reference.
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
REF_DIR = ROOT / "baseline" / "_ref"
SHIM_DIR = Path(__file__).resolve().parent / "golden" / "_shim"


def unavailable() -> str | None:
    """None when the reference can be imported and run here, else the reason."""
    if not (REF_DIR / "sonic_sampler").is_dir():
        return f"reference not installed in {REF_DIR.relative_to(ROOT)}"
    try:
        import torch

        if not torch.cuda.is_available():
            return "the reference's Triton kernels need a CUDA device"
        load()
    except Exception as exc:  # pragma: no cover - reported to the caller
        return f"reference import failed: {type(exc).__name__}: {exc}"
    return None


def load():
    """Import the reference package (`sonic_sampler`) from baseline/_ref; returns a namespace
    with its interface classes and functional entry points."""
    for p in (str(SHIM_DIR), str(REF_DIR)):
        if p not in sys.path:
            sys.path.insert(0, p)
    iface = importlib.import_module("sonic_sampler.interface")
    fsing = importlib.import_module("sonic_sampler.interface.functional.singular")
    fmult = importlib.import_module("sonic_sampler.interface.functional.multistep")
    copy = importlib.import_module("sonic_sampler.ops.copy")

    class Ref:
        UnshardedFusedSingular = iface.UnshardedFusedSingular
        UnshardedFusedMultistep = iface.UnshardedFusedMultistep
        UnshardedBoundedTopK = iface.UnshardedBoundedTopK
        fused_singular = fsing.fused_singular
        fused_multistep = fmult.fused_multistep
        indexed_copy = copy.indexed_copy

    return Ref
