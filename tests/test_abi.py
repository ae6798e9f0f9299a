"""The C-ABI library loads on a machine without a GPU, exports exactly what
include/sonic_b200.h declares, and validates arguments on the host before any launch."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from sonic_sampler_b200 import _abi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "sonic_b200.h"


@pytest.fixture(scope="module")
def lib():
    from sonic_sampler_b200 import build

    build.build()
    return _abi.load_library()


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(sonic_\w+)\s*\(", text))


def test_header_declares_the_python_mirror():
    assert declared_functions() == set(_abi.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == declared_functions()
    for name in declared_functions():
        assert hasattr(lib, name)


def test_abi_version(lib):
    assert lib.sonic_abi_version() == _abi.ABI_VERSION


def test_struct_layout_matches_header():
    """The ctypes mirror names every field of the header's structs in header order."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for cname, pyt in (("SonicSamplingParams", _abi.SamplingParams), ("SonicSingularArgs", _abi.SingularArgs),
                       ("SonicMultistepArgs", _abi.MultistepArgs), ("SonicTopKArgs", _abi.TopKArgs),
                       ("SonicPopulateArgs", _abi.PopulateArgs)):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (cname, cname), text, flags=re.S).group(1)
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            fields.append(re.findall(r"(\w+)\s*$", decl)[0])
        assert fields == [f for f, _ in pyt._fields_], cname


def test_workspace_queries_are_pure(lib):
    a = _abi.SingularArgs()
    a.rows, a.vocab_size = 64, 128256
    n1 = lib.sonic_fused_singular_workspace_size(ctypes.byref(a))
    n2 = lib.sonic_fused_singular_workspace_size(ctypes.byref(a))
    assert n1 == n2 > 64 * 128 * 8
    m = _abi.MultistepArgs()
    m.batch_size, m.lookahead, m.vocab_size = 32, 4, 128256
    assert lib.sonic_fused_multistep_workspace_size(ctypes.byref(m)) > 32 * 5 * 128 * 8
    t = _abi.TopKArgs()
    t.rows, t.vocab_size = 8, 32000
    assert lib.sonic_bounded_topk_workspace_size(ctypes.byref(t)) > 0
    assert lib.sonic_fused_singular_workspace_size(None) == 0


def _status(lib, fn, args):
    return getattr(lib, fn)(ctypes.byref(args), None), lib.sonic_last_error().decode()


def test_host_validation_without_gpu(lib):
    """Bad arguments are rejected before any CUDA call (so these run on CPU machines)."""
    a = _abi.SingularArgs()
    a.rows, a.vocab_size, a.block_n = 4, 1000, 1000
    st, msg = _status(lib, "sonic_fused_singular", a)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "block_n" in msg
    a.block_n = 1024
    st, msg = _status(lib, "sonic_fused_singular", a)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "indicators" in msg
    a.vocab_size = 64
    st, msg = _status(lib, "sonic_fused_singular", a)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "vocab_size" in msg
    a.rows = 0
    assert _status(lib, "sonic_fused_singular", a)[0] == _abi.SONIC_OK  # empty batch: no-op

    m = _abi.MultistepArgs()
    m.batch_size, m.lookahead, m.vocab_size, m.block_n = 2, 16, 4096, 1024
    st, msg = _status(lib, "sonic_fused_multistep", m)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "lookahead" in msg

    t = _abi.TopKArgs()
    t.rows, t.vocab_size, t.k = 2, 4096, 48
    st, msg = _status(lib, "sonic_bounded_topk", t)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "power of two" in msg


def test_static_entry_validates_before_touching_scratch(lib):
    """sonic_fused_singular_static checks every argument before it sizes, carves or clears its
    scratch: bad shapes return SONIC_ERR_INVALID_ARGUMENT and an oversize call
    SONIC_ERR_WORKSPACE, with no CUDA call made (so this runs on machines without a GPU)."""
    a = _abi.SingularArgs()
    a.rows, a.vocab_size, a.block_n = -1, 128256, 4096
    st, msg = _status(lib, "sonic_fused_singular_static", a)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "rows" in msg
    a.rows, a.vocab_size = 4, 0
    st, msg = _status(lib, "sonic_fused_singular_static", a)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "vocab_size" in msg
    assert lib.sonic_fused_singular_workspace_size(ctypes.byref(a)) == 0  # no division by the empty vocabulary
    # arguments that pass every check but need more than the 4 MiB scratch; the pointers are
    # never dereferenced because the size check fails first
    fake = 1 << 20
    a.rows, a.vocab_size = 4096, 128256
    a.params.indicators = a.tokens = a.gumbel = a.logits = fake
    st, msg = _status(lib, "sonic_fused_singular_static", a)
    assert st == _abi.SONIC_ERR_WORKSPACE and "static scratch" in msg


def test_update_counts_without_decode_counts_message(lib):
    """Same message as the reference's runtime check (functional/base.py:34-38)."""
    import torch

    from sonic_sampler_b200.interface.functional.singular import prepare_singular

    with pytest.raises(ValueError, match="`update_counts` is True but `decode_counts` is None"):
        prepare_singular(torch.zeros(2, 4096, dtype=torch.bfloat16), torch.zeros(2, dtype=torch.uint16),
                         update_counts=True)


def test_populate_host_validation_without_gpu(lib):
    """sonic_populate_slots rejects inconsistent arguments before launching."""
    p = _abi.PopulateArgs()
    assert _status(lib, "sonic_populate_slots", p)[0] == _abi.SONIC_OK  # nothing to do
    p.count, p.parts = 2, _abi.POPULATE_HISTOGRAM | _abi.POPULATE_DENSE_COUNTS
    st, msg = _status(lib, "sonic_populate_slots", p)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "exclusive" in msg
    p.parts = 0x40
    st, msg = _status(lib, "sonic_populate_slots", p)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "unknown" in msg
    p.parts = _abi.POPULATE_SCALARS
    st, msg = _status(lib, "sonic_populate_slots", p)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "positions" in msg
    p.num_slots, p.vocab_size, p.positions = 4, 1000, 16
    st, msg = _status(lib, "sonic_populate_slots", p)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "SCALARS" in msg
    p.parts = _abi.POPULATE_GRAMMAR
    p.grammar = p.grammar_rows = p.grammar_steps = p.grammar_words = 16
    p.timesteps, p.grammar_step = 2, 2
    st, msg = _status(lib, "sonic_populate_slots", p)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "grammar_step" in msg
    p.grammar_step, p.grammar_step_stride, p.grammar_slot_stride = -1, 32, 40
    st, msg = _status(lib, "sonic_populate_slots", p)
    assert st == _abi.SONIC_ERR_INVALID_ARGUMENT and "strides" in msg
    p.count = -1
    assert _status(lib, "sonic_populate_slots", p)[0] == _abi.SONIC_ERR_INVALID_ARGUMENT
