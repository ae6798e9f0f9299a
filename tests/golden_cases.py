"""Replays the golden cases of tests/golden/*.pt through the package's argument
marshalling, on host tensors (oracle) or device tensors (CUDA), and compares the outputs
with the reference's. Shared by the CPU oracle tests and the GPU parity tests."""

from __future__ import annotations

from pathlib import Path

import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
F32 = torch.float32
LOGPROB_ATOL = 1e-5  # fp32 logprobs vs the reference


def load(name: str) -> dict:
    return torch.load(GOLDEN / f"{name}.pt", weights_only=True)


def to(d: dict, device) -> dict:
    return {k: (v.to(device).clone() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def slots_of(inputs: dict, rows: int) -> list[int]:
    sm = inputs.get("slot_mapping")
    return list(range(rows)) if sm is None else [int(v) for v in sm.cpu()]


def singular_kwargs(case: dict, device) -> dict:
    inp = to(case["inputs"], device)
    meta = case["meta"]
    kw = dict(inp)
    if "grammar_full" in kw:
        kw["grammar"] = kw.pop("grammar_full")[:, meta["timestep"]]
    kw.update(block_n=meta["block_n"], enable_pdl=False)
    return kw
