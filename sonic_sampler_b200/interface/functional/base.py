"""Helpers of the functional rung (reference interface/functional/base.py:17-77)."""

from __future__ import annotations

import torch
from torch import Tensor

from sonic_sampler_b200 import ops

U32 = torch.uint32
I32 = torch.int32


def validate_count_update(flag: bool, buffer: Tensor | None) -> None:
    if flag and buffer is None:
        raise ValueError("`update_counts` is True but `decode_counts` is None")


def collapse_2d(value: Tensor) -> Tensor:
    return value.flatten(0, -2)


def resolve_workspace(buffer: Tensor | None, nbytes: int, device: torch.device) -> Tensor:
    """The caller's workspace when it is large enough, else a fresh zero-filled one.

    A workspace must come from this package (zero-filled once; the kernel leaves it zeroed).
    """
    if buffer is not None:
        if buffer.device != device:
            raise ValueError("scratchpad must live on the logits' device")
        if buffer.numel() * buffer.element_size() >= nbytes:
            return buffer
        raise ValueError(f"scratchpad holds {buffer.numel() * buffer.element_size()} bytes, "
                         f"the fused kernel needs {nbytes}")
    return ops.new_workspace(nbytes, device)
