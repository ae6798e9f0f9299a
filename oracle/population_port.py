"""ORACLE -- test infrastructure only.

The reference's host population sequence of `SamplingBuffers.allocate` (core/buffer.py:
1239-1352), restated with torch: pinned host mirrors filled on the host (PinnedRelay.populate
and update_bias :707-764, RepetitionPenalties.populate :562-582, TokenCounts.populate
:422-432, Flags.update core/flags.py:543-572), then one `copy_` per slot and field
(transfer :1098-1135, RepetitionPenalties.transfer :584-604, TokenCounts.allocate :434-457,
step_grammar :1026-1052). bench.py times it beside the batched `sonic_populate_slots` path
(`--workload populate`); it is never the product path. Noise refresh is left out of both.
"""

from __future__ import annotations

from itertools import chain, repeat

import torch

BF16 = torch.bfloat16
I32 = torch.int32
I64 = torch.int64
U16 = torch.uint16


class PinnedMirrors:
    """The reference's pinned host mirrors for `slots` slots of `vocab` columns."""

    def __init__(self, slots: int, vocab: int):
        pin = dict(device="cpu", pin_memory=True)
        self.float_values = torch.empty((3, slots), dtype=BF16, **pin).T
        self.int_values = torch.empty((2, slots), dtype=I32, **pin).T
        self.bias = torch.zeros((slots, vocab), dtype=BF16, **pin)
        self.penalties = torch.empty((3, slots), dtype=BF16, **pin).T
        self.counts = torch.empty((slots, vocab), dtype=I32, **pin)
        self.flags = torch.empty((2, slots), dtype=U16, **pin).T


def allocate_port(buf, pinned: PinnedMirrors, encodings, multiplicative, frequency, presence, biases, temperature,
                  top_k, top_p, min_p, top_logprobs, positions, target, draft, bitmasks=None, stream=None) -> None:
    """One admission through the reference's sequence, on `buf` (a SamplingBuffers on CUDA)."""
    idx = torch.tensor(positions, dtype=I64)
    with torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream()):
        if bitmasks:
            for j, i in enumerate(positions):
                if bitmasks[j] is not None:
                    buf.grammar[i, 0].copy_(bitmasks[j], non_blocking=True)
        values = torch.tensor([list(map(int, target)), list(map(int, draft))], dtype=U16)
        pinned.flags.view(torch.int16).index_copy_(0, idx, values.T.view(torch.int16))
        for i in positions:
            buf.flags.packed[i].copy_(pinned.flags[i], non_blocking=True)
        pinned.float_values.index_copy_(0, idx, torch.tensor([temperature, top_p, min_p], dtype=BF16).T)
        pinned.int_values.index_copy_(0, idx, torch.tensor([top_k, top_logprobs], dtype=I32).T)
        if any(biases):
            targets, tokens, vals, lengths = zip(*((i, m.keys(), m.values(), len(m))
                                                   for i, m in zip(positions, biases) if m))
            tok = torch.tensor(list(chain.from_iterable(tokens)), dtype=I64)
            val = torch.tensor(list(chain.from_iterable(vals)), dtype=BF16)
            offs = torch.tensor(list(chain.from_iterable(map(repeat, targets, lengths))), dtype=I64)
            pinned.bias.index_fill_(0, torch.tensor(targets, dtype=I64), 0)
            pinned.bias.flatten().scatter_(0, offs.mul_(pinned.bias.size(-1)).add_(tok), val)
        pinned.penalties.index_copy_(0, idx, torch.tensor([multiplicative, frequency, presence], dtype=BF16).T)
        rep = buf.repetition
        for i in positions:
            rep.multiplicative[i].copy_(pinned.penalties[i, 0], non_blocking=True)
            rep.frequency[i].copy_(pinned.penalties[i, 1], non_blocking=True)
            rep.presence[i].copy_(pinned.penalties[i, 2], non_blocking=True)
        for i, e in zip(positions, encodings):
            pinned.counts[i].zero_().scatter_add_(0, e, torch.ones_like(e, dtype=I32))
        for i in positions:
            rep.counts.context[i].copy_(pinned.counts[i], non_blocking=True)
            rep.counts.decode[i].zero_()
        for i in positions:
            buf.bias[i].copy_(pinned.bias[i], non_blocking=True)
            buf.temperature[i].copy_(pinned.float_values[i, 0], non_blocking=True)
            buf.top_p[i].copy_(pinned.float_values[i, 1], non_blocking=True)
            buf.min_p[i].copy_(pinned.float_values[i, 2], non_blocking=True)
            buf.top_k[i].copy_(pinned.int_values[i, 0], non_blocking=True)
            buf.top_logprobs[i].copy_(pinned.int_values[i, 1], non_blocking=True)
