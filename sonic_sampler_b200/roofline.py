"""Algorithmic HBM bytes of one fused singular call (the roofline numerator).

Each input a row's indicator bits require is counted once per row, at its full width;
the Gumbel noise counts as the 128 candidate entries the algorithm gathers; outputs count
once. Workspace and intermediates do not count. For the config-2 row (all processors,
V = 128256) the inputs come to 256,512 (logits) + 16,032 (grammar) + 513,024 (context
counts) + 513,024 (decode counts) + 256,512 (bias) + 256 (noise) = 1,555,360 bytes.
"""

from __future__ import annotations

MAXK = 128


def singular_row_bytes(indicator: int, vocab: int, *, logprobs: bool = False, top_z: int = 0,
                       has_grammar: bool = True, has_counts: bool = True, has_bias: bool = True) -> int:
    n = 2 * vocab  # bf16 logits
    if indicator & 0x1F:
        if has_grammar and indicator & 0x1:
            n += 4 * ((vocab + 31) // 32)
        if has_counts and indicator & 0xE:
            n += 4 * vocab  # decode counts
            if indicator & 0x2:
                n += 4 * vocab  # context counts
        if has_bias and indicator & 0x10:
            n += 2 * vocab
    greedy = bool(indicator & 0x40)
    if not greedy:
        n += 2 * MAXK  # gathered noise of the candidates
    n += 4  # token
    if logprobs and not greedy:
        n += 2 + 6 * top_z
    return n


def singular_call_bytes(indicators, vocab: int, **kw) -> int:
    return sum(singular_row_bytes(int(i), vocab, **kw) for i in indicators)


def multistep_request_bytes(indicator: int, vocab: int, steps: int, **kw) -> int:
    """Per request: logits and grammar per step; counts and bias once per request."""
    per_step = 2 * vocab
    if indicator & 0x1 and kw.get("has_grammar", True):
        per_step += 4 * ((vocab + 31) // 32)
    n = steps * per_step
    if indicator & 0xE:
        n += 4 * vocab * (2 if indicator & 0x2 else 1)
    if indicator & 0x10:
        n += 2 * vocab
    if not indicator & 0x40:
        n += 2 * MAXK + 4 * MAXK  # noise + draft probabilities gathered at the rejected step
    return n + 4 * steps + 4


def topk_row_bytes(vocab: int, k: int, elem: int = 2, index: int = 4) -> int:
    return elem * vocab + k * (elem + index)
