"""Generate the golden vectors that pin the CPU oracle to the reference implementation.

Runs the reference's own Triton kernels (tachyontrails/sonic-sampler, its functional API
`fused_singular` / `fused_multistep` and `UnshardedBoundedTopK`) on the CPU through Triton's
interpreter (see _reference_harness.py), on small seeded inputs, and saves inputs and
outputs to tests/golden/*.pt. Needs the reference sources (environment variable
SONIC_REFERENCE_SRC, the reference checkout's src/ directory); the GPU box never runs this
file.

    python tests/golden/make_golden.py            # all cases
    python tests/golden/make_golden.py topk_bf16  # one case

Logprob outputs are requested in fp32 (the reference's output containers are switched
from bf16 to fp32 for this run) so that they can be compared in fp32.
"""

from __future__ import annotations

import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import _reference_harness  # noqa: E402,F401  (must precede the reference imports)
import torch  # noqa: E402

import sonic_sampler.base.sampler as ref_sampler  # noqa: E402
from sonic_sampler.interface.base import TopKStrategy  # noqa: E402
from sonic_sampler.interface.functional import fused_multistep, fused_singular  # noqa: E402
from sonic_sampler.interface.topk import UnshardedBoundedTopK  # noqa: E402

BF16 = torch.bfloat16
I32 = torch.int32
RADIX = TopKStrategy(radix=True)

# fp32 logprob outputs for this run (see module docstring)
ref_sampler.BF16 = torch.float32


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def peaked_logits(rows: int, vocab: int, seed: int, sigma: float = 3.0, peaks: int = 4, lift: float = 12.0,
                  ties: bool = True) -> torch.Tensor:
    g = gen(seed)
    x = torch.randn(rows, vocab, generator=g) * sigma
    for r in range(rows):
        x[r, torch.randperm(vocab, generator=g)[:peaks]] += lift
    x = x.to(BF16)
    if ties:
        # exact ties inside and across tiles: copy a few large values to other columns
        for r in range(rows):
            src = torch.topk(x[r].float(), 6).indices
            dst = torch.randperm(vocab, generator=g)[:6]
            x[r, dst] = x[r, src]
    return x


def slot_params(slots: int, vocab: int, timesteps: int, seed: int, greedy_slots=(), all_bits: bool = True):
    """Heterogeneous per-slot parameters in the reference's SamplingBuffers dtypes."""
    g = gen(seed)
    words = (vocab + 31) // 32
    temperature = (torch.rand(slots, generator=g) + 0.5).to(BF16)
    top_k = torch.tensor([(128, 20, 50)[i % 3] for i in range(slots)], dtype=I32)
    top_p = (0.8 + 0.2 * torch.rand(slots, generator=g)).to(BF16)
    min_p = torch.tensor([(0.0, 0.05)[i % 2] for i in range(slots)], dtype=BF16)
    rep = torch.full((slots,), 1.1, dtype=BF16)
    freq = torch.full((slots,), 0.2, dtype=BF16)
    pres = torch.full((slots,), 0.3, dtype=BF16)
    top_logprobs = torch.tensor([(3, 5, 1, 0)[i % 4] for i in range(slots)], dtype=I32)
    bias = torch.zeros(slots, vocab, dtype=BF16)
    context = torch.zeros(slots, vocab, dtype=I32)
    decode = torch.zeros(slots, vocab, dtype=I32)
    for s in range(slots):
        cols = torch.randperm(vocab, generator=g)[:16]
        bias[s, cols] = (torch.rand(16, generator=g) * 10 - 5).to(BF16)
        hist = torch.randint(0, vocab, (512,), generator=g)
        context[s] += torch.bincount(hist, minlength=vocab).to(I32)
        recent = torch.randint(0, vocab, (64,), generator=g)
        decode[s] += torch.bincount(recent, minlength=vocab).to(I32)
        rep_cols = torch.randperm(vocab, generator=g)[:8]
        decode[s, rep_cols] += torch.randint(2, 8, (8,), generator=g).to(I32)
    bits = torch.where(torch.rand(slots, timesteps, words * 32, generator=g) < 0.3, 1, 0).to(torch.int64)
    words64 = (bits.view(slots, timesteps, words, 32) << torch.arange(32)).sum(-1)
    grammar = (words64 - (words64 >= 2**31).to(torch.int64) * 2**32).to(torch.int32).view(torch.uint32)
    indicators = []
    for s in range(slots):
        ind = 0x1 | 0x2 | 0x4 | 0x8 | 0x10 | 0x20 if all_bits else 0x20
        ind |= 0x80 if int(top_k[s]) < 128 else 0
        ind |= 0x100 | (0x200 if float(min_p[s]) > 0 else 0)
        ind |= 0x400 if int(top_logprobs[s]) > 0 else 0
        if s in greedy_slots:
            ind = (ind & 0x3F) | 0x40
        indicators.append(ind)
    # vary the processor mix across slots
    for s in range(slots):
        if s % 5 == 3:
            indicators[s] &= ~0x1
        if s % 4 == 2:
            indicators[s] &= ~0x2
        if s % 6 == 5:
            indicators[s] &= ~(0x1F)
    return dict(
        indicators=torch.tensor(indicators, dtype=torch.uint16),
        grammar=grammar,
        context_counts=context,
        decode_counts=decode,
        repetition_penalties=rep,
        frequency_penalties=freq,
        presence_penalties=pres,
        logit_bias=bias,
        temperature=temperature,
        top_k=top_k,
        top_p=top_p,
        min_p=min_p,
        top_k_logprobs=top_logprobs,
    )


def gumbel(shape, seed: int) -> torch.Tensor:
    return torch.empty(shape).exponential_(1.0, generator=gen(seed)).log_().to(BF16)


def save(name: str, inputs: dict, outputs: dict, meta: dict) -> None:
    path = HERE / f"{name}.pt"
    torch.save({"inputs": inputs, "outputs": outputs, "meta": meta}, path)
    size = path.stat().st_size
    print(f"  wrote {path.name} ({size / 1024:.0f} KiB)")


# --------------------------------------------------------------------------------------------
# cases
# --------------------------------------------------------------------------------------------


def case_topk_bf16():
    """UnshardedBoundedTopK, k = 32 and 128, radix strategy, with exact ties."""
    rows, vocab = 4, 8192
    x = peaked_logits(rows, vocab, seed=11, sigma=2.0, peaks=8, lift=10.0)
    out = {}
    for k in (32, 128):
        topk = UnshardedBoundedTopK.initialize(vocab, block_size=1024, batch_size=rows, k=k, pdl=False).clear()
        values, indices = topk(x, strategy=RADIX)
        # the reference stores row r's k results at flat offset r*k
        out[f"values_k{k}"] = topk.values.reshape(-1)[: rows * k].clone()
        out[f"indices_k{k}"] = topk.indices.reshape(-1)[: rows * k].clone()
    save("topk_bf16", {"logits": x}, out, {"block_n": 1024, "strategy": "radix"})


def case_topk_bitonic():
    """Same semantics through the reference's default (bitonic) strategy."""
    rows, vocab, k = 2, 2048, 128
    x = peaked_logits(rows, vocab, seed=12, sigma=2.0, peaks=8, lift=10.0)
    topk = UnshardedBoundedTopK.initialize(vocab, block_size=1024, batch_size=rows, k=k, pdl=False).clear()
    topk(x, strategy=TopKStrategy())
    save("topk_bitonic", {"logits": x},
         {"values": topk.values.reshape(-1)[: rows * k].clone(), "indices": topk.indices.reshape(-1)[: rows * k].clone()},
         {"block_n": 1024, "strategy": "bitonic", "k": k})


def case_singular_mixed():
    """Autoregressive step: heterogeneous processors, greedy + stochastic rows, slot mapping,
    decode-count update, fp32 logprobs + top-Z; one greedy row with a cross-tile tie."""
    slots, rows, vocab, block_n = 8, 6, 8192, 1024
    p = slot_params(slots, vocab, 1, seed=21, greedy_slots=(1, 6))
    x = peaked_logits(rows, vocab, seed=22)
    slot_mapping = torch.tensor([3, 1, 0, 7, 5, 6], dtype=I32)
    # row 5 -> slot 6 is greedy without processors: equal maxima at offsets 100 (tile 0)
    # and 5 (tile 1); the reference tile rule selects column 1029
    p["indicators"][6] = 0x40
    x[5] = (torch.randn(vocab, generator=gen(23)) * 2).to(BF16)
    x[5, 100] = 30.0
    x[5, 1024 + 5] = 30.0
    noise = gumbel((slots, vocab), seed=24)
    inputs = dict(logits=x, slot_mapping=slot_mapping, gumbel_noise=noise, **p)
    decode = p["decode_counts"].clone()
    kw = dict(inputs, decode_counts=decode)
    sel = fused_singular(block_n=block_n, enable_pdl=False, update_counts=True, return_logprobs=True,
                         max_top_logprobs=5, topk_strategy=RADIX, **kw)
    lp = sel.logprobs
    save("singular_mixed", inputs,
         {"tokens": sel.tokens.clone(), "logprobs": lp.selected.clone(), "top_logprobs": lp.top_k.logprobs.clone(),
          "top_tokens": lp.top_k.tokens.clone(), "decode_counts": decode},
         {"block_n": block_n, "max_top_logprobs": 5, "update_counts": True, "prefill": False})


def case_singular_drafting():
    """Drafting step t = 1: d2t (int64) into a larger target vocab, slot mapping, drafted-token
    counts, candidate probabilities written into an fp32 [slots, V_t] buffer."""
    slots, rows, vd, vt, lookahead, block_n = 8, 5, 4096, 8192, 3, 1024
    p = slot_params(slots, vt, lookahead + 1, seed=31, greedy_slots=(2,))
    p["indicators"] = p["indicators"] & ~0x400  # drafting disables top-Z logprobs
    x = peaked_logits(rows, vd, seed=32)
    d2t = torch.randperm(vt, generator=gen(33))[:vd].to(torch.int64)
    slot_mapping = torch.tensor([4, 2, 7, 0, 1], dtype=I32)
    tokens = torch.randint(0, vt, (slots, lookahead + 1), generator=gen(34), dtype=I32)
    # make some drafted ids land on the sampled vocabulary
    tokens[:, :lookahead] = d2t[torch.randint(0, vd, (slots, lookahead), generator=gen(35))].to(I32)
    noise = gumbel((slots, vt), seed=36)
    probs = torch.zeros(slots, vt, dtype=torch.float32)
    inputs = dict(logits=x, slot_mapping=slot_mapping, d2t_mapping=d2t, drafted_tokens=tokens, gumbel_noise=noise,
                  **{k: v for k, v in p.items() if k != "top_k_logprobs"})
    sel = fused_singular(lookahead=lookahead, target_vocab=vt, block_n=block_n, enable_pdl=False,
                         return_probabilities=True, draft_probabilities=probs, topk_strategy=RADIX,
                         grammar=p["grammar"][:, 1], top_k_logprobs=p["top_k_logprobs"],
                         **{k: v for k, v in inputs.items() if k != "grammar"})
    inputs["grammar_full"] = inputs.pop("grammar")
    inputs["top_k_logprobs"] = p["top_k_logprobs"]
    save("singular_drafting", inputs, {"tokens": sel.tokens.clone(), "probabilities": probs},
         {"block_n": block_n, "lookahead": lookahead, "target_vocab": vt, "timestep": 1})


def _multistep_case(name, *, batch, gamma, vocab, block_n, seed, greedy_slots=(), greedy_draft_slots=(),
                    varlen_lengths=None, with_q=True, slot_mapping=None, slots=None):
    slots = slots or batch
    p = slot_params(slots, vocab, gamma + 1, seed=seed, greedy_slots=greedy_slots)
    for s in greedy_draft_slots:
        p["indicators"][s] = int(p["indicators"][s]) | 0x800
    g = gen(seed + 1)
    if varlen_lengths is None:
        rows = batch * (gamma + 1)
        cu = None
    else:
        cu = torch.tensor([0] + torch.tensor(varlen_lengths).cumsum(0).tolist(), dtype=I32)
        rows = int(cu[-1])
    x = peaked_logits(rows, vocab, seed=seed + 2)
    # draft distribution: softmax of the target logits plus noise, drafted tokens drawn from it
    q = None
    drafted = torch.zeros(rows, dtype=I32)
    qfull = torch.softmax(x.float() + torch.randn(rows, vocab, generator=g) * 0.5, dim=-1)
    draw = torch.multinomial(qfull, 1, generator=g).flatten().to(I32)
    # half of the requests draft the target argmax so greedy chains get accepted
    argmax = x.float().argmax(-1).to(I32)
    for b in range(batch):
        m = b * (gamma + 1) if cu is None else int(cu[b])
        n = gamma + 1 if cu is None else varlen_lengths[b]
        src = argmax if b % 2 == 0 else draw
        drafted[m:m + n] = src[m:m + n]
        if b % 3 == 1 and n > 2:
            drafted[m + 1] = (drafted[m + 1] + 7) % vocab
    if with_q:
        q = torch.zeros(slots, gamma, vocab, dtype=torch.float32)
        for b in range(batch):
            m = b * (gamma + 1) if cu is None else int(cu[b])
            n = gamma + 1 if cu is None else varlen_lengths[b]
            slot = b if slot_mapping is None else int(slot_mapping[b])
            for s in range(min(gamma, n - 1)):
                q[slot, s] = qfull[m + s]
    noise = gumbel((slots, gamma + 1, vocab), seed=seed + 3)
    uniform = torch.empty(slots, gamma + 1).uniform_(torch.finfo(BF16).tiny, 1.0, generator=gen(seed + 4)).to(BF16)
    logits = x if cu is not None else x.view(batch, gamma + 1, vocab)
    tokens = drafted if cu is not None else drafted.view(batch, gamma + 1)
    inputs = dict(logits=logits, drafted_tokens=tokens, gumbel_noise=noise, uniform_noise=uniform, **p)
    if q is not None:
        inputs["draft_probabilities"] = q
    if cu is not None:
        inputs["cu_seqlens"] = cu
    if slot_mapping is not None:
        inputs["slot_mapping"] = slot_mapping
    decode = p["decode_counts"].clone()
    kw = dict(inputs, decode_counts=decode)
    ver = fused_multistep(lookahead=gamma, max_top_logprobs=5, enable_pdl=False, update_counts=True,
                          return_logprobs=True, block_n=block_n, topk_strategy=RADIX, **kw)
    out = {"tokens": ver.tokens.clone(), "offsets": ver.offsets.clone(), "decode_counts": decode,
           "logprobs": ver.logprobs.selected.clone(), "top_logprobs": ver.logprobs.top_k.logprobs.clone(),
           "top_tokens": ver.logprobs.top_k.tokens.clone()}
    save(name, inputs, out, {"block_n": block_n, "lookahead": gamma, "max_top_logprobs": 5, "update_counts": True})


def case_multistep_stochastic():
    _multistep_case("multistep_stochastic", batch=4, gamma=3, vocab=4096, block_n=1024, seed=41)


def case_multistep_mixed():
    """Greedy requests, a stochastic request verifying a greedy draft (0x800), slot mapping."""
    _multistep_case("multistep_mixed", batch=4, gamma=3, vocab=4096, block_n=1024, seed=51, slots=6,
                    greedy_slots=(2, 5), greedy_draft_slots=(4,), slot_mapping=torch.tensor([5, 0, 4, 2], dtype=I32))


def case_multistep_varlen():
    """Variable draft lengths through cu_seqlens (functional rung only in the reference)."""
    _multistep_case("multistep_varlen", batch=4, gamma=3, vocab=4096, block_n=1024, seed=61,
                    greedy_slots=(3,), varlen_lengths=[2, 4, 1, 3])


def case_indexed_copy():
    """The reference's noise staging kernel (ops/copy.py:21-127) on [slots, T, V] bf16 noise:
    a row that fits one block, and rows of several 8192-column blocks with a ragged last one."""
    import sonic_sampler.ops.copy as ref_copy

    ref_copy.total_sm = lambda device: 148  # no GPU here: the grid rule's SM count
    inputs, outputs = {}, {}
    for tag, (slots, steps, vocab) in {"small": (6, 3, 1000), "blocks": (5, 2, 8192 + 4100)}.items():
        g = gen(7 + slots)
        source = torch.randn(slots, steps, vocab, generator=g).to(BF16)
        target = torch.randn(slots, steps, vocab, generator=g).to(BF16)
        indices = torch.randperm(slots, generator=g)[: slots - 1].to(torch.int64)
        indicator = torch.zeros(slots, dtype=torch.uint16)
        indicator[indices[1]] = 0x40  # a greedy slot: not staged
        indicator[indices[2]] = 0x41  # greedy with another bit
        indicator[indices[3]] = 0x3F  # every bit below greedy: staged
        inputs[tag] = dict(source=source.clone(), target=target.clone(), indices=indices.clone(),
                           indicator=indicator.clone())
        ref_copy.indexed_copy(source, target, indices, indicator)
        outputs[tag] = dict(target=target.clone())
    save("indexed_copy", inputs, outputs, {"reference": "ops/copy.py:21-127 indexed_copy"})


def _state(b) -> dict:
    """The device-side fields of a reference SamplingBuffers, cloned."""
    rep = b.repetition
    w = b.weights
    plain = lambda t: t.as_subclass(torch.Tensor).clone()  # noqa: E731
    return {k: plain(v) for k, v in dict(
        flags=b.flags.packed.clone(), temperature=b.temperature.clone(), top_p=b.top_p.clone(), min_p=b.min_p.clone(),
        top_k=b.top_k.clone(), top_logprobs=b.top_logprobs.clone(), multiplicative=rep.multiplicative.clone(),
        frequency=rep.frequency.clone(), presence=rep.presence.clone(), context=rep.counts.context.clone(),
        decode=rep.counts.decode.clone(), bias=b.bias.clone(), grammar=b.grammar.view(torch.int32).clone(),
        gumbel_target=torch.Tensor(w.gumbel.target).clone(), gumbel_draft=torch.Tensor(w.gumbel.draft).clone(),
        uniform=torch.Tensor(w.uniform).clone(),
    ).items()}


def case_populate():
    """The reference's own SamplingBuffers.allocate / update (core/buffer.py:1139-1352) on host
    tensors: its pinned host mirrors become ordinary host tensors for this run (`pin_memory`
    is dropped, there is no GPU here), and its pinned bias mirror starts zeroed. A sequence of
    calls on one buffer per shape; the state after each call is saved.

    Bitmasks are given only where `positions` is the identity prefix: the reference's
    step_grammar indexes the bitmask list by slot id (core/buffer.py:1041-1049) while every
    other list is aligned with `positions`, and the two readings agree only there."""
    import sonic_sampler.ops.copy as ref_copy
    from sonic_sampler.core.buffer import SamplingBuffers as RefBuffers

    ref_copy.total_sm = lambda device: 148
    originals = {n: getattr(torch, n) for n in ("empty", "empty_like", "tensor", "zeros")}

    def nopin(fn):
        def wrapped(*args, **kwargs):
            kwargs.pop("pin_memory", None)
            return fn(*args, **kwargs)
        return wrapped

    for n, f in originals.items():
        setattr(torch, n, nopin(f))
    try:
        inputs, outputs = {}, {}
        for tag, (B, T, V) in {"small": (6, 3, 1000), "ranges": (3, 2, 9000)}.items():
            g = gen(41 + V)
            W = (V + 31) // 32
            torch.manual_seed(5 + V)
            buf = RefBuffers.default(B, T, V, device=torch.device("cpu"))
            buf.pinned.bias.zero_()
            inputs[tag] = dict(shape=(B, T, V), initial=_state(buf), calls=[])
            outputs[tag] = []

            def params(n):
                return dict(
                    multiplicative=[float(x) for x in (torch.rand(n, generator=g) * 0.6 + 0.7)],
                    frequency=[float(x) for x in (torch.rand(n, generator=g) - 0.5)],
                    presence=[float(x) for x in (torch.rand(n, generator=g) * 0.4)],
                    temperature=[float(x) for x in (torch.rand(n, generator=g) + 0.4)],
                    top_k=[(128, 20, 1, 64)[int(i)] for i in torch.randint(0, 4, (n,), generator=g)],
                    top_p=[float(x) for x in (torch.rand(n, generator=g) * 0.3 + 0.7)],
                    min_p=[(0.0, 0.05)[int(i)] for i in torch.randint(0, 2, (n,), generator=g)],
                    top_logprobs=[int(i) for i in torch.randint(0, 6, (n,), generator=g)],
                )

            def biases(n):
                out = []
                for j in range(n):
                    if j % 3 == 1:
                        out.append(None)
                    else:
                        toks = torch.randperm(V, generator=g)[: 2 + j % 4].tolist()
                        out.append({t: float(torch.randn(1, generator=g)) * 2 for t in toks})
                return out

            def masks(n, full):
                out = []
                for j in range(n):
                    if j % 2 == 1:
                        out.append(None)
                    else:
                        rows = T if (full and j % 4 == 0) else 1
                        m = torch.randint(-2**31, 2**31 - 1, (rows, W), generator=g, dtype=torch.int64).to(torch.int32)
                        out.append(m[0] if rows == 1 else m)
                return out

            if tag == "small":
                plan = [
                    ("allocate", [4, 1, 3], False),
                    ("allocate", [0, 1], True),
                    ("update", [2, 0, 5], False),
                    ("update", None, True),
                ]
            else:
                plan = [("allocate", [2, 0], False), ("update", [0, 1, 2], True)]
            for k, (kind, positions, grammar) in enumerate(plan):
                n = len(positions) if positions else B
                kw = params(n)
                kw["biases"] = biases(n)
                kw["greedy_drafts"] = [bool(j % 2) for j in range(n)]
                if grammar:
                    kw["bitmasks"] = masks(n, full=(kind == "update"))
                if kind == "allocate":
                    kw["encodings"] = [torch.randint(0, V, (int(torch.randint(0, 3 * V // 2, (1,), generator=g)),),
                                                     generator=g) for _ in range(n)]
                    kw["positions"] = positions
                else:
                    kw["counts"] = [(torch.randint(0, 9, (V,), generator=g, dtype=torch.int32),
                                     torch.randint(0, 5, (V,), generator=g, dtype=torch.int32)) for _ in range(n)]
                    kw["target_gumbel"] = [None] * n
                    kw["positions"] = positions
                seed = 1000 + 17 * k
                inputs[tag]["calls"].append(dict(kind=kind, kwargs=kw, generator_seed=seed))
                getattr(buf, kind)(generator=torch.Generator().manual_seed(seed), **kw)
                outputs[tag].append(_state(buf))
            if tag == "ranges":  # the larger shape keeps only its final noise
                for snap in outputs[tag][:-1]:
                    for key in ("gumbel_target", "gumbel_draft", "uniform"):
                        snap.pop(key)
    finally:
        for n, f in originals.items():
            setattr(torch, n, f)
    save("populate", inputs, outputs, {"reference": "core/buffer.py:1139-1352 SamplingBuffers.update / allocate"})


CASES = {
    "populate": case_populate,
    "indexed_copy": case_indexed_copy,
    "topk_bf16": case_topk_bf16,
    "topk_bitonic": case_topk_bitonic,
    "singular_mixed": case_singular_mixed,
    "singular_drafting": case_singular_drafting,
    "multistep_stochastic": case_multistep_stochastic,
    "multistep_mixed": case_multistep_mixed,
    "multistep_varlen": case_multistep_varlen,
}

if __name__ == "__main__":
    wanted = sys.argv[1:] or list(CASES)
    for name in wanted:
        t0 = time.time()
        print(f"{name} ...", flush=True)
        CASES[name]()
        print(f"  {time.time() - t0:.1f} s", flush=True)
