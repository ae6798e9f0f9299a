"""Host-side logic of the drop-in interface: tile-size dispatch, constructor contracts,
shape resolution, indicator bits."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from sonic_sampler_b200.core.flags import Indicator
from sonic_sampler_b200.interface.base import TopKStrategy, TwoStageTiling
from sonic_sampler_b200.interface.dispatch import DispatchSummary, next_power_of_2
from sonic_sampler_b200.interface.functional.multistep import resolve_batch_vocab

# the reference's tuning tables, from its unmodified install in baseline/_ref (git-ignored)
REFERENCE_TABLES = Path(__file__).resolve().parents[1] / "baseline" / "_ref" / "sonic_sampler" / "resources" / "dispatch"


@pytest.mark.skipif(not REFERENCE_TABLES.is_dir(), reason="reference not installed in baseline/_ref")
@pytest.mark.parametrize("arch", [90, 100])
def test_dispatch_table_matches_reference_toml(arch):
    import tomllib

    ref = tomllib.loads((REFERENCE_TABLES / f"sm{arch}_k128.toml").read_text())
    ours = DispatchSummary.load(k=128, arch=arch)
    assert [v["size"] for v in ref["vocab"]] == [v.size for v in ours.vocab]
    for rv, ov in zip(ref["vocab"], ours.vocab):
        assert [b["size"] for b in rv["batch"]] == [b.size for b in ov.batch]
        for rb, ob in zip(rv["batch"], ov.batch):
            cfg = sorted(rb["config"], key=lambda c: c["priority"])
            assert [(c["strategy"], c["block_n"], c["first_warps"], c["second_warps"]) for c in cfg] == \
                   [(c.strategy, c.block_n, c.first_warps, c.second_warps) for c in ob.config]


def test_block_n_resolution_follows_reference_rules():
    d = DispatchSummary.load(arch=100)
    bucket = d.get_vocab(128256)
    assert bucket.size == 131072 and bucket.block_n == 4096
    assert d.get_vocab(32000).size == 32768 and d.get_vocab(32000).block_n == 2048
    assert d.get_vocab(256000).size == 262144
    assert d.get_vocab(262144 * 2) is None
    assert bucket.get_batch(8).best.block_n == 8192
    assert bucket.get_batch(40).size == 32  # within +50 % of the last bucket
    assert bucket.get_batch(64) is None  # beyond: defaults


def test_tiling_tuning_matches_reference():
    dispatch, vocab, block_n = TwoStageTiling.resolve(128256, arch=100)
    t = TwoStageTiling(pdl=True, block_n=block_n, vocabulary=vocab, scratchpad=torch.empty(0), dispatch=dispatch)
    cfg, strat, bn = t.tuning(16)
    assert (bn, strat.key) == (16384, "adaptive")
    cfg, strat, bn = t.tuning(64)
    assert (bn, strat.key, cfg.first, cfg.second) == (4096, "bitonic", 16, 8)
    cfg, strat, bn = t.tuning(16, strategy=TopKStrategy(radix=True))
    assert (bn, strat.key) == (16384, "radix")


@pytest.mark.parametrize("kwargs, message", [
    (dict(vocab_size=128256, k=256), "maximum supported top-k"),
    (dict(vocab_size=128256, k=96), "power of 2"),
    (dict(vocab_size=1024, block_size=1024), "greater than 1"),
    (dict(vocab_size=128256, top_logprobs=129), "top logprobs"),
    (dict(vocab_size=10**7, arch=100), "vocabulary size"),
    (dict(vocab_size=128256, arch=80), "dispatch summary"),
])
def test_resolve_value_errors(kwargs, message):
    with pytest.raises(ValueError, match=message):
        TwoStageTiling.resolve(**kwargs)


def test_multistep_shape_resolution():
    x3 = torch.empty(4, 5, 100)
    assert resolve_batch_vocab(x3, None, None) == (False, 4, 4, 100)
    x2 = torch.empty(20, 100)
    assert resolve_batch_vocab(x2, None, 4) == (False, 4, 4, 100)
    with pytest.raises(ValueError, match="zero lookahead"):
        resolve_batch_vocab(x2, None, None)
    with pytest.raises(ValueError, match="multiple of lookahead"):
        resolve_batch_vocab(torch.empty(21, 100), None, 4)
    cu = torch.tensor([0, 2, 5], dtype=torch.int32)
    assert resolve_batch_vocab(torch.empty(5, 100), cu, 3) == (True, 2, 3, 100)
    with pytest.raises(ValueError, match="maximum lookahead"):
        resolve_batch_vocab(torch.empty(5, 100), cu, None)
    with pytest.raises(ValueError, match="fixed timestep"):
        resolve_batch_vocab(x3, cu, 3)


def test_indicator_from_params_and_greedy():
    ind = Indicator.from_params(grammar=True, multiplicative=1.1, temperature=0.7, top_k=20, top_p=0.9,
                                min_p=0.05, top_k_logprobs=5)
    assert int(ind) == 0x1 | 0x2 | 0x20 | 0x80 | 0x100 | 0x200 | 0x400
    g = ind.greedy()
    assert int(g) == 0x1 | 0x2 | 0x40
    assert int(Indicator.from_params(top_k=1, top_p=0.5)) == 0x40
    assert next_power_of_2(5) == 8 and next_power_of_2(8) == 8 and next_power_of_2(0) == 0
