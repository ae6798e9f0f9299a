"""Noise staging (`sonic_indexed_copy`, reference ops/copy.py:21-127) on the GPU against the
oracle restatement: bit-exact rows, untouched rows unchanged. Covers the bulk-copy path
(16-byte rows), the element path (odd row sizes, unaligned views), int32/int64 indices,
duplicates, greedy slots, empty calls, and the golden vectors of the reference kernel."""

from __future__ import annotations

import pytest
import torch

from golden_cases import load

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from sonic_sampler_b200 import _abi

    _abi.load_library()
    return torch.device("cuda", 0)


def _bits(t):
    t = t.detach().cpu()
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def _check(dev, source, target, indices, indicator):
    """Run the GPU copy on device copies and the oracle on host copies; compare bit for bit."""
    from oracle import oracle
    from sonic_sampler_b200.ops import indexed_copy

    expect = target.detach().cpu().clone()
    oracle.indexed_copy(source.detach().cpu(), expect, indices.cpu(), indicator.cpu())
    indexed_copy(source, target, indices.to(dev), indicator.to(dev))
    torch.cuda.synchronize()
    assert torch.equal(_bits(target), _bits(expect))


def _case(dev, slots, steps, vocab, seed, dtype=BF16, greedy_every=3):
    g = torch.Generator().manual_seed(seed)
    both = torch.randn(2, slots, steps, vocab, generator=g).to(dtype).to(dev)
    indicator = torch.zeros(slots, dtype=torch.int32)
    indicator[::greedy_every] = 0x40
    indicator[1::5] |= 0x25  # other bits never matter
    return both[0], both[1], indicator.to(torch.uint16), g


@pytest.mark.parametrize("index_dtype", [torch.int64, torch.int32])
def test_bulk_rows_config_shape(dev, index_dtype):
    """Rows of 4 x 128256 bf16 (16-byte multiples): the bulk-copy ring."""
    draft, target, indicator, g = _case(dev, 48, 4, 128256, seed=1)
    indices = torch.randperm(48, generator=g)[:32].to(index_dtype)
    _check(dev, draft, target, indices, indicator)


def test_bulk_rows_smaller_than_a_chunk(dev):
    draft, target, indicator, g = _case(dev, 40, 1, 2048, seed=2)  # 4 KB rows
    _check(dev, draft, target, torch.randperm(40, generator=g)[:25], indicator)


def test_duplicates_and_all_greedy(dev):
    draft, target, indicator, g = _case(dev, 8, 2, 4096, seed=3)
    _check(dev, draft, target, torch.tensor([3, 3, 5, 3, 7], dtype=torch.int64), indicator)
    indicator = torch.full((8,), 0x40, dtype=torch.uint16)
    before = target.clone()
    _check(dev, draft, target, torch.arange(8), indicator)
    assert torch.equal(target, before)


@pytest.mark.parametrize("dtype", [BF16, torch.float32])
def test_element_path_odd_rows(dev, dtype):
    """Rows of 3 x 1001 elements are not 16-byte multiples: the element-wise kernel."""
    draft, target, indicator, g = _case(dev, 12, 3, 1001, seed=4, dtype=dtype)
    _check(dev, draft, target, torch.randperm(12, generator=g)[:9], indicator)


def test_element_path_unaligned_views(dev):
    """Noise views that start one element into their allocation."""
    g = torch.Generator().manual_seed(5)
    slots, steps, vocab = 10, 2, 4096
    n = slots * steps * vocab
    flat = torch.randn(2, n + 1, generator=g).to(BF16).to(dev)
    draft, target = flat[0, 1:].view(slots, steps, vocab), flat[1, 1:].view(slots, steps, vocab)
    indicator = torch.zeros(slots, dtype=torch.uint16)
    indicator[4] = 0x40
    _check(dev, draft, target, torch.randperm(slots, generator=g), indicator)


def test_empty_and_out_of_range_indices(dev):
    from sonic_sampler_b200.ops import indexed_copy

    draft, target, indicator, _ = _case(dev, 6, 1, 4096, seed=6)
    before = target.clone()
    indexed_copy(draft, target, torch.empty(0, dtype=torch.int64, device=dev), indicator.to(dev))
    # an index outside the rows is skipped (the reference would read out of bounds)
    indexed_copy(draft, target, torch.tensor([-1, 6, 100], dtype=torch.int64, device=dev), indicator.to(dev))
    torch.cuda.synchronize()
    assert torch.equal(target, before)


@pytest.mark.parametrize("tag", ["small", "blocks"])
def test_golden_reference_outputs(dev, tag):
    """The reference kernel's own outputs (generated through Triton's interpreter)."""
    from sonic_sampler_b200.ops import indexed_copy

    case = load("indexed_copy")
    i, o = case["inputs"][tag], case["outputs"][tag]
    target = i["target"].to(dev)
    indexed_copy(i["source"].to(dev), target, i["indices"].to(dev), i["indicator"].to(dev))
    torch.cuda.synchronize()
    assert torch.equal(_bits(target), _bits(o["target"]))


def test_stage_weights_on_buffers(dev):
    """`GumbelNoise.stage_weights` (reference core/buffer.py:151-157) on sampling buffers."""
    from oracle import oracle
    from sonic_sampler_b200 import workloads

    b = workloads.sampling_buffers(16, 4, 32000, dev, 7, workloads.config2_params(16, 8))
    noise = b.weights.gumbel
    indices = torch.tensor([1, 4, 9, 12, 15], dtype=torch.int64, device=dev)
    indicator = b.flags.draft
    expect = noise.target.cpu().clone()
    oracle.indexed_copy(noise.draft.cpu(), expect, indices.cpu(), indicator.cpu())
    noise.stage_weights(indices, indicator)
    torch.cuda.synchronize()
    assert torch.equal(_bits(noise.target), _bits(expect))
