"""Host-side logic: workload definitions, FLOP accounting, seeding, sharding."""
import pytest
import torch

from rocm_attn_b200.workloads import WORKLOADS, Shape, make_qkv, parse_shapes, shard_range, slice_seed
from rocm_attn_b200.sharding import local_view


def test_config_flops():
    # 4*B*H*Lq*Lk*D non-causal; causal counts exactly the unmasked pairs
    assert WORKLOADS["c1"].flops() == pytest.approx(68.72e9, rel=1e-3)
    assert WORKLOADS["c2"].flops() == pytest.approx(4 * 32 * 128 * 2048 * 2049 / 2)
    assert WORKLOADS["c3"].flops() == pytest.approx(34.36e9, rel=1e-3)
    assert WORKLOADS["c4"].flops() == pytest.approx(4 * 64 * 128 * 16384 * 16385 / 2)
    assert WORKLOADS["c5"].flops() == pytest.approx(1380.3e9, rel=1e-3)


def test_causal_pairs_cross_shapes():
    assert Shape(1, 1, 4, 6, 8).unmasked_pairs(True) == 1 + 2 + 3 + 4
    assert Shape(1, 1, 6, 4, 8).unmasked_pairs(True) == 1 + 2 + 3 + 4 + 4 + 4


def test_parse_shapes_reference_syntax():
    # benchmark/bench_attention.py:25-44 syntax, e.g. the preset file entries
    s = parse_shapes("2560,8,16,64;16,5,2560,93,64")
    assert s == [Shape(2560, 8, 16, 16, 64), Shape(16, 5, 2560, 93, 64)]
    with pytest.raises(ValueError):
        parse_shapes("1,2,3")
    with pytest.raises(ValueError):
        parse_shapes(" ; ")


@pytest.mark.parametrize("n,world", [(64, 1), (64, 8), (32, 3), (5, 8), (1, 2)])
def test_shard_range_partitions(n, world):
    parts = [shard_range(n, world, r) for r in range(world)]
    flat = [i for p in parts for i in p]
    assert flat == list(range(n))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1


def test_slice_seeds_distinct_and_inputs_deterministic():
    seeds = {slice_seed(0, t, b, h) for t in "qkv" for b in range(4) for h in range(16)}
    assert len(seeds) == 3 * 4 * 16
    s = Shape(2, 3, 10, 12, 64)
    a = make_qkv(s, torch.float16, seed=1)
    b = make_qkv(s, torch.float16, seed=1)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    # a rank can regenerate its own heads without the rest
    part = make_qkv(s, torch.float16, seed=1, bh_range=range(2, 5))
    for full, p in zip(a, part):
        assert torch.equal(full.reshape(1, 6, *full.shape[2:])[:, 2:5], p)


def test_local_view_is_a_view():
    t = torch.arange(2 * 3 * 4 * 8, dtype=torch.float32).view(2, 3, 4, 8)
    v = local_view(t, 4, 1)
    assert v.shape == (1, 2, 4, 8) and v.data_ptr() == t[0, 1].data_ptr()


def test_pinned_entry_rejects_pageable_tensors():
    # checked before any CUDA call, so this runs without a GPU
    import pytest
    import rocm_attn_b200
    x = torch.zeros(1, 1, 8, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="pinned"):
        rocm_attn_b200.attn_forward_pinned(x, x, x)


@pytest.mark.parametrize("BH,base", [(64, 4), (32, 2), (64, 8), (8, 4), (20, 2), (100, 7), (33, 3), (15, 1), (1, 1),
                                     (5, 16)])
def test_pinned_chunk_schedule_covers_every_slice(BH, base):
    from rocm_attn_b200.pipeline import _chunk_sizes
    sizes = _chunk_sizes(BH, base, uniform=False)
    assert sum(sizes) == BH and all(s > 0 for s in sizes)
    if BH >= 8 * base:  # long splits end in chunks that halve down to one slice
        tail = sizes[-(len(bin(2 * base)) - 2) - 1:]  # 2*base, halvings down to 1, and 1
        assert tail[0] == 2 * base and tail[-2:] == [1, 1] and tail == sorted(tail, reverse=True)
    else:
        assert sizes == [min(base, BH - c) for c in range(0, BH, base)]
    assert _chunk_sizes(BH, base, uniform=True) == [min(base, BH - c) for c in range(0, BH, base)]
    assert _chunk_sizes(64, 4, uniform=False) == [12, 12, 12, 12, 8, 4, 2, 1, 1]
