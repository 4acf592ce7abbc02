"""The benchmark's workload definitions (bench.py) on CPU: configuration 3
draws per token and layer a seeded active set of 20-40 % of 192 groups
(k = round(f * 192) in [38, 77]); configuration 5
uses 90 of 448 groups (20 %) over 80 layers at H 8192; the sets are the same
on every rank (a function of the step and layer only); round-robin sharding
covers every active group once; the algorithmic bytes per group are the
INT4 records plus fp16 scales."""
import importlib

import numpy as np


def _bench(config):
    import bench

    bench = importlib.reload(bench)
    bench.set_config(config)
    return bench


def test_config3_active_sets():
    b = _bench(3)
    assert (b.H, b.NGROUPS, b.LAYERS, b.G) == (4096, 192, 36, 64)
    assert b.ALG_BYTES_PER_GROUP == 405_504
    ks = []
    for step in range(4):
        sets = b.active_sets(step)
        assert len(sets) == 36
        for ids in sets:
            assert len(set(ids.tolist())) == len(ids) and ids.min() >= 0 and ids.max() < 192
            assert np.all(np.diff(ids) > 0)
            ks.append(len(ids))
    assert 38 <= min(ks) and max(ks) <= 77
    # a function of (step, layer) only: identical on every call (every rank)
    assert all(np.array_equal(a, c) for a, c in zip(b.active_sets(2), b.active_sets(2)))


def test_config5_geometry_and_sets():
    b = _bench(5)
    assert (b.H, b.I, b.NGROUPS, b.LAYERS) == (8192, 28672, 448, 80)
    assert b.ALG_BYTES_PER_GROUP == 811_008
    assert {len(ids) for ids in b.active_sets(0)} == {90}


def test_round_robin_sharding_and_balance():
    from leanstream_b200 import tp

    b = _bench(3)
    ids = b.active_sets(5)[7]
    for world in (2, 4, 8):
        owned = sorted(int(g) for r in range(world) for g in tp.rank_descriptors(ids, r, world)[:, 0])
        assert owned == sorted(int(g) for g in ids)
        bal = b.rank_balance(3, 5, world)
        assert bal["busiest_over_mean"] >= 1.0 and bal["worst_busiest_over_mean"] >= bal["busiest_over_mean"]
        assert abs(bal["mean_groups_per_rank_layer"] * world - np.mean(
            [len(s) for st in range(3, 5) for s in b.active_sets(st)])) < 1e-9


def test_config5_batch8_union_and_masks():
    """--batch 8: step s decodes tokens 8s .. 8s+7; per layer the union is the
    sorted set of their groups (about 1 - 0.8^8 = 83 % of 448 at 20 % each)
    and mask row b marks exactly token 8s + b's own groups."""
    from leanstream_b200.synthetic import descriptors

    b = _bench(5)
    per_token = [b.active_sets(8 * 2 + t) for t in range(8)]
    layers = b.batch_union(2)
    assert len(layers) == 80
    fractions = []
    for layer, (union, mask) in enumerate(layers):
        expect = sorted(set().union(*(set(per_token[t][layer].tolist()) for t in range(8))))
        assert union.tolist() == expect
        assert mask.shape == (8, len(union)) and mask.dtype == np.uint8
        for t in range(8):
            assert union[mask[t] == 1].tolist() == per_token[t][layer].tolist()
        fractions.append(len(union) / 448)
        rows = descriptors(union)  # what the bench uploads: logical = physical = cache slot
        assert rows.shape == (len(union), 5) and rows[:, 0].tolist() == expect
        assert np.array_equal(rows[:, 2], rows[:, 0]) and np.array_equal(rows[:, 3], np.arange(len(union)))
    assert 0.78 < np.mean(fractions) < 0.88
    # the per-layer image the bench writes fits its fixed stride
    assert 448 * 20 + 8 * 448 <= ((448 * 20 + 8 * 448 + 255) // 256) * 256
