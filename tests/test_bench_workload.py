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
