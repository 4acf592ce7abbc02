"""Tensor-parallel host logic on CPU with two gloo ranks (no GPU): groups are
sharded round-robin (leanstream_b200/tp.py), each rank computes the fp32
partial output of its own groups with the oracle, the partials are summed by
an allreduce, and every rank applies the single fp16 rounding + residual of
the layer epilogue. The result must equal the one-process computation within
the output tolerance, and be identical on both ranks."""
import os
import socket

import numpy as np
import pytest

H, G, NGROUPS = 1024, 64, 24
TOL = 2e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer_and_active():
    from leanstream_b200.synthetic import make_layer

    L = make_layer(77, H, NGROUPS, G)
    active = np.sort(np.random.default_rng(5).permutation(NGROUPS)[:11])
    return L, active


def _rank_main(rank, world, port, out_path):
    import torch
    import torch.distributed as dist

    from leanstream_b200 import tp
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L, active = _layer_and_active()
        gb = G * 3 * H // 2
        packed = L.packed.reshape(NGROUPS, gb)
        scales = L.scales.reshape(NGROUPS, -1)
        mine = tp.local_groups(NGROUPS, rank, world)
        local_packed = tp.shard_groups(packed, rank, world).reshape(-1)
        local_scales = tp.shard_groups(scales, rank, world).reshape(-1)
        rows = tp.rank_descriptors(active, rank, world)
        assert all(int(g) in mine for g in rows[:, 0])
        if len(rows):
            _, y32, _ = O.mlp(H, G, L.x, local_packed, local_scales, rows)
        else:
            y32 = np.zeros(H, np.float32)
        t = torch.from_numpy(y32.copy())
        dist.all_reduce(t)
        y16 = t.numpy().astype(np.float16)
        hidden = O.residual(L.x, y16)
        np.save(out_path.format(rank), np.stack([y16.astype(np.float32), hidden.astype(np.float32)]))
    finally:
        dist.destroy_process_group()


def test_two_rank_allreduce_matches_single_process(tmp_path):
    import torch.multiprocessing as mp

    from leanstream_b200 import tp
    from leanstream_b200.synthetic import descriptors
    from oracle import oracle as O

    world = 2
    out = str(tmp_path / "rank{}.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    r0, r1 = np.load(out.format(0)), np.load(out.format(1))
    assert np.array_equal(r0, r1), "ranks must hold identical y and next hidden state"

    L, active = _layer_and_active()
    y_ref, _, _ = O.mlp(H, G, L.x, L.packed, L.scales, descriptors(active))
    ref = y_ref.astype(np.float32)
    assert np.abs(r0[0] - ref).max() <= TOL * np.abs(ref).max()
    hid_ref = O.residual(L.x, y_ref).astype(np.float32)
    assert np.abs(r0[1] - hid_ref).max() <= TOL * np.abs(hid_ref).max() + 1e-3
    # every active group is computed exactly once across the ranks
    owned = sorted(int(g) for r in range(world) for g in tp.rank_descriptors(active, r, world)[:, 0])
    assert owned == sorted(int(g) for g in active)


def test_sharding_is_round_robin():
    from leanstream_b200 import tp

    for world in (1, 2, 4, 8):
        groups = [tp.local_groups(192, r, world) for r in range(world)]
        assert sorted(g for gs in groups for g in gs) == list(range(192))
        for r, gs in enumerate(groups):
            assert all(tp.owner(g, world) == r and tp.local_slot(g, world) == i for i, g in enumerate(gs))
    rows = tp.rank_descriptors(np.array([1, 2, 5, 6, 9]), 1, 4)
    assert rows[:, 0].tolist() == [1, 5, 9]           # global order kept
    assert rows[:, 1].tolist() == [0, 1, 2]           # local slot = physical group on the rank
    assert rows[:, 3].tolist() == [0, 1, 2]           # dense destination slots
