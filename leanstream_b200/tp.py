"""Tensor-parallel sharding of logical groups across the GPUs of one box.

Logical group g lives on rank g mod R at local slot g // R (static,
round-robin residency: 1/R of each layer's weights per GPU). The active set
is chosen globally; every rank enqueues only its own descriptors and
computes an fp32 partial of y. Two ways to combine the partials, with the
same arithmetic (sum over ranks, one fp16 rounding, the residual), so every
rank holds the same next hidden state:
- inside the persistent launch (ls_b200_tp_setup / ls_b200_tp_connect): the
  reducer CTAs store each layer's partial into every rank's exchange buffer
  over NVLink peer memory and every CTA forms the next input from them --
  one launch per token per rank, no collective library on the data path;
- between launches: LS_B200_NO_OUTPUT + output_f32, an allreduce of the
  partials, and ls_b200_tp_epilogue.
"""
from __future__ import annotations

import numpy as np


def owner(group: int, world: int) -> int:
    return int(group) % world


def local_slot(group: int, world: int) -> int:
    return int(group) // world


def local_groups(n_groups: int, rank: int, world: int) -> list:
    return [g for g in range(n_groups) if g % world == rank]


def rank_descriptors(active, rank: int, world: int) -> np.ndarray:
    """ExecDesc rows of this rank for a globally chosen active set, in the
    global order: [logical, physical(local), source_slot(local), dest, cache]."""
    mine = [int(g) for g in active if int(g) % world == rank]
    rows = np.zeros((len(mine), 5), dtype=np.uint32)
    for pos, g in enumerate(mine):
        s = local_slot(g, world)
        rows[pos] = (g, s, s, pos, 0)
    return rows


def shard_groups(array: np.ndarray, rank: int, world: int) -> np.ndarray:
    """Rows of a [n_groups, ...] array that rank `rank` stores, in local-slot order."""
    return np.ascontiguousarray(array[rank::world])
