"""Seeded synthetic weights, scales and activations in LeanStream's packed format.

Format (kernels/streaming_mlp.cu:8-10,23,27-39; backends/triton/core.py:10-17;
examples/ministral/pack/int4_format.py:1-18):
  * a neuron record is [gate H/2 B | up H/2 B | down H/2 B], signed INT4,
    low nibble = even coordinate;
  * a logical group is G consecutive neuron records, group_bytes = G*3H/2;
    cache / staging slot s starts at s*group_bytes;
  * scales are fp16 [physical_group][G][3][H/128], one per 128 coordinates.

Random stream (numpy PCG64 via default_rng(seed)), drawn in this order:
  1. q      = integers(-8, 8, size=(N, G, 3, H), int8)     uniform in [-8, 7]
  2. scales = uniform(0.005, 0.02, size=(N, G, 3, H/128)) -> float16
  3. x      = standard_normal(H) -> float16
The public benchmark of the reference is not a dataset: BASELINE.json's
configurations are synthetic, and these draws stand in for them.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def pack_int4(q: np.ndarray) -> np.ndarray:
    """Packs signed INT4 values along the last axis, low nibble first."""
    q = np.asarray(q, dtype=np.int8)
    if q.shape[-1] % 2:
        raise ValueError("last axis must be even")
    u = q.view(np.uint8) & 15
    return (u[..., 0::2] | (u[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Inverse of pack_int4 (int4_format.py:21-26)."""
    packed = np.asarray(packed, dtype=np.uint8)
    q = np.empty((*packed.shape[:-1], packed.shape[-1] * 2), dtype=np.int8)
    q[..., 0::2] = (packed & 15).astype(np.int8)
    q[..., 1::2] = (packed >> 4).astype(np.int8)
    q[q >= 8] -= 16
    return q


def dequantize(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """w = fp16(float(q) * float(scale[c/128])) as float32 (core.py:17)."""
    s = np.repeat(np.asarray(scales, dtype=np.float16).astype(np.float32), 128, axis=-1)
    return (q.astype(np.float32) * s).astype(np.float16).astype(np.float32)


@dataclass
class Layer:
    hidden: int
    group_size: int
    groups: int
    q: np.ndarray        # int8 [N, G, 3, H]
    packed: np.ndarray   # uint8 [N * G * 3H/2], slot-major
    scales: np.ndarray   # float16 [N, G, 3, H/128]
    x: np.ndarray        # float16 [H]

    @property
    def group_bytes(self) -> int:
        return self.group_size * 3 * self.hidden // 2


def make_layer(seed: int, hidden: int, groups: int, group_size: int = 64) -> Layer:
    if hidden % 256:
        raise ValueError("hidden must be a multiple of 256")
    rng = np.random.default_rng(seed)
    q = rng.integers(-8, 8, size=(groups, group_size, 3, hidden), dtype=np.int8)
    scales = rng.uniform(0.005, 0.02, size=(groups, group_size, 3, hidden // 128)).astype(np.float16)
    x = rng.standard_normal(hidden).astype(np.float16)
    return Layer(hidden, group_size, groups, q, pack_int4(q).reshape(-1), scales, x)


def representative_rows(layer: Layer) -> np.ndarray:
    """ls_predict fp32 weights [rows, 2, stride]: per group, the fp32 mean of its
    G dequantised gate rows and of its G up rows (a documented choice of
    representative row; predictor.h:12)."""
    gate = dequantize(layer.q[:, :, 0, :], layer.scales[:, :, 0, :]).mean(axis=1, dtype=np.float32)
    up = dequantize(layer.q[:, :, 1, :], layer.scales[:, :, 1, :]).mean(axis=1, dtype=np.float32)
    return np.ascontiguousarray(np.stack([gate, up], axis=1).astype(np.float32))


def seeded_selection(seed: int, groups: int, fraction: float) -> np.ndarray:
    """Top-`fraction` active set from a seeded ranking (3)."""
    k = int(round(fraction * groups))
    return np.random.default_rng(seed).permutation(groups)[:k].astype(np.int32)


def descriptors(ids, cache_slots=None, physical=None, core: int = 0) -> np.ndarray:
    """ExecDesc rows [logical, physical, source_slot, dest_slot, kind] for ids in
    final order: dest = position (weight_manager.cpp:177-178), cache source."""
    ids = np.asarray(ids, dtype=np.uint32)
    out = np.zeros((len(ids), 5), dtype=np.uint32)
    out[:, 0] = ids
    out[:, 1] = ids if physical is None else np.asarray(physical, dtype=np.uint32)[ids]
    out[:, 2] = ids if cache_slots is None else np.asarray(cache_slots, dtype=np.uint32)[ids]
    out[:, 3] = np.arange(core, core + len(ids), dtype=np.uint32)
    out[:, 4] = 0
    return out
