"""Batched union decode over the C ABI (ls_b200_batch_mlp).

The reference runtime decodes one token per layer step. With up to 8 tokens
in flight, the union of their active groups is dense enough (about 83 % of
the groups at 20 % per token) for the tensor-core path: every weight byte of
the union is read once for all tokens, and a per-token mask keeps each
token's result equal to the one-token MLP over its own groups.

`union_plan` builds the host side of one layer: the sorted union, its
ExecDesc rows (include/leanstream/types.h:16-20) and the [token][union]
mask. `BatchMLP` owns the device scratch and launches the kernels on a
stream; the caller owns every other buffer until the stream has run.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import numpy as np

from . import _native as N
from .backend import _check, _ptr

MAX_TOKENS = 8


def union_plan(active_sets: Sequence[Sequence[int]], cache_slots=None, physical=None, staging=None):
    """Per-token active logical groups -> (union ids, ExecDesc rows [U][5]
    uint32, mask [tokens][U] uint8).

    Rows are in union order: logical id, physical group (`physical[id]`, or
    the id), source slot (`cache_slots[id]`, or the id) and kind 0 (cache);
    ids listed in `staging` (a dict id -> staging slot) read from staging
    (kind 1) instead, as WeightManager descriptors do for streamed groups.
    dest_slot is the union position (the batch kernels do not use it)."""
    if not 1 <= len(active_sets) <= MAX_TOKENS:
        raise ValueError(f"1..{MAX_TOKENS} tokens, got {len(active_sets)}")
    sets = [np.unique(np.asarray(s, dtype=np.int64)) for s in active_sets]
    for s in sets:
        if s.size and s[0] < 0:
            raise ValueError("negative group id")
    union = np.unique(np.concatenate(sets)) if any(s.size for s in sets) else np.zeros(0, np.int64)
    rows = np.zeros((len(union), 5), dtype=np.uint32)
    rows[:, 0] = union
    rows[:, 1] = union if physical is None else np.asarray(physical, dtype=np.int64)[union]
    rows[:, 2] = union if cache_slots is None else np.asarray(cache_slots, dtype=np.int64)[union]
    rows[:, 3] = np.arange(len(union), dtype=np.uint32)
    for i, g in enumerate(union.tolist()):
        if staging and g in staging:
            rows[i, 2] = staging[g]
            rows[i, 4] = N.SOURCE_STAGING
    mask = np.stack([np.isin(union, s) for s in sets]).astype(np.uint8) if len(union) else \
        np.zeros((len(sets), 0), np.uint8)
    return union, rows, mask


class BatchMLP:
    """One batched MLP layer call at a fixed geometry. Scratch is allocated
    once here (device memory for `max_union` groups) and reused by every
    call; calls on one BatchMLP must not overlap. `scratch` = (pointer,
    bytes) supplies caller-owned device memory instead; `error` is then the
    device address of a caller-owned, zeroed 32-bit error word (or None: the
    kernels record none), so that nothing is allocated here."""

    def __init__(self, hidden: int, group_size: int, max_union: int, device=None,
                 scratch: Optional[tuple] = None, error: Optional[int] = None):
        self.lib = N.load()
        self.hidden, self.group_size, self.max_union = hidden, group_size, max_union
        self.scratch_bytes = int(self.lib.ls_b200_batch_scratch_bytes(hidden, group_size, max_union))
        self._scratch = None
        if scratch is not None:
            self.scratch_ptr, have = int(scratch[0]), int(scratch[1])
            if have < self.scratch_bytes:
                raise ValueError(f"scratch of {have} B, {self.scratch_bytes} B needed")
            self._error = None
            self.error_ptr = int(error or 0)
        else:
            import torch

            self._scratch = torch.empty(self.scratch_bytes, dtype=torch.uint8, device=device or "cuda")
            self.scratch_ptr = self._scratch.data_ptr()
            # the tensor-core kernels' error word (ls_b200_batch_args.error), sticky
            self._error = torch.zeros(1, dtype=torch.int32, device=device or "cuda")
            self.error_ptr = self._error.data_ptr()

    def args(self, *, x, output, cache, scales, union_descs, union_count: int, tokens: int, mask=None,
             residual=None, hidden_out=None, output_f32=None, staging=None, norm_input=False, rms_eps=1e-5,
             norm_weight=None, mma_sync=False, timeout_ns=0) -> N.BatchArgs:
        """norm_input: HF RMSNorm of each token before the MLP (with residual
        and hidden_out, one layer of a decode stack). mma_sync: the legacy
        warp-level MMA kernels instead of tcgen05 (for comparison).
        timeout_ns: bound of the tcgen05 kernels' waits (0 = 2 s)."""
        if union_count > self.max_union:
            raise ValueError(f"union of {union_count} groups, BatchMLP sized for {self.max_union}")
        return N.BatchArgs(self.hidden, self.group_size, union_count, tokens, _ptr(x), _ptr(output),
                           _ptr(output_f32), _ptr(residual), _ptr(hidden_out), _ptr(cache), _ptr(staging),
                           _ptr(scales), _ptr(union_descs), _ptr(mask), self.scratch_ptr, self.scratch_bytes,
                           (N.NORM_INPUT if norm_input else 0) | (N.BATCH_MMA_SYNC if mma_sync else 0), rms_eps,
                           _ptr(norm_weight), self.error_ptr, int(timeout_ns))

    def clear_error(self) -> None:
        """Zeroes the owned error word (stream-ordered on torch's current stream)."""
        if self._error is None:
            raise RuntimeError("the error word is caller-owned (BatchMLP(error=...)): clear it there")
        self._error.zero_()

    def error(self) -> int:
        """Nonzero when a bounded wait of a tensor-core kernel gave up (the
        outputs of that call are invalid); reads a device word."""
        if self._error is None:
            raise RuntimeError("the error word is caller-owned (BatchMLP(error=...)): read it there")
        return int(self._error.item())

    def run(self, stream=None, **kw) -> None:
        """Enqueues one layer (three launches) on `stream` (a torch stream,
        a raw cudaStream_t as int, or None for torch's current stream).
        Keyword arguments as `args`; tensors or raw device pointers."""
        a = self.args(**kw)
        if stream is None:
            import torch

            stream = torch.cuda.current_stream()
        handle = stream if isinstance(stream, int) else stream.cuda_stream
        _check(self.lib.ls_b200_batch_mlp(C.byref(a), handle), "ls_b200_batch_mlp")
