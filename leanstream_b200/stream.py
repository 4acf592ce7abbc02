"""Streaming IO over pinned host memory (ls_b200_stream_*): the IOBackend of
include/leanstream/weight_manager.h:14-24 for a discrete GPU.

The engine copies the groups a WeightManager asks for from pinned host memory
into HBM staging (group g at ``staging + g * stride``), one cudaMemcpyAsync per
group on its own stream, in the priority order of the last ``update`` and then
the committed final reads; ``io_states`` words turn READY before the
completion callback runs. ``IOBackendView`` exposes the same seven entry
points for Python callers and tests.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, Optional, Sequence

import numpy as np

from . import _native as N

_BEGIN = C.CFUNCTYPE(C.c_int, C.c_void_p, N.IO_COMPLETION_FN, C.c_void_p, C.c_uint32)
_SPAN = C.CFUNCTYPE(C.c_int, C.c_void_p, N.GroupSpan)
_RETIRE = C.CFUNCTYPE(C.c_int, C.c_void_p)
_READY_SLOT = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.c_int32)
_REQUESTS = C.CFUNCTYPE(C.c_uint64, C.c_void_p)
_WAIT = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int)


def _check(rc: int, what: str) -> None:
    if rc:
        raise RuntimeError(f"{what} failed: {rc}")


class StreamEngine:
    """Owns one engine (worker thread, copy stream, events) on `device`.

    `host_base`: address of pinned host memory holding every group;
    `offsets[g]`: byte offset of group g there; `staging`: device address of
    the staging area (stride `stride` >= `group_bytes`)."""

    def __init__(self, host_base: int, offsets: Sequence[int], staging: int, stride: int, group_bytes: int,
                 queue_depth: int = 8, device: int = 0, delay_mean_us: float = 0.0, delay_seed: int = 0,
                 file_path: Optional[str] = None, file_offsets: Optional[Sequence[int]] = None,
                 read_workers: int = 4, o_direct: bool = True, file_alignment: int = 4096):
        """With `file_path`, each admitted group is first read from the file
        at `file_offsets[g]` into its host slot (the SSD leg), then copied."""
        self.lib = N.load()
        self.count = len(offsets)
        self.offsets = np.ascontiguousarray(np.asarray(offsets, dtype=np.uint64))
        self.io_states = np.zeros(self.count + 1, dtype=np.uint32)  # shared with the worker
        self.file_offsets = (np.ascontiguousarray(np.asarray(file_offsets, dtype=np.uint64))
                             if file_offsets is not None else None)
        self._path = file_path.encode() if file_path else None
        cfg = N.StreamConfig(host_base, self.offsets.ctypes.data, staging, stride, group_bytes,
                             self.io_states.ctypes.data, self.count, queue_depth, device, delay_mean_us, delay_seed,
                             self._path, self.file_offsets.ctypes.data if self.file_offsets is not None else None,
                             read_workers, 1 if o_direct else 0, file_alignment)
        self.engine = self.lib.ls_b200_stream_create(C.byref(cfg))
        if not self.engine:
            raise RuntimeError(f"ls_b200_stream_create failed (errno {C.get_errno()})")

    def view(self) -> N.IOBackend:
        v = N.IOBackend()
        _check(self.lib.ls_b200_stream_view(self.engine, C.byref(v)), "ls_b200_stream_view")
        return v

    def stats(self) -> dict:
        s = N.StreamStats()
        _check(self.lib.ls_b200_stream_stats(self.engine, C.byref(s)), "ls_b200_stream_stats")
        return {k: getattr(s, k) for k, _ in N.StreamStats._fields_}

    def issue_log(self) -> list:
        out = (C.c_int32 * self.count)()
        n = self.lib.ls_b200_stream_issue_log(self.engine, out, self.count)
        return list(out[:n])

    def close(self) -> None:
        if self.engine:
            self.lib.ls_b200_stream_destroy(self.engine)
            self.engine = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class IOBackendView:
    """Calls through an IOBackend table (any implementation), the way a
    WeightManager does (weight_manager.cpp:124-205)."""

    def __init__(self, table: N.IOBackend):
        self.table = table
        self.ctx = table.context
        self._begin = _BEGIN(table.begin)
        self._update = _SPAN(table.update)
        self._consume = _SPAN(table.consume)
        self._retire = _RETIRE(table.retire)
        self._ready_slot = _READY_SLOT(table.ready_slot)
        self._requests = _REQUESTS(table.requests)
        self._wait = _WAIT(table.wait)
        self._callback = None

    def begin(self, on_completion: Callable[[int, int, int, int, int], None], epoch: int) -> int:
        """on_completion(epoch, group, slot, error, sequence) runs on the engine's worker thread."""

        def trampoline(_arg, c):
            v = c.contents
            on_completion(v.epoch, v.logical_group, v.staging_slot, v.error, v.slot_sequence)

        callback = N.IO_COMPLETION_FN(trampoline)
        rc = self._begin(self.ctx, callback, None, epoch)
        if rc == 0:
            # the engine calls it until the session retires: keep it alive (a
            # refused begin leaves the running session's callback in place)
            self._callback = callback
        return rc

    @staticmethod
    def _span(ids):
        arr = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        return arr, N.GroupSpan(arr.ctypes.data if arr.size else None, arr.size)

    def update(self, ids) -> int:
        arr, span = self._span(ids)
        return self._update(self.ctx, span)

    def consume(self, ids) -> int:
        arr, span = self._span(ids)
        return self._consume(self.ctx, span)

    def retire(self) -> int:
        return self._retire(self.ctx)

    def ready_slot(self, group: int) -> int:
        return self._ready_slot(self.ctx, group)

    def requests(self) -> int:
        return self._requests(self.ctx)

    def wait(self, timeout_ms: int) -> int:
        return self._wait(self.ctx, timeout_ms)
