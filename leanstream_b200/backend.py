"""Host-side mirror of the reference's native backend API, over the B200 C ABI.

`B200Backend` follows backends/triton/binding.py:29-67 (NativeBackend):
create / create_table, cold configuration, enqueue, close. The caller owns
every buffer and keeps it alive until GPU completion. `ExecutionQueue`
restates include/leanstream/execution_queue.h:19-34 on mapped pinned memory.
PyTorch only supplies device / pinned allocations and streams.
"""
from __future__ import annotations

import ctypes as C
import errno
from typing import Optional, Sequence

import numpy as np

from . import _native as N


def _check(rc: int, what: str) -> None:
    if rc:
        name = errno.errorcode.get(rc, str(rc))
        raise RuntimeError(f"{what} failed: {name} ({rc})")


def _ptr(t) -> Optional[int]:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


class ExecutionQueue:
    """ExecutionQueue over a DeviceExecQueue whose storage is mapped pinned
    host memory (GPU-readable through UVA, written by host release stores).

    Mirrors reset/prepare/append_unpublished/activate/seal/publish_all/
    publish/fail of src/runtime/execution_queue.cpp:4-46.
    """

    def __init__(self, capacity: int):
        import torch

        self.capacity = capacity
        self.desc = torch.zeros(max(capacity, 1) * 5, dtype=torch.int32, pin_memory=True)
        self.indices = torch.zeros(max(capacity, 1), dtype=torch.int32, pin_memory=True)
        self.control = torch.zeros(32, dtype=torch.int32, pin_memory=True)  # 128 B, QueueControl
        self.view = N.DeviceExecQueue(self.desc.data_ptr(), self.indices.data_ptr(), self.control.data_ptr(),
                                      capacity)
        self._q = N.Queue()
        N.load().ls_b200_queue_bind(C.byref(self._q), self.view)

    # host views
    @property
    def desc_host(self) -> np.ndarray:
        return self.desc.numpy().view(np.uint32).reshape(-1, 5)

    @property
    def control_host(self) -> np.ndarray:
        return self.control.numpy().view(np.uint32)

    def write_descriptors(self, rows) -> None:
        rows = np.asarray(rows, dtype=np.uint32).reshape(-1, 5)
        if len(rows) > self.capacity:
            raise ValueError("more descriptors than capacity")
        self.desc_host[: len(rows)] = rows

    def reset(self, epoch: int) -> None:
        _check(N.load().ls_b200_queue_reset(C.byref(self._q), epoch), "queue reset")

    def prepare(self, total: int) -> None:
        _check(N.load().ls_b200_queue_prepare(C.byref(self._q), total), "queue prepare")

    def append_unpublished(self, index: int) -> None:
        _check(N.load().ls_b200_queue_append_unpublished(C.byref(self._q), index), "queue append")

    def activate(self) -> None:
        _check(N.load().ls_b200_queue_activate(C.byref(self._q)), "queue activate")

    def seal(self, total: int) -> None:
        _check(N.load().ls_b200_queue_seal(C.byref(self._q), total), "queue seal")

    def publish_all(self) -> None:
        _check(N.load().ls_b200_queue_publish_all(C.byref(self._q)), "queue publish_all")

    def publish(self, index: int) -> None:
        _check(N.load().ls_b200_queue_publish(C.byref(self._q), index), "queue publish")

    def fail(self, error: int) -> None:
        _check(N.load().ls_b200_queue_fail(C.byref(self._q), error), "queue fail")


class DeviceQueue:
    """All-ready plan in DEVICE memory: descriptors, ready indices and
    QueueControl are built on a pinned host image with the same producer
    protocol, then copied with one cudaMemcpyAsync per buffer."""

    def __init__(self, capacity: int, device=None):
        import torch

        self.capacity = capacity
        self.host = ExecutionQueue(capacity)
        dev = device or torch.device("cuda")
        self.desc = torch.zeros_like(self.host.desc, device=dev)
        self.indices = torch.zeros_like(self.host.indices, device=dev)
        self.control = torch.zeros_like(self.host.control, device=dev)
        self.view = N.DeviceExecQueue(self.desc.data_ptr(), self.indices.data_ptr(), self.control.data_ptr(),
                                      capacity)

    def plan(self, rows, epoch: int) -> None:
        """Writes an all-ready plan (reset, descriptors, publish_all, epoch)."""
        h = self.host
        h.reset(epoch)
        h.write_descriptors(rows)
        h.prepare(len(np.asarray(rows).reshape(-1, 5)))
        h.publish_all()
        h.activate()

    def upload(self, stream=None) -> int:
        """Copies the host image to the device on `stream`; returns bytes copied."""
        import torch

        s = stream or torch.cuda.current_stream()
        with torch.cuda.stream(s):
            self.desc.copy_(self.host.desc, non_blocking=True)
            self.indices.copy_(self.host.indices, non_blocking=True)
            self.control.copy_(self.host.control, non_blocking=True)
        return (self.desc.numel() + self.indices.numel() + self.control.numel()) * 4


class B200Backend:
    """Owns one native backend context (NativeBackend, binding.py:29-67)."""

    def __init__(self, offline_table: Optional[Sequence[Sequence[int]]] = None):
        self.lib = N.load()
        self._table = None
        if offline_table is None:
            self.context = self.lib.ls_b200_create()
        else:
            layers, buckets = len(offline_table), len(offline_table[0])
            if not all(len(row) == buckets for row in offline_table):
                raise ValueError("Ragged LUT")
            self._table = (C.c_uint8 * (layers * buckets))(*(v for row in offline_table for v in row))
            self.context = self.lib.ls_b200_create_table(self._table, layers, buckets)
        if not self.context:
            raise MemoryError("Native backend allocation failed")
        self.geometry = None
        self._bound = None
        self._view = None

    # -- cold setup
    def configure(self, hidden: int, group_size: int, group_count: int, max_layers: int = 0, cache_slots: int = 0,
                  staging_slots: int = 0, physical_groups: int = 0, timeout_us: int = 0, rms_eps: float = 1e-5):
        g = N.Geometry(hidden, group_size, group_count, max_layers, cache_slots, staging_slots, physical_groups,
                       timeout_us, rms_eps)
        _check(self.lib.ls_b200_configure(self.context, C.byref(g)), "ls_b200_configure")
        self.geometry = g
        return self

    @staticmethod
    def layer_args(*, input=None, output=None, cache=None, staging=None, scales=None, core=None, core_count=0,
                   epoch=0, queue: Optional[N.DeviceExecQueue] = None, mode=N.MODE_PROGRESSIVE, flags=0,
                   candidate=-1, layer=0, activations=None, executions=None, first_compute=None, residual=None,
                   hidden_out=None, output_f32=None, norm_weight=None, trace=None, importance=None,
                   importance_flag=None) -> N.LayerArgs:
        a = N.LayerArgs()
        a.input, a.output = _ptr(input), _ptr(output)
        a.cache, a.staging, a.scales = _ptr(cache), _ptr(staging), _ptr(scales)
        a.core, a.core_count, a.epoch = _ptr(core), core_count, epoch
        if queue is not None:
            a.queue = queue
        a.mode, a.flags, a.candidate, a.layer = mode, flags, candidate, layer
        a.activations, a.executions, a.first_compute = _ptr(activations), _ptr(executions), _ptr(first_compute)
        a.residual, a.hidden_out, a.output_f32, a.norm_weight = (_ptr(residual), _ptr(hidden_out),
                                                                  _ptr(output_f32), _ptr(norm_weight))
        a.trace = _ptr(trace)
        a.importance, a.importance_flag = _ptr(importance), _ptr(importance_flag)
        return a

    def set_buffers(self, **kw) -> None:
        self._bound = self.layer_args(**kw)
        _check(self.lib.ls_b200_set_buffers(self.context, C.byref(self._bound)), "ls_b200_set_buffers")

    def set_state(self, layer: int, io_bucket: int) -> None:
        self.lib.ls_b200_set_state(self.context, layer, io_bucket)

    # -- submission
    def launch(self, args: N.LayerArgs, stream=None) -> None:
        _check(self.lib.ls_b200_launch(self.context, C.byref(args), _stream(stream)), "ls_b200_launch")

    def launch_rc(self, args: N.LayerArgs, stream=None) -> int:
        return int(self.lib.ls_b200_launch(self.context, C.byref(args), _stream(stream)))

    def plan_size(self) -> int:
        return int(self.lib.ls_b200_plan_size())

    def encode_plan(self, args: N.LayerArgs) -> bytes:
        """Encodes one layer (validated on the host) for ls_b200_launch_plans."""
        buf = (C.c_uint8 * self.plan_size())()
        _check(self.lib.ls_b200_encode_plan(self.context, C.byref(args), buf), "ls_b200_encode_plan")
        return bytes(buf)

    def launch_plans(self, device_plans, count: int, host_plans, candidate: int = -1, trace=None,
                     stream=None) -> None:
        """One persistent launch over `count` layers. `device_plans` is a
        16-byte-aligned device copy of `host_plans` (encoded plans)."""
        hp = host_plans if isinstance(host_plans, int) else _ptr(host_plans)
        _check(self.lib.ls_b200_launch_plans(self.context, _ptr(device_plans), count, hp, candidate, _ptr(trace),
                                             _stream(stream)), "ls_b200_launch_plans")

    # -- tensor parallel inside one launch
    def tp_setup(self, rank: int, world: int) -> bytes:
        """Allocates this rank's exchange buffer; returns its IPC handle."""
        h = (C.c_uint8 * N.TP_HANDLE_BYTES)()
        _check(self.lib.ls_b200_tp_setup(self.context, rank, world, h), "ls_b200_tp_setup")
        return bytes(h)

    def tp_connect(self, handles: Sequence[bytes]) -> None:
        """Maps the peers' exchange buffers (handles in rank order). Every
        launch afterwards is a collective of the ranks."""
        if any(len(h) != N.TP_HANDLE_BYTES for h in handles):
            raise ValueError("IPC handles of the wrong size")
        blob = (C.c_uint8 * (N.TP_HANDLE_BYTES * len(handles))).from_buffer_copy(b"".join(handles))
        _check(self.lib.ls_b200_tp_connect(self.context, blob), "ls_b200_tp_connect")

    def enqueue(self, layer: int, io_bucket: int, epoch: int, stream=None) -> None:
        _check(self.lib.ls_b200_enqueue(self.context, layer, io_bucket, epoch, _stream(stream)), "ls_b200_enqueue")

    def view(self) -> N.ComputeBackend:
        v = N.ComputeBackend()
        _check(self.lib.ls_b200_view(self.context, C.byref(v)), "ls_b200_view")
        self._view = v
        return v

    # -- state
    def status(self) -> list:
        words = (C.c_uint32 * N.STATUS_WORDS)()
        _check(self.lib.ls_b200_status(self.context, words, N.STATUS_WORDS), "ls_b200_status")
        return list(words)

    def clear_status(self) -> None:
        _check(self.lib.ls_b200_clear_status(self.context), "ls_b200_clear_status")

    def completed_epoch(self, layer: int) -> int:
        v = C.c_uint32()
        _check(self.lib.ls_b200_completed_epoch(self.context, layer, C.byref(v)), "ls_b200_completed_epoch")
        return v.value

    def select(self, layer: int, io_bucket: int) -> int:
        return int(self.lib.ls_b200_select(self.context, layer, io_bucket))

    def candidate(self, cid: int) -> dict:
        c = N.KernelCandidate()
        _check(self.lib.ls_b200_candidate(self.context, cid, C.byref(c)), "ls_b200_candidate")
        return dict(id=c.id, workers=c.workers, name=c.name.decode(), cta_count=c.cta_count, available=c.available)

    def scratch_bytes(self) -> int:
        return int(self.lib.ls_b200_scratch_bytes(self.context))

    def close(self) -> None:
        """Caller must have proved GPU completion before closing."""
        if self.context:
            self.lib.ls_b200_destroy(self.context)
            self.context = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _stream(stream) -> Optional[int]:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def quantize_io_load(remaining: int, total: int, buckets: int = 8) -> int:
    """quantize_io_load (src/runtime/kernel_selector.cpp:4-8) via the C ABI."""
    return int(N.load().ls_b200_quantize_io_load(remaining, total, buckets))
