"""Helpers for the GPU tests: device buffers of one layer and a driver that
launches the fused kernel through the C ABI (leanstream_b200.B200Backend)."""
from __future__ import annotations

import time

import numpy as np
import torch

from leanstream_b200 import B200Backend, ExecutionQueue
from leanstream_b200 import _native as N


def to_dev(a: np.ndarray, dtype=None, device="cuda") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(device)


class LayerBuffers:
    """Device copies of one layer (packed cache, scales, x) + outputs."""

    def __init__(self, H, G, N_groups, packed, scales, x, staging=None, device="cuda"):
        self.H, self.G, self.N = H, G, N_groups
        self.cache = to_dev(np.asarray(packed, dtype=np.uint8), device=device)
        self.staging = self.cache if staging is None else to_dev(np.asarray(staging, dtype=np.uint8), device=device)
        self.scales = to_dev(np.asarray(scales, dtype=np.float16).reshape(-1).view(np.int16), torch.float16, device)
        self.x = to_dev(np.asarray(x, dtype=np.float16).view(np.int16), torch.float16, device)
        self.y = torch.zeros(H, dtype=torch.float16, device=device)
        self.y32 = torch.zeros(H, dtype=torch.float32, device=device)
        self.act = torch.zeros(N_groups * G, dtype=torch.float16, device=device)
        self.execs = torch.zeros(N_groups, dtype=torch.int32, device=device)
        self.stamps = torch.zeros(N_groups, dtype=torch.int64, device=device)


def make_backend(H, G, N_groups, timeout_us=2_000_000, table=None, **kw) -> B200Backend:
    return B200Backend(table).configure(H, G, N_groups, timeout_us=timeout_us, **kw)


def run_layer(backend: B200Backend, buf: LayerBuffers, core_rows, queue_rows, *, mode=N.MODE_PROGRESSIVE,
              candidate=-1, epoch=1, order=None, publish="all", flags=0, residual=None, hidden_out=None,
              stream=None, core_dev=None, importance=None, importance_flag=None):
    """One layer with `core_rows` (A) and `queue_rows` (B) descriptors.

    publish="all": the plan is sealed and fully published before launch.
    publish="none": only the epoch is activated; the caller publishes.
    Returns (queue, core tensor)."""
    q = ExecutionQueue(max(len(queue_rows), 1))
    q.reset(epoch)
    if len(queue_rows):
        q.write_descriptors(queue_rows)
    q.prepare(len(queue_rows))
    if publish == "all":
        for i in (order if order is not None else range(len(queue_rows))):
            q.append_unpublished(int(i))
    q.activate()
    core = core_dev
    if core is None and len(core_rows):
        core = to_dev(np.asarray(core_rows, dtype=np.uint32).reshape(-1).view(np.int32))
    args = backend.layer_args(input=buf.x, output=buf.y, cache=buf.cache, staging=buf.staging, scales=buf.scales,
                              core=core, core_count=len(core_rows), epoch=epoch, queue=q.view, mode=mode,
                              candidate=candidate, activations=buf.act, executions=buf.execs,
                              first_compute=buf.stamps, output_f32=buf.y32, flags=flags, residual=residual,
                              hidden_out=hidden_out, importance=importance, importance_flag=importance_flag)
    backend.launch(args, stream)
    return q, core


def wait_stream(stream=None, timeout_s=10.0):
    """Polls the stream with a host deadline (persistent_mlp_test.cu:41-44)."""
    s = stream or torch.cuda.current_stream()
    ev = torch.cuda.Event()
    ev.record(s)
    deadline = time.monotonic() + timeout_s
    while not ev.query():
        if time.monotonic() > deadline:
            raise AssertionError("GPU work did not finish before the host deadline")
        time.sleep(0.001)
    torch.cuda.synchronize()
