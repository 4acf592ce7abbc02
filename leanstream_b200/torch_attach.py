"""Inference-only PyTorch attachment on the B200 backend: the interface of
leanstream/integrations/torch (attach_leanstream, contracts.py, attachment.py,
inspection.py) with the sm_100a kernel in place of the Triton Group2 bundle
(compute.py:8-66) and a host step in place of the native bridge
(integrations/torch/native/bridge.cpp:56-110).

Per decoder layer, `SparseMLP` replaces the MLP module for batch-1 decode
([1, 1, H] fp16 on CUDA) and delegates every other shape to the original
module (attachment.py:12-38). A layer step follows the reference runtime's
order (runtime.h, weight_manager.cpp:124-205): begin (decoder pre-hook, early
prediction -> update) -> Progressive: enqueue the kernel, then the final
prediction -> finalize (the kernel consumes descriptors as they are
published) / basic: finalize, wait for the reads, then enqueue -> output ->
commit. Resident groups live in HBM (`cache`, slot = position in
CachePolicy.resident); the others stay in pinned host memory and are copied
to HBM staging by the streaming IO engine (ls_b200_stream_*) when predicted.
Unlike the reference's Group2 bundle, any group size the kernel supports
works (WeightSpec.group_size; the reference fixes 2), there is no SM87 gate,
and core groups need not come in pairs.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass
from functools import wraps
from pathlib import Path
from typing import Callable, Optional

import numpy as np
import torch

from . import _native as N
from .backend import B200Backend, ExecutionQueue
from .stream import IOBackendView, StreamEngine


# ------------------------------------------------------------------ contracts (contracts.py)
@dataclass(frozen=True)
class ModelPoints:
    layers: str = "model.layers"
    mlp: str = "mlp"
    attention: str = "self_attn"
    pre_mlp_norm: str = "post_attention_layernorm"

    @classmethod
    def auto(cls):
        return cls(layers="auto")


@dataclass(frozen=True)
class GroupLayout:
    logical_group: int
    physical_group: int
    file_offset: int
    bytes: int


@dataclass(frozen=True)
class WeightSpec:
    """Packed INT4 groups in a file: group g's G neuron records
    [gate H/2 | up H/2 | down H/2] at layout[g].file_offset; fp16 scales
    [physical_group, G, 3, H/128] on the CPU."""
    path: Path
    width: int
    layout: tuple
    scales: object
    group_size: int = 2

    @property
    def group_count(self):
        return len(self.layout)

    @property
    def group_bytes(self):
        return self.group_size * 3 * self.width // 2

    def validate(self):
        n, b = self.group_count, self.group_bytes
        if n < 1 or self.width < 256 or self.width % 256 or not 1 <= self.group_size <= 256:
            raise ValueError("width must be a multiple of 256 (<= 8192), group size 1..256")
        if {x.logical_group for x in self.layout} != set(range(n)) or \
                {x.physical_group for x in self.layout} != set(range(n)):
            raise ValueError("Logical and physical IDs must each be permutations")
        if any(x.bytes != b or x.file_offset < 0 for x in self.layout):
            raise ValueError("Invalid extents")
        ranges = sorted((x.file_offset, x.file_offset + b) for x in self.layout)
        if any(a[1] > c[0] for a, c in zip(ranges, ranges[1:])):
            raise ValueError("Overlapping weight extents")
        if not Path(self.path).is_file() or Path(self.path).stat().st_size < ranges[-1][1]:
            raise ValueError("Missing/truncated weight file")
        if self.scales.device.type != "cpu" or self.scales.dtype != torch.float16 or \
                self.scales.numel() != n * self.group_size * 3 * self.width // 128 or \
                not torch.isfinite(self.scales).all():
            raise ValueError("Expected finite CPU FP16 physical scale table")


@dataclass(frozen=True)
class CachePolicy:
    resident: tuple
    core: tuple

    def validate(self, n):
        for ids in (self.resident, self.core):
            if len(set(ids)) != len(ids) or any(type(i) != int or not 0 <= i < n for i in ids):
                raise ValueError("Invalid resident/core IDs")
        if not set(self.core) <= set(self.resident):
            raise ValueError("Core must be a resident subset")


@dataclass(frozen=True)
class PredictionStage:
    predictor: Callable
    budget: int
    io_budget: int


@dataclass(frozen=True)
class PredictionSchedule:
    final: PredictionStage
    early: Optional[PredictionStage] = None

    def validate(self, n, mode):
        if mode not in ("basic", "progressive"):
            raise ValueError("Mode must be basic or progressive")
        if (mode == "progressive") != (self.early is not None):
            raise ValueError("Progressive requires early; Basic excludes early")
        for stage in (self.early, self.final):
            if stage and (not callable(stage.predictor) or not 0 < stage.budget <= n or
                          not 0 <= stage.io_budget <= n):
                raise ValueError("Invalid prediction budget")


@dataclass(frozen=True)
class ComputeSpec:
    candidate: int = -1        # KernelSelector catalog id, -1 = the selector's choice
    queue_depth: int = 8       # copies in flight per layer (ManagerConfig::qd)
    timeout_us: int = 2_000_000
    check_execution: bool = False  # per-dest execution counters (correctness only)


def ranked_ids(value, n, budget):
    ids = list(value)
    if len(ids) > budget or any(type(i) != int or not 0 <= i < n for i in ids) or len(set(ids)) != len(ids):
        raise ValueError("Predictor must return unique, in-range Python integer logical IDs within budget")
    return ids


# ------------------------------------------------------------------ inspection (inspection.py)
def resolve(root, path):
    value = root
    for part in path.split("."):
        value = value[int(part)] if part.isdecimal() else getattr(value, part)
    return value


def inspect_model(model, points=None):
    """Structural discovery of decoder layers with gated (gate/up/down) MLPs."""
    points = points or ModelPoints.auto()
    paths = [points.layers] if points.layers != "auto" else ["model.layers", "model.model.layers", "layers"]
    candidates = []
    for path in paths:
        try:
            layers = resolve(model, path)
            if len(layers) > 0:
                candidates.append((path, layers))
        except (AttributeError, TypeError, KeyError):
            pass
    report = dict(compatible=False, ambiguities=[], missing=[], layers=[], points=None)
    if len(candidates) != 1:
        report["ambiguities"] = [p for p, _ in candidates]
        report["missing"] = ["Specify a unique decoder layer path"]
        return report
    path, layers = candidates[0]
    chosen = ModelPoints(path, points.mlp, points.attention, points.pre_mlp_norm)
    seen = set()
    for i, layer in enumerate(layers):
        row = dict(index=i, path=f"{path}.{i}", compatible=False)
        try:
            mlp = resolve(layer, chosen.mlp)
            norm = resolve(layer, chosen.pre_mlp_norm)
            if id(layer) in seen or id(mlp) in seen:
                raise ValueError("Shared/reentrant layers or MLPs unsupported")
            seen.update([id(layer), id(mlp)])
            g, u, d = mlp.gate_proj, mlp.up_proj, mlp.down_proj
            h, j = g.in_features, g.out_features
            if u.in_features != h or u.out_features != j or d.in_features != j or d.out_features != h:
                raise ValueError("Inconsistent gated projections")
            if any(getattr(p, "bias", None) is not None for p in (g, u, d)):
                raise ValueError("Bias unsupported")
            if norm.weight.numel() != h:
                raise ValueError("Normalization geometry")
            row.update(compatible=True, hidden=h, intermediate=j)
        except (AttributeError, ValueError, TypeError) as e:
            row["reason"] = str(e)
            report["missing"].append(f"{path}.{i}: {e}")
        report["layers"].append(row)
    report["compatible"] = bool(report["layers"]) and all(r["compatible"] for r in report["layers"])
    report["points"] = chosen
    return report


# ------------------------------------------------------------------ one layer's runtime
class LayerRuntime:
    """Device state and the layer step of one decoder layer: the roles of the
    reference's WeightManager (weight_manager.cpp:124-205) and bridge
    (bridge.cpp:80-110) over the B200 backend and streaming engine."""

    def __init__(self, spec: WeightSpec, policy: CachePolicy, compute: ComputeSpec, device=None):
        spec.validate()
        policy.validate(spec.group_count)
        self.spec, self.policy, self.compute = spec, policy, compute
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.dev = dev
        n, gb, H, G = spec.group_count, spec.group_bytes, spec.width, spec.group_size
        self.n, self.gb = n, gb
        by_id = {x.logical_group: x for x in spec.layout}
        raw = np.fromfile(spec.path, dtype=np.uint8)
        self.cache_slot = np.full(n, -1, np.int64)
        for i, g in enumerate(policy.resident):
            self.cache_slot[g] = i
        res = [raw[by_id[g].file_offset:by_id[g].file_offset + gb] for g in policy.resident]
        self.cache = torch.from_numpy(np.concatenate(res) if res else np.zeros(gb, np.uint8)).to(dev)
        # non-resident groups: pinned host memory, streamed into staging slot = logical id
        self.host = torch.zeros(n * gb, dtype=torch.uint8).pin_memory()
        host_np = self.host.numpy()
        for g in range(n):
            if self.cache_slot[g] < 0:
                host_np[g * gb:(g + 1) * gb] = raw[by_id[g].file_offset:by_id[g].file_offset + gb]
        self.staging = torch.zeros(n * gb, dtype=torch.uint8, device=dev)
        self.scales = spec.scales.contiguous().reshape(-1).to(dev)
        self.physical = np.array([by_id[g].physical_group for g in range(n)], np.uint32)
        core_rows = np.array([[g, self.physical[g], self.cache_slot[g], i, N.SOURCE_CACHE]
                              for i, g in enumerate(policy.core)], np.uint32).reshape(-1, 5)
        self.core = torch.from_numpy(core_rows.reshape(-1).view(np.int32).copy()).to(dev) if len(policy.core) else None
        self.x = torch.zeros(H, dtype=torch.float16, device=dev)
        self.y = torch.zeros(H, dtype=torch.float16, device=dev)
        self.execs = torch.zeros(n, dtype=torch.int32, device=dev) if compute.check_execution else None
        self.backend = B200Backend().configure(H, G, n, max_layers=1, staging_slots=n, physical_groups=n,
                                               timeout_us=compute.timeout_us)
        self.queue = ExecutionQueue(n)
        self.engine = StreamEngine(self.host.data_ptr(), [g * gb for g in range(n)], self.staging.data_ptr(), gb, gb,
                                   queue_depth=compute.queue_depth, device=dev.index or 0)
        self.io = IOBackendView(self.engine.view())
        self.lock = threading.Lock()
        self.epoch = 0
        self.active = self.finalized = False
        self.final_index = {}
        self.published = set()
        self.done = torch.cuda.Event()

    # -- IO completions (worker thread): publish a landed final read
    def _landed(self, epoch, group, slot, error, seq):
        if error:
            with self.lock:
                self.queue.fail(error)
            return
        with self.lock:
            if not self.active or epoch != self.epoch or not self.finalized:
                return
            self._publish(group)

    def _publish(self, g):
        i = self.final_index.get(g)
        if i is None or g in self.published:
            return
        self.published.add(g)
        self.queue.publish(i)

    def begin(self):
        if self.active:
            raise RuntimeError("layer step already active")
        self.epoch += 1
        self.queue.reset(self.epoch)
        self.final_index, self.published = {}, set()
        self.finalized = False
        if self.execs is not None:
            self.execs.zero_()
        rc = self.io.begin(self._landed, self.epoch)
        if rc:
            raise RuntimeError(f"IO begin failed: {rc}")
        self.active = True

    def update(self, ids, io_budget):
        # only groups that are neither resident nor already read (weight_manager.cpp:135-151)
        todo = [g for g in ids if self.cache_slot[g] < 0 and self.engine.io_states[g] == N.IO_EMPTY][:io_budget]
        rc = self.io.update(todo)
        if rc:
            raise RuntimeError(f"IO update failed: {rc}")

    def finalize(self, ids):
        core = set(self.policy.core)
        if not core <= set(ids):
            raise ValueError("Final selection must include every configured core group")
        rest = [g for g in ids if g not in core]
        if len(rest) > self.n:
            raise ValueError("final set exceeds the queue")
        rows = np.zeros((len(rest), 5), np.uint32)
        nc = len(self.policy.core)
        for i, g in enumerate(rest):
            slot = self.cache_slot[g]
            rows[i] = (g, self.physical[g], slot if slot >= 0 else g, nc + i,
                       N.SOURCE_CACHE if slot >= 0 else N.SOURCE_STAGING)
        reads = [g for g in rest if self.cache_slot[g] < 0]
        with self.lock:
            if len(rows):
                self.queue.write_descriptors(rows)
            self.final_index = {g: i for i, g in enumerate(rest)}
            self.queue.prepare(len(rest))
            self.finalized = True
            for i, g in enumerate(rest):
                if self.cache_slot[g] >= 0 or self.engine.io_states[g] == N.IO_READY:
                    self.published.add(g)
                    self.queue.append_unpublished(i)
            self.queue.activate()
        rc = self.io.consume(reads)
        if rc:
            with self.lock:
                self.queue.fail(rc)
            raise RuntimeError(f"IO consume failed: {rc}")

    def wait_io(self, timeout_ms=5000):
        return self.io.wait(timeout_ms)

    def enqueue(self, x, stream=None):
        self.x.copy_(x.reshape(-1))
        args = self.backend.layer_args(input=self.x, output=self.y, cache=self.cache, staging=self.staging,
                                       scales=self.scales, core=self.core, core_count=len(self.policy.core),
                                       epoch=self.epoch, queue=self.queue.view, mode=N.MODE_PROGRESSIVE,
                                       candidate=self.compute.candidate, executions=self.execs)
        self.backend.launch(args, stream)
        self.done.record(stream)

    def output(self, shape):
        return self.y.reshape(shape).clone()

    def commit(self):
        self.done.synchronize()  # GPU completion before the reads' buffers are recycled
        st = self.backend.status()
        rc = self.io.retire()
        self.active = False
        if st[N.STATUS_ERROR]:
            self.backend.clear_status()
            raise RuntimeError(f"device status {st}")
        if rc:
            raise RuntimeError(f"IO retire failed: {rc}")

    def abort(self):
        if not self.active:
            return
        with self.lock:
            self.queue.fail(125)  # ECANCELED: the kernel observes the error word and exits
        torch.cuda.current_stream().synchronize()
        self.io.retire()
        self.active = False
        if self.backend.status()[N.STATUS_ERROR]:
            self.backend.clear_status()

    def close(self):
        self.abort()
        self.engine.close()
        self.backend.close()


# ------------------------------------------------------------------ module replacement (attachment.py)
class SparseMLP(torch.nn.Module):
    def __init__(self, original, owner, index, runtime: LayerRuntime):
        super().__init__()
        self.original, self.owner, self.index, self.runtime = original, owner, index, runtime
        self.pending = False
        self.future = None
        self.trace = []

    @staticmethod
    def decode(x):
        return x.ndim == 3 and tuple(x.shape[:2]) == (1, 1)

    def predict(self, stage, x, source):
        return stage.predictor(source, self.index, x, stage.budget)

    def publish(self, value, stage):
        if hasattr(value, "done"):
            if not value.done():
                return False
            value = value.result()
        ids = ranked_ids(value, self.runtime.n, stage.budget)
        self.runtime.update(ids, stage.io_budget)
        return ids

    def begin(self, x):
        if torch.is_grad_enabled():
            raise RuntimeError("Use torch.inference_mode(); training/autograd unsupported")
        if not self.decode(x):
            if x.ndim != 3 or x.shape[0] != 1:
                raise ValueError("Only batch1 [1,sequence,H] supported")
            return
        if x.device.type != "cuda" or x.dtype != torch.float16:
            raise ValueError("Decode requires CUDA FP16")
        self.runtime.begin()
        self.pending = True
        self.trace = []
        early = self.owner.prediction.early
        if early:
            try:
                self.future = self.predict(early, x, "layer_input")
                self.publish(self.future, early)
            except BaseException:
                self.abort()
                raise

    def abort(self):
        if self.pending:
            self.runtime.abort()
            self.pending = False

    def forward(self, x):
        if not self.decode(x):
            return self.original(x)
        if not self.pending:
            raise RuntimeError("MLP must run inside its configured decoder layer")
        try:
            if x.dtype != torch.float16 or x.device.type != "cuda" or x.shape[-1] != self.runtime.spec.width:
                raise ValueError("MLP input geometry/dtype")
            final = self.owner.prediction.final
            stream = torch.cuda.current_stream()
            if self.owner.mode == "progressive":
                # the launch precedes the final prediction: the kernel consumes
                # the queue as descriptors are published
                self.runtime.enqueue(x, stream)
                self.trace.append("pre_enqueue")
            ids = self.publish(self.predict(final, x, "mlp_input"), final)
            if ids is False:
                raise ValueError("Final prediction must already be CPU-ready")
            self.runtime.finalize(ids)
            self.trace.append("finalize")
            if self.owner.mode == "basic":
                rc = self.runtime.wait_io(5000)
                if rc:
                    raise RuntimeError(f"IO wait failed: {rc}")
                self.runtime.enqueue(x, stream)
                self.trace.append("basic_enqueue_after_io")
            result = self.runtime.output(x.shape)
            self.runtime.commit()
            self.pending = False
            return result
        except BaseException:
            self.abort()
            raise


class Attachment:
    def __init__(self, model, points, weights, compute, cache_policy, prediction, mode):
        if getattr(model, "_leanstream_attachment", None) is not None:
            raise ValueError("Model already attached")
        if model.training:
            raise ValueError("Call model.eval(); training is unsupported")
        report = inspect_model(model, points)
        if not report["compatible"]:
            raise ValueError(f"Manual inspection required: {report}")
        points = report["points"]
        layers = resolve(model, points.layers)
        if not len(weights) == len(cache_policy) == len(layers):
            raise ValueError("One weight/policy specification per layer required")
        self.model, self.prediction, self.mode = model, prediction, mode
        self.entries, self.hooks, self.guards, self.closed = [], [], [], False
        for row, w, p in zip(report["layers"], weights, cache_policy):
            w.validate()
            p.validate(w.group_count)
            prediction.validate(w.group_count, mode)
            if row["hidden"] != w.width or row["intermediate"] != w.group_count * w.group_size:
                raise ValueError("Packed weight/model dimensions differ")
        try:
            for i, (layer, w, p) in enumerate(zip(layers, weights, cache_policy)):
                original = resolve(layer, points.mlp)
                replacement = SparseMLP(original, self, i, LayerRuntime(w, p, compute))
                parent = resolve(layer, points.mlp.rsplit(".", 1)[0]) if "." in points.mlp else layer
                name = points.mlp.split(".")[-1]
                setattr(parent, name, replacement)
                self.entries.append((parent, name, original, replacement))

                def begin(module, args, kwargs, r=replacement):
                    x = args[0] if args else kwargs.get("hidden_states")
                    if not isinstance(x, torch.Tensor):
                        raise ValueError("Decoder must expose hidden_states as first positional/keyword Tensor")
                    r.begin(x)

                original_forward = layer.forward

                @wraps(original_forward)
                def guarded(*args, _forward=original_forward, _r=replacement, **kwargs):
                    try:
                        return _forward(*args, **kwargs)
                    finally:
                        if _r.pending:
                            _r.abort()

                self.guards.append((layer, original_forward))
                layer.forward = guarded
                self.hooks.append(layer.register_forward_pre_hook(begin, with_kwargs=True))
            model._leanstream_attachment = self
        except BaseException:
            self.close()
            raise

    def refine(self, layer, ids, io_budget):
        r = self.entries[layer][3]
        if not r.pending:
            raise ValueError("No active layer to refine")
        ids = ranked_ids(ids, r.runtime.n, r.runtime.n)
        if not 0 <= io_budget <= r.runtime.n:
            raise ValueError("Invalid I/O budget")
        r.runtime.update(ids, io_budget)

    def reset(self):
        for *_, r in self.entries:
            r.abort()

    def close(self):
        if self.closed:
            return
        for hook in self.hooks:
            hook.remove()
        self.hooks.clear()
        for layer, original_forward in self.guards:
            layer.forward = original_forward
        self.guards.clear()
        for parent, name, original, r in reversed(self.entries):
            try:
                r.abort()
                r.runtime.close()
            finally:
                setattr(parent, name, original)
        self.entries.clear()
        self.closed = True
        if getattr(self.model, "_leanstream_attachment", None) is self:
            del self.model._leanstream_attachment

    detach = close

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def attach_leanstream(model, *, points, weights, compute, cache_policy, prediction, mode="progressive"):
    """Returns a lifecycle handle; keep calling the original model.forward/generate."""
    return Attachment(model, points, weights, compute, cache_policy, prediction, mode)
