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
from pathlib import Path
from typing import Callable, Optional

import numpy as np
import torch

from . import _native as N
from .backend import B200Backend, ExecutionQueue
from .stream import IOBackendView, StreamEngine


# ------------------------------------------------------------------ contracts
# Field names follow leanstream/integrations/torch/contracts.py so that
# attach_leanstream callers pass the same objects; every check below is this
# module's own (failures raise ValueError naming the offending field).
def _require(ok, what: str) -> None:
    if not ok:
        raise ValueError(what)


@dataclass(frozen=True)
class ModelPoints:
    """Where the decoder layers, their MLP, attention and pre-MLP norm live
    (dotted attribute paths; integers index sequences). layers="auto"
    searches the model for the decoder-layer list."""
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
        n, gb, H, G = self.group_count, self.group_bytes, self.width, self.group_size
        _require(n >= 1, "WeightSpec.layout: no groups")
        _require(256 <= H <= 8192 and H % 256 == 0, f"WeightSpec.width {H}: a multiple of 256 up to 8192")
        _require(1 <= G <= 256, f"WeightSpec.group_size {G}: 1..256")
        logical = np.sort(np.fromiter((e.logical_group for e in self.layout), np.int64, n))
        physical = np.sort(np.fromiter((e.physical_group for e in self.layout), np.int64, n))
        _require(np.array_equal(logical, np.arange(n)), "WeightSpec.layout: logical_group must cover 0..n-1 once")
        _require(np.array_equal(physical, np.arange(n)), "WeightSpec.layout: physical_group must cover 0..n-1 once")
        starts = np.sort(np.fromiter((e.file_offset for e in self.layout), np.int64, n))
        _require(all(e.bytes == gb for e in self.layout), f"WeightSpec.layout: every extent is {gb} bytes")
        _require(starts[0] >= 0 and np.all(np.diff(starts) >= gb), "WeightSpec.layout: extents overlap")
        path = Path(self.path)
        _require(path.is_file(), f"WeightSpec.path {path}: not a file")
        _require(path.stat().st_size >= starts[-1] + gb, f"WeightSpec.path {path}: shorter than the layout")
        sc = self.scales
        _require(isinstance(sc, torch.Tensor) and sc.device.type == "cpu" and sc.dtype == torch.float16,
                 "WeightSpec.scales: a CPU float16 tensor")
        _require(sc.numel() == n * G * 3 * (H // 128), "WeightSpec.scales: [physical_group, G, 3, H/128] elements")
        _require(bool(torch.isfinite(sc).all()), "WeightSpec.scales: non-finite entries")


@dataclass(frozen=True)
class CachePolicy:
    """Groups kept in HBM (resident, slot = position) and the core groups,
    a resident subset computed in every step."""
    resident: tuple
    core: tuple

    def validate(self, n):
        for name in ("resident", "core"):
            ids = getattr(self, name)
            _require(all(isinstance(i, int) and not isinstance(i, bool) for i in ids),
                     f"CachePolicy.{name}: Python int group IDs")
            _require(len(ids) == len(set(ids)), f"CachePolicy.{name}: repeated group IDs")
            _require(all(0 <= i < n for i in ids), f"CachePolicy.{name}: group IDs outside 0..{n - 1}")
        missing = sorted(set(self.core) - set(self.resident))
        _require(not missing, f"CachePolicy.core: groups {missing} are not resident")


@dataclass(frozen=True)
class PredictionStage:
    predictor: Callable
    budget: int
    io_budget: int


@dataclass(frozen=True)
class PredictionSchedule:
    """`final` chooses each step's groups; `early` (Progressive only) starts
    the reads before the final choice."""
    final: PredictionStage
    early: Optional[PredictionStage] = None

    def validate(self, n, mode):
        _require(mode in ("basic", "progressive"), f"mode {mode!r}: 'basic' or 'progressive'")
        if mode == "progressive":
            _require(self.early is not None, "PredictionSchedule.early: required in progressive mode")
        else:
            _require(self.early is None, "PredictionSchedule.early: only used in progressive mode")
        for name in ("early", "final"):
            st = getattr(self, name)
            if st is None:
                continue
            _require(callable(st.predictor), f"PredictionSchedule.{name}.predictor: not callable")
            _require(0 < st.budget <= n, f"PredictionSchedule.{name}.budget {st.budget}: 1..{n}")
            _require(0 <= st.io_budget <= n, f"PredictionSchedule.{name}.io_budget {st.io_budget}: 0..{n}")


@dataclass(frozen=True)
class ComputeSpec:
    candidate: int = -1        # KernelSelector catalog id, -1 = the selector's choice
    queue_depth: int = 8       # copies in flight per layer (ManagerConfig::qd)
    timeout_us: int = 2_000_000
    check_execution: bool = False  # per-dest execution counters (correctness only)


def checked_selection(value, n, budget):
    """A predictor's answer as a list of distinct group IDs in 0..n-1, at
    most `budget` of them, in the predictor's (priority) order."""
    ids = list(value)
    _require(len(ids) <= budget, f"prediction: {len(ids)} groups exceed the budget {budget}")
    _require(all(isinstance(i, int) and not isinstance(i, bool) for i in ids), "prediction: Python int group IDs")
    _require(all(0 <= i < n for i in ids), f"prediction: group IDs outside 0..{n - 1}")
    _require(len(set(ids)) == len(ids), "prediction: repeated group IDs")
    return ids


# ------------------------------------------------------------------ model inspection
def _walk(root, dotted: str):
    """The object at a dotted path below `root` (decimal parts index)."""
    obj = root
    for part in filter(None, dotted.split(".")):
        obj = obj[int(part)] if part.isdigit() else getattr(obj, part)
    return obj


def _has(root, dotted: str) -> bool:
    try:
        _walk(root, dotted)
        return True
    except (AttributeError, IndexError, KeyError, TypeError):
        return False


def _decoder_lists(model, points):
    """(path, ModuleList) pairs of the model whose every element carries
    the configured MLP point: the decoder-layer lists."""
    found = []
    for name, mod in model.named_modules():
        if isinstance(mod, torch.nn.ModuleList) and len(mod) and all(_has(m, points.mlp) for m in mod):
            found.append((name, mod))
    return found


class _Row(dict):
    """One decoder layer of an inspection report (dict access kept for
    callers of the reference's report)."""


def inspect_model(model, points=None):
    """Finds the decoder layers and checks that each has a bias-free gated
    MLP (gate/up: H -> I, down: I -> H) and a pre-MLP norm of width H.

    Returns a dict: compatible (bool), points (the resolved ModelPoints),
    layers (per layer: index, path, compatible, hidden, intermediate or
    reason), missing (what stops attachment) and ambiguities (candidate
    layer paths when the search is not unique)."""
    points = points or ModelPoints.auto()
    report = {"compatible": False, "points": None, "layers": [], "missing": [], "ambiguities": []}
    if points.layers == "auto":
        found = _decoder_lists(model, points)
        if len(found) != 1:
            report["ambiguities"] = [name for name, _ in found]
            report["missing"].append(f"{len(found)} module lists carry '{points.mlp}': set ModelPoints.layers")
            return report
        path, layers = found[0]
    else:
        path = points.layers
        try:
            layers = _walk(model, path)
            len(layers)
        except (AttributeError, IndexError, KeyError, TypeError):
            report["missing"].append(f"no decoder-layer sequence at '{path}'")
            return report
    points = ModelPoints(path, points.mlp, points.attention, points.pre_mlp_norm)
    owners = {}
    for i, layer in enumerate(layers):
        row = _Row(index=i, path=f"{path}.{i}", compatible=False)
        report["layers"].append(row)
        problem = None
        try:
            mlp, norm = _walk(layer, points.mlp), _walk(layer, points.pre_mlp_norm)
            for obj in (layer, mlp):
                if id(obj) in owners:
                    problem = f"shares a module with layer {owners[id(obj)]}"
                owners.setdefault(id(obj), i)
            proj = [getattr(mlp, k, None) for k in ("gate_proj", "up_proj", "down_proj")]
            if problem is None and any(not isinstance(p, torch.nn.Linear) for p in proj):
                problem = "MLP without gate_proj/up_proj/down_proj linear layers"
            if problem is None:
                gate, up, down = proj
                hid, inter = gate.in_features, gate.out_features
                shapes = [(p.in_features, p.out_features) for p in proj]
                if shapes != [(hid, inter), (hid, inter), (inter, hid)]:
                    problem = f"projection shapes {shapes} are not a gated MLP"
                elif any(p.bias is not None for p in proj):
                    problem = "projections with bias"
                elif getattr(norm, "weight", None) is None or norm.weight.numel() != hid:
                    problem = f"pre-MLP norm is not of width {hid}"
                else:
                    row.update(compatible=True, hidden=hid, intermediate=inter)
        except (AttributeError, IndexError, KeyError, TypeError) as exc:
            problem = f"missing module ({exc})"
        if problem:
            row["reason"] = problem
            report["missing"].append(f"{row['path']}: {problem}")
    report["points"] = points
    report["compatible"] = bool(report["layers"]) and not report["missing"]
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


# ------------------------------------------------------------------ module replacement
def _single_token(x) -> bool:
    """Batch-1 decode input: [1, 1, H]."""
    return x.dim() == 3 and x.shape[0] == 1 and x.shape[1] == 1


def _hidden_states(args, kwargs):
    """The decoder layer's hidden-state input: the `hidden_states` keyword,
    else the first positional argument."""
    x = kwargs.get("hidden_states", args[0] if args else None)
    if not isinstance(x, torch.Tensor):
        raise ValueError("decoder layer called without a hidden_states tensor (first argument or keyword)")
    return x


class _LayerStep:
    """One open decode step of one layer, from the decoder's pre-hook to the
    MLP's output. The order of its calls is the reference runtime's layer
    step (begin -> early update -> [Progressive: enqueue] -> final
    prediction -> finalize -> [basic: wait for the reads, enqueue] ->
    output -> commit; runtime.h, weight_manager.cpp:124-205)."""

    def __init__(self, mlp: "SparseMLP", hidden):
        self.mlp, self.rt = mlp, mlp.runtime
        self.closed = False
        self.rt.begin()
        early = mlp.owner.prediction.early
        if early is not None:
            try:
                self.deliver(early.predictor("layer_input", mlp.index, hidden, early.budget), early)
            except BaseException:
                self.cancel()
                raise

    def deliver(self, answer, stage):
        """Hands a prediction to the reads; None while a future is pending."""
        if hasattr(answer, "done"):
            if not answer.done():
                return None
            answer = answer.result()
        ids = checked_selection(answer, self.rt.n, stage.budget)
        self.rt.update(ids, stage.io_budget)
        return ids

    def run(self, x):
        rt, mlp = self.rt, self.mlp
        _require(x.is_cuda and x.dtype == torch.float16 and x.shape[-1] == rt.spec.width,
                 f"layer {mlp.index} MLP input: CUDA float16 [1, 1, {rt.spec.width}]")
        stream = torch.cuda.current_stream()
        basic = mlp.owner.mode == "basic"
        if not basic:  # the kernel is queued first and consumes groups as they are published
            rt.enqueue(x, stream)
            mlp.trace.append("pre_enqueue")
        final = mlp.owner.prediction.final
        ids = self.deliver(final.predictor("mlp_input", mlp.index, x, final.budget), final)
        _require(ids is not None, f"layer {mlp.index}: the final prediction returned an unfinished future")
        rt.finalize(ids)
        mlp.trace.append("finalize")
        if basic:
            rc = rt.wait_io(5000)
            if rc:
                raise RuntimeError(f"layer {mlp.index}: reads did not complete (rc {rc})")
            rt.enqueue(x, stream)
            mlp.trace.append("basic_enqueue_after_io")
        out = rt.output(x.shape)
        rt.commit()
        self.closed = True
        return out

    def cancel(self):
        if not self.closed:
            self.closed = True
            self.rt.abort()


class SparseMLP(torch.nn.Module):
    """Replacement MLP of one decoder layer: single-token decode runs the
    sparse B200 path over the predicted groups, any other input shape the
    original module."""

    def __init__(self, original, owner, index, runtime: LayerRuntime):
        super().__init__()
        self.original, self.owner, self.index, self.runtime = original, owner, index, runtime
        self.step: Optional[_LayerStep] = None
        self.trace = []

    @property
    def pending(self) -> bool:
        return self.step is not None and not self.step.closed

    def open(self, hidden):
        """Decoder pre-hook: opens this layer's decode step."""
        if torch.is_grad_enabled():
            raise RuntimeError("the LeanStream attachment is inference-only: use torch.inference_mode()")
        if not _single_token(hidden):
            _require(hidden.dim() == 3 and hidden.shape[0] == 1,
                     f"hidden_states {tuple(hidden.shape)}: only batch 1, [1, S, H]")
            return
        _require(hidden.is_cuda and hidden.dtype == torch.float16, "decode hidden_states must be CUDA float16")
        self.trace = []
        self.step = None
        self.step = _LayerStep(self, hidden)

    def abort(self):
        if self.step is not None:
            step, self.step = self.step, None
            step.cancel()

    def forward(self, x):
        if not _single_token(x):
            return self.original(x)
        if not self.pending:
            raise RuntimeError(f"layer {self.index}: the sparse MLP ran outside its decoder layer's step")
        try:
            return self.step.run(x)
        except BaseException:
            self.abort()
            raise
        finally:
            if self.step is not None and self.step.closed:
                self.step = None


def _check_attachment(model, report, layers, weights, cache_policy, prediction, mode):
    _require(getattr(model, "_leanstream_attachment", None) is None, "this model already has an attachment")
    _require(not model.training, "attach to a model in eval() mode")
    _require(report["compatible"], f"model not attachable: {report['missing'] or report['ambiguities']}")
    _require(len(weights) == len(layers) and len(cache_policy) == len(layers),
             f"{len(layers)} decoder layers need as many WeightSpecs and CachePolicies "
             f"({len(weights)}, {len(cache_policy)} given)")
    for row, w, p in zip(report["layers"], weights, cache_policy):
        w.validate()
        p.validate(w.group_count)
        prediction.validate(w.group_count, mode)
        _require(row["hidden"] == w.width and row["intermediate"] == w.group_count * w.group_size,
                 f"{row['path']}: model H={row['hidden']}, I={row['intermediate']}; packed weights "
                 f"H={w.width}, I={w.group_count * w.group_size}")


class Attachment:
    """Lifecycle handle of attach_leanstream: the replaced MLP modules and
    the decoder hooks that open and close their decode steps."""

    def __init__(self, model, points, weights, compute, cache_policy, prediction, mode):
        report = inspect_model(model, points)
        layers = _walk(model, report["points"].layers) if report["points"] else []
        _check_attachment(model, report, layers, weights, cache_policy, prediction, mode)
        self.model, self.prediction, self.mode = model, prediction, mode
        self.points = report["points"]
        self.entries, self.handles, self.closed = [], [], False
        try:
            for i, (layer, w, p) in enumerate(zip(layers, weights, cache_policy)):
                self._install(i, layer, LayerRuntime(w, p, compute))
            model._leanstream_attachment = self
        except BaseException:
            self.close()
            raise

    def _install(self, index, layer, runtime):
        parent_path, _, name = self.points.mlp.rpartition(".")
        parent = _walk(layer, parent_path) if parent_path else layer
        original = getattr(parent, name)
        mlp = SparseMLP(original, self, index, runtime)
        setattr(parent, name, mlp)
        self.entries.append((parent, name, original, mlp))
        self.handles.append(layer.register_forward_pre_hook(
            lambda _m, args, kwargs: mlp.open(_hidden_states(args, kwargs)), with_kwargs=True))
        # always_call: runs when the decoder layer raises too, so a step that
        # its MLP never reached (or left open) is cancelled
        self.handles.append(layer.register_forward_hook(lambda *_: mlp.abort() if mlp.pending else None,
                                                        always_call=True))

    def refine(self, layer, ids, io_budget):
        """A mid-step prediction update for `layer` (reorders its pending reads)."""
        mlp = self.entries[layer][3]
        _require(mlp.pending, f"layer {layer} has no open decode step to refine")
        n = mlp.runtime.n
        _require(0 <= io_budget <= n, f"io_budget {io_budget}: 0..{n}")
        mlp.runtime.update(checked_selection(ids, n, n), io_budget)

    def reset(self):
        for entry in self.entries:
            entry[3].abort()

    def close(self):
        if self.closed:
            return
        self.closed = True
        for handle in self.handles:
            handle.remove()
        self.handles.clear()
        while self.entries:
            parent, name, original, mlp = self.entries.pop()
            try:
                mlp.abort()
                mlp.runtime.close()
            finally:
                setattr(parent, name, original)
        if getattr(self.model, "_leanstream_attachment", None) is self:
            del self.model._leanstream_attachment

    detach = close

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def attach_leanstream(model, *, points, weights, compute, cache_policy, prediction, mode="progressive"):
    """Attaches the B200 sparse MLP to every decoder layer of `model` and
    returns the handle (close() restores the model); keep calling the
    model's own forward / generate."""
    return Attachment(model, points, weights, compute, cache_policy, prediction, mode)
