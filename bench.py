#!/usr/bin/env python3
"""Benchmark of the B200 sparse streaming-MLP path (BASELINE.json metric).

Workload: configuration 3 -- a 36-layer MLP stack at the 4096/12288
geometry (192 logical groups of 64 neurons, INT4 group-128 weights, fp16
scales), batch-1 decode. Every step (= one token) draws, per layer, a fresh
seeded active set of 20-40 % of the groups, passed to the GPU as
ExecutionQueue ready descriptors. Per layer: HF RMSNorm prologue -> sparse
SwiGLU MLP -> residual add, all inside one fused launch on one GPU.
With N GPUs (torchrun), groups are sharded round-robin (group g on rank
g mod N); each rank computes an fp32 partial output, NCCL allreduces it,
and a small epilogue adds the residual (strong scaling: the token is fixed).

Inputs are seeded synthetic data of BASELINE.json's shapes and value
distributions (signed INT4 uniform in [-7,7] -- the range of the reference
quantizer, zero-mean so that 36 residual layers stay finite in fp16 --
scales U(0.005,0.02), hidden N(0,1)).
Each token streams ~841 MB of distinct weights, far more than the 126 MB L2,
so no L2 flush is needed between steps.

Configuration 5 (--config 5): an 80-layer stack at 8192/28672 (448 groups
of 64, 20 % active: 90 groups per layer), batch 1 -- ~5.8 GB of weights per
token.

--batch 8 (one GPU): each step decodes 8 tokens of the same seeded stream
through ls_b200_batch_mlp, over the union of their active groups per layer
(~83 % of the groups at 20 % per token), each token masked to its own set;
the layers are chained (RMSNorm of each token in the batch call, residual
hidden_out the next layer's input).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 3|5] [--batch 1|8]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, I, G, NGROUPS, LAYERS = 4096, 12288, 64, 192, 36
FMIN, FMAX = 0.2, 0.4
GROUP_BYTES = G * 3 * H // 2                  # packed INT4 bytes per group
SCALE_BYTES = G * 3 * (H // 128) * 2          # fp16 scale bytes per group
ALG_BYTES_PER_GROUP = GROUP_BYTES + SCALE_BYTES  # 405,504 B (algorithmic bytes)
# DRAM bytes (read + write) per algorithmic byte of the fused kernel, from
# ncu (dram__bytes_read.sum + dram__bytes_write.sum) over the 13 launches of
# `bench.py --layers 8 --steps 2 --warmup 3 --headline-only --no-cpu-baseline`
# (8-layer stacks: 189.3 MB read + 2.0 MB written per launch against 196.5 MB
# algorithmic): weights are read once, slightly less at 8 layers because
# consecutive tokens' active sets overlap in L2.
TRAFFIC_PER_ALG_BYTE = 0.974
SEED = 3
EPS = 1e-5
WORKLOAD = "config3: 36-layer MLP stack, H4096/I12288, 192x64 groups, 20-40% active/layer, batch 1"
METRIC = "MLP-stack tokens/s (batch-1 decode, 36 layers, H4096/I12288, 20-40% active INT4 groups)"
CONFIG = 3


def set_config(config: int) -> None:
    """Geometry of BASELINE.json configuration 3 (the headline) or 5."""
    global H, I, NGROUPS, LAYERS, FMIN, FMAX, GROUP_BYTES, SCALE_BYTES, ALG_BYTES_PER_GROUP
    global TRAFFIC_PER_ALG_BYTE, WORKLOAD, METRIC, CONFIG
    CONFIG = config
    if config == 5:
        H, I, NGROUPS, LAYERS = 8192, 28672, 448, 80
        FMIN = FMAX = 0.2  # k = round(0.2 * 448) = 90 groups per layer
        # the same capture on `--config 5 --layers 4` (296.4 MB read + 29.7 MB
        # written per launch against 292.0 MB algorithmic; the writes are
        # partial rows evicted from L2)
        TRAFFIC_PER_ALG_BYTE = 1.117
        WORKLOAD = "config5: 80-layer MLP stack, H8192/I28672, 448x64 groups, 20% active/layer, batch 1"
        METRIC = "MLP-stack tokens/s (batch-1 decode, 80 layers, H8192/I28672, 20% active INT4 groups)"
    GROUP_BYTES = G * 3 * H // 2
    SCALE_BYTES = G * 3 * (H // 128) * 2
    ALG_BYTES_PER_GROUP = GROUP_BYTES + SCALE_BYTES


def active_sets(step: int):
    """Per-layer active logical groups of one token (same on every rank)."""
    out = []
    for layer in range(LAYERS):
        rng = np.random.default_rng([SEED, step, layer])
        k = int(round(rng.uniform(FMIN, FMAX) * NGROUPS))
        out.append(np.sort(rng.permutation(NGROUPS)[:k]).astype(np.int64))
    return out


BATCH = 8  # tokens per step of the batched (--batch 8) workload


def batch_union(step: int):
    """Batch step `step` decodes tokens 8*step .. 8*step + 7 of the same seeded
    stream as the batch-1 workload. Per layer: the sorted union of their
    active groups and the [token][union] mask of each token's own set."""
    from leanstream_b200.batch import union_plan

    per_token = [active_sets(BATCH * step + b) for b in range(BATCH)]
    out = []
    for layer in range(LAYERS):
        union, _, mask = union_plan([per_token[b][layer] for b in range(BATCH)])
        out.append((union, mask))
    return out


def rank_balance(first: int, last: int, world: int) -> dict:
    """Load imbalance of round-robin sharding over the timed tokens: per layer,
    the busiest rank's active groups against the mean over ranks (the active
    set is global, so one layer's time follows its busiest rank)."""
    ratios, per_rank = [], []
    for step in range(first, last):
        for ids in active_sets(step):
            counts = np.bincount(np.asarray(ids) % world, minlength=world)
            per_rank.append(counts.mean())
            ratios.append(counts.max() / max(counts.mean(), 1e-9))
    return {"mean_groups_per_rank_layer": float(np.mean(per_rank)), "busiest_over_mean": float(np.mean(ratios)),
            "worst_busiest_over_mean": float(np.max(ratios))}


def workload_config(world: int, args) -> dict:
    """The `config` object of the JSON line: the workload only (shapes,
    active sets of the timed steps, sharding), identical for the GPU arm and
    the CPU reference arm of the same arguments. How each arm times it is
    the line's `timing` key."""
    first, last = args.warmup, args.warmup + args.steps
    cfg = {"workload": WORKLOAD, "hidden": H, "intermediate": I, "layers": LAYERS, "groups": NGROUPS,
           "group_size": G, "active_fraction": [FMIN, FMAX],
           "int4_values": "signed INT4 uniform in [-7, 7] (zero-mean like the reference quantizer, "
                          "examples/ministral/pack/int4_format.py:16; BASELINE.json's [-8, 7] has mean -0.5, "
                          "which overflows fp16 through the residual stack); fp16 scales U(0.005, 0.02)"}
    if getattr(args, "batch", 1) == BATCH:
        unions = [len(u) for s in range(first, last) for (u, _) in batch_union(s)]
        cfg.update({"batch": BATCH, "mean_union_groups_per_layer": float(np.mean(unions)), "layers_chained": True,
                    "parallelism": "single GPU",
                    "l2": f"inputs larger than L2: ~{np.mean(unions) * ALG_BYTES_PER_GROUP / 1e6:.0f} MB of "
                          "distinct weights per layer"})
        return cfg
    mean_active = float(np.mean([len(ids) for s in range(first, last) for ids in active_sets(s)]))
    cfg.update({"batch": 1, "mean_active_groups_per_layer": mean_active,
                "rank_balance": rank_balance(first, last, world) if world > 1 else None,
                "parallelism": f"tp{world} (groups round-robin; fp32 partials exchanged over NVLink peer memory "
                               "inside the persistent launch)" if world > 1 else "single GPU",
                "l2": f"inputs larger than L2: ~{mean_active * LAYERS * ALG_BYTES_PER_GROUP / 1e6:.0f} MB of "
                      "distinct weights per token"})
    return cfg


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region: NVML
    polled from a thread every 2 ms (the timed region lasts milliseconds), or
    nvidia-smi at its 100 ms floor when NVML is unavailable. Read-only."""

    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.thread = None
        self.samples, self.reasons, self.smax = [], set(), None
        self.stop_flag = False

    def _nvml_loop(self, nv, handle):
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        while not self.stop_flag:
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM)))
                active = nv.nvmlDeviceGetCurrentClocksEventReasons(handle)
                self.reasons.update(name for name, bit in bits.items() if active & bit)
            except Exception:  # a failed query ends sampling, it never stops the bench
                break
            time.sleep(0.002)

    def start(self):
        try:
            import threading

            import pynvml as nv

            nv.nvmlInit()
            handle = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.smax = float(nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM))
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, handle), daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def mark(self):
        """Drops the samples taken so far: only the timed region counts."""
        self.samples = []
        self.reasons = set()

    def stop(self):
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(timeout=5)
            return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.smax,
                    "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.strip()]
        sm, smax, reasons = [], None, set()
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for name, val in zip(self.NAMES, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


# --------------------------------------------------------------------- GPU arm
def shard_weights(layer: int, rank: int, nloc: int, dev):
    """Packed INT4 groups and fp16 scales of rank `rank`'s `nloc` groups of
    one layer, drawn on the device from a seed of (layer, rank), so any rank
    can regenerate another rank's shard. Zero-mean signed nibbles, uniform in
    [-7, 7] as the reference quantizer produces
    (examples/ministral/pack/int4_format.py:16); a [-8, 7] draw has mean
    -0.5, and through the residual stack that bias feeds back into gate/up
    until fp16 overflows."""
    import torch

    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 * SEED + 17 * layer + rank)
    nib = torch.randint(-7, 8, (2, nloc * GROUP_BYTES), dtype=torch.int16, device=dev, generator=gen)
    packed = ((nib[0] & 15) | ((nib[1] & 15) << 4)).to(torch.uint8)
    del nib
    s = torch.empty(nloc * G * 3 * (H // 128), dtype=torch.float32, device=dev)
    s.uniform_(0.005, 0.02, generator=gen)
    return packed, s.half()


PARITY_LAYERS = 3  # layers of one token checked against the oracle after the timed region


def stack_parity(st, graph, token: int, world: int, rank: int):
    """Oracle check of the first PARITY_LAYERS layers of token `token`, run
    through its own graph after the timed region, on every rank:
    * the ranks' hidden states are all-gathered and must be bit-identical
      (the in-kernel exchange sums the same partials in the same order);
    * on rank 0, each layer equals the oracle: RMSNorm of the layer's input,
      every rank's sparse MLP over its own shard (regenerated from the
      shard seeds), the fp32 partials summed, one fp16 rounding and the
      residual (backends/triton/reduction.py:14-20)."""
    import torch
    import torch.distributed as dist

    from leanstream_b200.tp import local_groups, rank_descriptors

    graph.replay()
    torch.cuda.synchronize()
    xs = torch.stack([st.xs[l] for l in range(PARITY_LAYERS + 1)])
    identical = True
    if world > 1:
        gathered = [torch.empty_like(xs) for _ in range(world)]
        dist.all_gather(gathered, xs)
        identical = all(torch.equal(gathered[0], g) for g in gathered[1:])
    if rank != 0:
        return None
    from oracle import oracle as O

    x_host = xs.cpu().numpy()
    sets = active_sets(token)
    worst, bound_min, ok = 0.0, None, identical
    for l in range(PARITY_LAYERS):
        x_l = x_host[l]
        xin = O.rmsnorm(x_l, None, EPS)
        total = np.zeros(H, np.float32)
        for r in range(world):
            rows = rank_descriptors(sets[l], r, world)
            if not len(rows):
                continue
            nloc = len(local_groups(NGROUPS, r, world))
            packed, sc = (st.cache[l], st.scales[l]) if r == rank else shard_weights(l, r, nloc, st.dev)
            _, y32, _ = O.mlp(H, G, xin, packed.cpu().numpy(), sc.cpu().numpy(), rows)
            total += y32
        ref = O.residual(x_l, total.astype(np.float16)).astype(np.float32)
        got = x_host[l + 1].astype(np.float32)
        err = float(np.abs(got - ref).max())
        bound = 2e-3 * float(np.abs(ref).max()) + 1e-3
        worst = max(worst, err)
        bound_min = bound if bound_min is None else min(bound_min, bound)
        ok = ok and bool(np.isfinite(got).all()) and err <= bound
    return {"ok": ok, "token": token, "layers_checked": PARITY_LAYERS, "max_abs": worst, "bound": bound_min,
            "ranks_identical": identical,
            "rule": "per layer: max|x_{l+1} - oracle| <= 2e-3 max|oracle| + 1e-3, oracle = fp16(x_l + "
                    "fp16(sum over ranks of fp32 partials)); ranks all-gathered bit-identical"}


CONFIG2_GROUPS = 58  # round(0.3 * 192) groups, all resident and READY


def run_layer_path(st, args, stream, world):
    """The reference's per-layer call path on this backend: every layer is
    one ComputeBackend.enqueue (ls_b200_view) as LayerStep::enqueue_compute
    issues it (src/runtime/runtime.cpp:36-43), one launch per layer.

    * config 2: one H 4096 layer, 58 of 192 groups, all resident and READY
      (BatchCompat plan in device memory), no norm or residual; the launches
      cycle over the stack's 36 weight sets with a seeded 58-group set each
      (36 x 23.5 MB, far above the 126 MB L2, so every launch streams its
      weights from HBM). Reported as us per layer (GPU time of `reps` launches
      captured in one CUDA graph, and the same launches issued from the host).
    * config 3, one launch per layer: the timed tokens' 36 layers chained
      through per-layer enqueues (RMSNorm input, residual hidden_out), one
      CUDA graph per token, tokens/s.
    Both use the bound buffers of ls_b200_set_buffers for the per-layer
    weights, as the reference's TritonBackend binds its MLP buffers."""
    import torch

    from leanstream_b200 import _native as N
    from leanstream_b200.tp import local_groups, rank_descriptors

    be = st.backend
    vb = be.view()
    span = N.ExecSpan(None, 0)
    img = torch.zeros((LAYERS, st.slot_words), dtype=torch.int32, pin_memory=True)
    sets = []
    for layer in range(LAYERS):
        ids = np.sort(np.random.default_rng([SEED, 2, layer]).permutation(NGROUPS)[:CONFIG2_GROUPS])
        sets.append(ids)
        st._write_plan(img[layer], ids)
    img_dev = img.to(st.dev)
    views = [st.queue_view(img_dev[layer]) for layer in range(LAYERS)]
    x, y = st.xs[0], st.y

    def enqueue_c2(i, strm):
        layer = i % LAYERS
        be.set_buffers(cache=st.cache[layer], scales=st.scales[layer])
        rc = vb.enqueue(vb.context, layer, x.data_ptr(), y.data_ptr(), strm, span, views[layer], 1,
                        N.MODE_BATCH_COMPAT)
        if rc:
            raise RuntimeError(f"ComputeBackend.enqueue returned {rc}")

    reps = 4 * LAYERS
    with torch.cuda.stream(stream):
        for i in range(LAYERS):
            enqueue_c2(i, stream.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(reps):
            enqueue_c2(i, torch.cuda.current_stream().cuda_stream)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    with torch.cuda.stream(stream):
        g.replay()  # warm-up
        ev[0].record(stream)
        g.replay()
        ev[1].record(stream)
        ev[2].record(stream)
        for i in range(reps):
            enqueue_c2(i, stream.cuda_stream)
        ev[3].record(stream)
    torch.cuda.synchronize()
    us_graph = ev[0].elapsed_time(ev[1]) * 1e3 / reps
    us_host = ev[2].elapsed_time(ev[3]) * 1e3 / reps
    g.reset()
    local = [len(rank_descriptors(ids, st.rank, world)) for ids in sets]
    layer_bytes = float(np.mean(local)) * ALG_BYTES_PER_GROUP
    out = {"config2": {
        "metric": "us per layer (config 2: one H4096/I12288 layer, 58 of 192 groups READY, BatchCompat) through "
                  "ComputeBackend.enqueue of ls_b200_view, one launch per layer",
        "value": us_graph, "unit": "us/layer", "higher_is_better": False,
        "host_launched_us_per_layer": us_host,
        "launches": reps, "target_us_at_70pct_of_8TBs": 4.20,
        "roofline": {"bound": "hbm", "achieved": layer_bytes / (us_graph * 1e-6) / 1e9, "unit": "GB/s",
                     "bytes_per_layer_per_rank": layer_bytes},
        "l2": "launches cycle over 36 weight sets (~845 MB), each read from HBM"}}

    # config 3 through one enqueue per layer
    tok_graphs = []
    for k in range(args.steps):
        s = args.warmup + k
        gk = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gk, stream=stream):
            cs = torch.cuda.current_stream().cuda_stream
            for layer in range(LAYERS):
                be.set_buffers(cache=st.cache[layer], scales=st.scales[layer], flags=N.NORM_INPUT,
                               residual=st.xs[layer], hidden_out=st.xs[layer + 1])
                rc = vb.enqueue(vb.context, layer, st.xs[layer].data_ptr(), y.data_ptr(), cs, span,
                                st.queue_view(st.plans_dev[s][layer]), 1, N.MODE_BATCH_COMPAT)
                if rc:
                    raise RuntimeError(f"ComputeBackend.enqueue returned {rc}")
        tok_graphs.append(gk)
    with torch.cuda.stream(stream):
        tok_graphs[0].replay()
        ev[0].record(stream)
        for gk in tok_graphs:
            gk.replay()
        ev[1].record(stream)
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1])
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms, us_graph], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, out["config2"]["value"] = float(t[0].item()), float(t[1].item())
    for gk in tok_graphs:
        gk.reset()
    out["config3_per_layer_launches"] = {
        "metric": "MLP-stack tokens/s, config 3 with one ComputeBackend.enqueue (one launch) per layer",
        "value": args.steps / (ms * 1e-3), "unit": "tokens/s", "us_per_layer": ms * 1e3 / (args.steps * LAYERS),
        "launches_per_token": LAYERS}
    return out


class Stack:
    """Device state of one rank: weights of its groups for every layer, plan
    images (ExecutionQueue ready descriptors) and activation buffers."""

    def __init__(self, rank: int, world: int, steps: int):
        import torch
        from leanstream_b200 import B200Backend
        from leanstream_b200 import _native as N

        self.torch, self.N = torch, N
        self.rank, self.world = rank, world
        from leanstream_b200.tp import local_groups

        self.local = local_groups(NGROUPS, rank, world)
        self.nloc = len(self.local)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        gen = torch.Generator(device=dev)
        self.cache, self.scales = [], []
        for layer in range(LAYERS):
            packed, sc = shard_weights(layer, rank, self.nloc, dev)
            self.cache.append(packed)
            self.scales.append(sc)
        gen.manual_seed(SEED)
        self.x0 = torch.randn(H, device=dev, generator=gen).half()
        self.xs = [torch.zeros(H, dtype=torch.float16, device=dev) for _ in range(LAYERS + 1)]
        self.y = torch.zeros(H, dtype=torch.float16, device=dev)
        self.y32 = torch.zeros(H, dtype=torch.float32, device=dev)
        self.backend = B200Backend().configure(H, G, max(self.nloc, 1), max_layers=LAYERS, cache_slots=self.nloc,
                                               physical_groups=self.nloc, timeout_us=5_000_000, rms_eps=EPS)
        # plan image per (step, layer): [desc nloc*5 | idx nloc | control 32] u32, 128-B aligned parts
        self.d_words = ((self.nloc * 5 + 31) // 32) * 32
        self.i_words = ((self.nloc + 31) // 32) * 32
        self.slot_words = self.d_words + self.i_words + 32
        self.steps = steps
        self.plans_host = torch.zeros((steps, LAYERS, self.slot_words), dtype=torch.int32, pin_memory=True)
        self.active_local = []  # per step: per-layer local active count
        for st in range(steps):
            counts = []
            for layer, ids in enumerate(active_sets(st)):
                counts.append(self._write_plan(self.plans_host[st, layer], ids))
            self.active_local.append(counts)
        self.plans_dev = self.plans_host.to(dev)
        self.slot_dev = torch.zeros((LAYERS, self.slot_words), dtype=torch.int32, device=dev)

    def _write_plan(self, img, ids) -> int:
        """All-ready plan through the ExecutionQueue producer protocol."""
        import ctypes as C

        N = self.N
        from leanstream_b200.tp import rank_descriptors

        rows = rank_descriptors(ids, self.rank, self.world)
        a = img.numpy().view(np.uint32)
        base = img.data_ptr()
        view = N.DeviceExecQueue(base, base + 4 * self.d_words, base + 4 * (self.d_words + self.i_words),
                                 max(self.nloc, 1))
        q = N.Queue()
        lib = N.load()
        lib.ls_b200_queue_bind(C.byref(q), view)
        assert lib.ls_b200_queue_reset(C.byref(q), 1) == 0
        a[: rows.size] = rows.reshape(-1)  # descriptors, written before publication
        assert lib.ls_b200_queue_prepare(C.byref(q), len(rows)) == 0
        assert lib.ls_b200_queue_publish_all(C.byref(q)) == 0
        assert lib.ls_b200_queue_activate(C.byref(q)) == 0
        return len(rows)

    def queue_view(self, words):
        base = words.data_ptr()
        return self.N.DeviceExecQueue(base, base + 4 * self.d_words, base + 4 * (self.d_words + self.i_words),
                                      max(self.nloc, 1))

    def connect(self):
        """Tensor parallel: exchange the ranks' IPC handles of their exchange
        buffers (host collective, once); the data path is inside the kernel."""
        import torch.distributed as dist

        mine = self.backend.tp_setup(self.rank, self.world)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine)
        self.backend.tp_connect(handles)

    def layer_args(self, layer: int, plan_words):
        N = self.N
        return self.backend.layer_args(
            input=self.xs[layer], output=self.y, cache=self.cache[layer], scales=self.scales[layer],
            epoch=1, queue=self.queue_view(plan_words), mode=N.MODE_BATCH_COMPAT, layer=layer,
            flags=N.NORM_INPUT, residual=self.xs[layer], hidden_out=self.xs[layer + 1])

    def encode_token(self, plan_rows, base_dev):
        """Encoded plans of one token for the multi-layer launch."""
        import torch

        blobs = [self.backend.encode_plan(self.layer_args(layer, plan_rows[layer])) for layer in range(LAYERS)]
        host = torch.frombuffer(bytearray(b"".join(blobs)), dtype=torch.uint8).pin_memory()
        dev = host.to(base_dev)
        return host, dev

    def enqueue_token(self, plan_rows, stream, encoded):
        """Enqueues one token (all layers) on `stream` as one persistent
        multi-layer launch; returns launches of ours. N GPUs: every rank issues
        the same launch over its own groups, and the kernel exchanges the fp32
        partial outputs of each layer over NVLink peer memory."""
        host, dev = encoded
        self.backend.launch_plans(dev, LAYERS, host, stream=stream)
        return 1


def trace_report(st, encoded, stream, rank=0):
    """Phase stamps (LS_B200_TRACE_*, LS_B200_LTRACE_*) of one multi-layer
    launch, summarised to stderr: per layer, the median over CTAs of each
    stamp relative to the first CTA's entry. With N GPUs every rank issues
    the traced launch (it is a collective); rank 0 prints its own stamps."""
    import torch

    grid = torch.cuda.get_device_properties(0).multi_processor_count
    pieces = 128
    trace = torch.zeros(grid * 8 + grid * LAYERS * 8 + 4 * pieces * 4, dtype=torch.int64, device=st.dev)
    host, dev = encoded
    with torch.cuda.stream(stream):
        st.N.load().ls_b200_spin(1_000_000, stream.cuda_stream)
        st.backend.launch_plans(dev, LAYERS, host, trace=trace, stream=stream)
    torch.cuda.synchronize()
    if rank != 0:
        return
    t = trace.cpu().numpy().astype(np.int64)
    cta = t[: grid * 8].reshape(grid, 8)
    lay = t[grid * 8: grid * 8 + grid * LAYERS * 8].reshape(grid, LAYERS, 8)
    pcs = t[grid * 8 + grid * LAYERS * 8:].reshape(4, pieces, 4)
    t0 = cta[:, 0].min()
    rel = lambda a: np.where(a > 0, (a - t0) / 1000.0, np.nan)
    names = {0: "entry", 1: "decided", 2: "first", 3: "pieces", 4: "produced", 6: "roles_done", 7: "exit"}
    print("trace(us min/med/max): " + " ".join(
        f"{n}={np.nanmin(rel(cta[:, i])):.1f}/{np.nanmedian(rel(cta[:, i])):.1f}/{np.nanmax(rel(cta[:, i])):.1f}"
        for i, n in names.items()), file=sys.stderr)
    lnames = ["decided", "issued", "pieces_done", "partials_ready", "reduced", "next_ready", "loaded"]
    print("layer  " + " ".join(f"{n:>14s}" for n in lnames) + "   (median over CTAs / max)", file=sys.stderr)
    for l in range(min(LAYERS, 12)):
        cols = []
        for w in range(7):
            v = rel(lay[:, l, w])
            cols.append(f"{np.nanmedian(v):6.1f}/{np.nanmax(v):6.1f}" if np.isfinite(v).any() else f"{'-':>13s}")
        print(f"{l:5d}  " + " ".join(f"{c:>14s}" for c in cols), file=sys.stderr)
    wst = t[grid * 8 + grid * LAYERS * 8 + 64 * 4: grid * 8 + grid * LAYERS * 8 + 64 * 4 + 12 * 16].reshape(12, 16)
    print("CTA0 per-warp piece completion, pieces 8..19 (us after the piece's first warp; warps 0..15)",
          file=sys.stderr)
    for i in range(12):
        v = rel(wst[i])
        if np.isfinite(v).any():
            print(f"  {8 + i:3d} " + " ".join(f"{x - np.nanmin(v):5.2f}" for x in v), file=sys.stderr)
    for c in range(2):
        print(f"CTA{c} pieces: idx issued closed ready done (us)", file=sys.stderr)
        for i in range(min(pieces, 64)):
            v = rel(pcs[c, i])
            if not np.isfinite(v).any():
                break
            print(f"  {i:3d} " + " ".join(f"{x:7.2f}" for x in v), file=sys.stderr)


def run_gpu(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    steps_total = args.warmup + args.steps
    t_start = time.time()

    def progress(msg):  # phase marks on stderr (the JSON line is stdout's only content)
        print(f"[bench rank {rank}/{world} {time.time() - t_start:7.2f}s] {msg}", file=sys.stderr, flush=True)

    st = Stack(rank, world, steps_total)
    if world > 1:
        st.connect()
    progress("weights and plans resident")
    stream = torch.cuda.Stream()
    N = st.N
    lib = N.load()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- capture one CUDA graph per token (kernel params point at that token's plans)
    st.xs[0].copy_(st.x0)
    torch.cuda.synchronize()
    graphs = []
    launches_per_token = 0
    encoded = [st.encode_token(st.plans_dev[s], st.dev) for s in range(steps_total)]
    for s in range(steps_total):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launches_per_token = st.enqueue_token(st.plans_dev[s], torch.cuda.current_stream(), encoded[s])
        graphs.append(g)
    torch.cuda.synchronize()
    barrier()
    progress(f"{len(graphs)} token graphs captured")

    # ---- value: device-resident inputs, K graph replays
    with torch.cuda.stream(stream):
        for s in range(args.warmup):
            graphs[s].replay()
    barrier()
    assert st.backend.status()[N.STATUS_ERROR] == 0, st.backend.status()
    progress("warm-up done")
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    clocks.mark()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for s in range(args.warmup, steps_total):
            graphs[s].replay()
        e1.record(stream)
    torch.cuda.synchronize()
    clock = clocks.stop()
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    status = st.backend.status()
    if status[N.STATUS_ERROR]:
        raise RuntimeError(f"device status {status}")
    ms_per_step = ms / args.steps
    progress(f"timed region: {ms_per_step:.3f} ms per token")
    barrier()
    with torch.cuda.stream(stream):
        parity = stack_parity(st, graphs[args.warmup], args.warmup, world, rank)
    barrier()
    progress(f"parity of {PARITY_LAYERS} layers: {parity}")

    # ---- kernel-only durations: pre-queued, event-bracketed multi-layer
    # launches (N GPUs: each rank's launch over its own groups, including the
    # in-kernel exchange). Each is a replay of the token's graph (the launch
    # alone), so the host's enqueue cost cannot leave gaps inside a bracket
    # once the 2 ms delay has run out.
    barrier()
    reps = min(args.steps, 8)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * reps)]
    with torch.cuda.stream(stream):
        lib.ls_b200_spin(2_000_000, stream.cuda_stream)  # queue everything behind a 2 ms delay
        for i in range(reps):
            s = args.warmup + i
            ev[2 * i].record(stream)
            graphs[s].replay()
            ev[2 * i + 1].record(stream)
    torch.cuda.synchronize()
    kern_ms = [ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(reps)]
    kern_bytes = [sum(st.active_local[args.warmup + i]) * ALG_BYTES_PER_GROUP for i in range(reps)]
    kernel_name = f"fused_mlp_kernel ({LAYERS}-layer persistent launch" + (", per-rank shard)" if world > 1 else ")")
    achieved_gbs = sum(kern_bytes) / (sum(kern_ms) * 1e-3) / 1e9
    if world > 1:  # the slowest rank's HBM rate
        t = torch.tensor([-achieved_gbs], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        achieved_gbs = -float(t.item())
    progress("kernel-only timing done")
    if args.trace:
        barrier()
        trace_report(st, encoded[args.warmup], stream, rank)
    layer_path = None
    if CONFIG == 3 and not args.headline_only and not args.layers:
        barrier()
        layer_path = run_layer_path(st, args, stream, world)
        barrier()
        progress(f"per-layer enqueue path: {layer_path['config2']['value']:.2f} us per config-2 layer, "
                 f"{layer_path['config3_per_layer_launches']['value']:.0f} tokens/s with one launch per layer")

    # ---- e2e: host plans + host x in, host y out, through the C ABI each step
    barrier()
    e2e_graph = torch.cuda.CUDAGraph()
    slot_encoded = st.encode_token(st.slot_dev, st.dev)
    with torch.cuda.graph(e2e_graph, stream=stream):
        st.enqueue_token(st.slot_dev, torch.cuda.current_stream(), slot_encoded)
    x_host = st.x0.cpu().pin_memory()
    y_host = torch.zeros(H, dtype=torch.float16, pin_memory=True)
    h2d = st.plans_host[0].numel() * 4 + x_host.numel() * 2
    d2h = y_host.numel() * 2
    barrier()
    with torch.cuda.stream(stream):
        for s in range(args.warmup):
            st.slot_dev.copy_(st.plans_host[s], non_blocking=True)
            st.xs[0].copy_(x_host, non_blocking=True)
            e2e_graph.replay()
            y_host.copy_(st.xs[LAYERS], non_blocking=True)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for s in range(args.warmup, steps_total):
            st.slot_dev.copy_(st.plans_host[s], non_blocking=True)
            st.xs[0].copy_(x_host, non_blocking=True)
            e2e_graph.replay()
            y_host.copy_(st.xs[LAYERS], non_blocking=True)
        f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    progress("end-to-end timing done")
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    if not np.isfinite(y_host.numpy().astype(np.float32)).all():
        bad = [l for l in range(LAYERS + 1) if not torch.isfinite(st.xs[l].float()).all()]
        mags = [float(st.xs[l].float().abs().max()) for l in range(LAYERS + 1)]
        raise RuntimeError(f"non-finite hidden state: layers {bad[:5]}; max|x| per layer {mags[:8]}")
    if st.backend.status()[N.STATUS_ERROR]:
        raise RuntimeError(f"device status {st.backend.status()}")

    result = None
    if rank == 0:
        peaks = {}
        try:
            peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        except (OSError, ValueError):
            pass
        peak = float(peaks.get("hbm_gbs", 6650.0))
        mean_active = float(np.mean([sum(c) for c in st.active_local[args.warmup:]])) / LAYERS
        # DRAM bytes (read + write) of one launch, from the ncu capture of
        # the same kernel on an 8-layer stack, scaled by the algorithmic
        # bytes the launch processes (traffic grows with the active groups).
        traffic = TRAFFIC_PER_ALG_BYTE * float(np.mean(kern_bytes)) if TRAFFIC_PER_ALG_BYTE else None
        result = {
            "metric": METRIC,
            "value": args.steps / (ms * 1e-3),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "us_per_layer": ms_per_step * 1e3 / LAYERS,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "int4 weights x fp16 activations, fp32 accumulate",
            "data": "synthetic (seeded INT4/fp16, BASELINE.json shapes)",
            "config": workload_config(world, args),
            "timing": "CUDA graph per token, CUDA events on the launching stream, max over ranks",
            "arithmetic": "variant 1 (KernelSelector default): exact integer/fp32 sums with the fp16 scales "
                          "applied per 128-block; the reference rounds each weight to fp16 first (variant 0, "
                          "candidate 5); outputs within the 2e-3 x max|y| tolerance of the reference math",
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peak, "unit": "GB/s",
                         "frac": achieved_gbs / peak, "traffic": traffic,
                         "kernel": kernel_name, "kernel_us_mean": 1e3 * float(np.mean(kern_ms)),
                         "algorithmic_bytes_per_group": ALG_BYTES_PER_GROUP,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if peaks else "fallback",
                         "frac_of_8TBs_nominal": achieved_gbs / 8000.0,
                         "stack_frac": (mean_active * LAYERS * ALG_BYTES_PER_GROUP / (ms_per_step * 1e-3)) / 1e9 / peak},
            "e2e": {"value": args.steps / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": launches_per_token * args.steps,
            "clocks": clock,
            "parity": parity,
        }
        if layer_path:
            result.update(layer_path)
    # Release every graph before tearing down the process group: a graph that
    # still holds NCCL work keeps destroy_process_group waiting for good (the
    # capture loop's own variable referenced the last token graph).
    torch.cuda.synchronize()
    for gr in graphs:
        gr.reset()
    e2e_graph.reset()
    del graphs, e2e_graph, g
    torch.cuda.synchronize()
    progress("graphs released")
    if world > 1:
        dist.barrier()
    del st
    progress("done")
    return result


def run_batch(args, rank, world, local_rank):
    """Batch-8 union decode (--batch 8): each step runs the stack's layers for
    8 tokens through ls_b200_batch_mlp, over the union of the tokens' active
    groups with each token masked to its own set. Layers are chained: each
    call normalises its 8 hidden states (HF RMSNorm) and writes
    hidden_out = fp16(x + y), the next layer's input. One GPU."""
    import torch

    from leanstream_b200.batch import BatchMLP, union_plan

    if world > 1:
        raise SystemExit("--batch runs on one GPU")
    torch.cuda.set_device(local_rank)
    steps_total = args.warmup + args.steps
    t_start = time.time()

    def progress(msg):
        print(f"[bench batch {time.time() - t_start:7.2f}s] {msg}", file=sys.stderr, flush=True)

    st = Stack(0, 1, 1)  # the batch-1 workload's weights (all groups resident); its plans go unused
    dev = st.dev
    # per step, one image of every layer's [descriptors U x 20 B | mask 8 x U B]
    lstride = ((NGROUPS * 20 + BATCH * NGROUPS + 255) // 256) * 256
    img_host = torch.zeros((steps_total, LAYERS * lstride), dtype=torch.uint8, pin_memory=True)
    unions = np.zeros((steps_total, LAYERS), np.int64)
    for s in range(steps_total):
        a = img_host[s].numpy()
        for layer, (union, mask) in enumerate(batch_union(s)):
            rows = union_plan([union])[1].reshape(-1).view(np.uint8)  # all groups resident: slot = id
            off = layer * lstride
            a[off:off + rows.size] = rows
            a[off + NGROUPS * 20:off + NGROUPS * 20 + mask.size] = mask.reshape(-1)
            unions[s, layer] = len(union)
    img_dev = img_host.to(dev)
    slot_dev = torch.zeros(LAYERS * lstride, dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED)
    x = torch.randn(BATCH, H, device=dev, generator=gen).half()
    y = torch.zeros(BATCH, H, dtype=torch.float16, device=dev)
    # chained stack: layer l reads xs[l], RMSNorm in the batch call, and
    # writes xs[l+1] = fp16(xs[l] + y)
    xs = [x] + [torch.zeros(BATCH, H, dtype=torch.float16, device=dev) for _ in range(LAYERS)]
    mlp = BatchMLP(H, G, NGROUPS, device=dev)  # the public batch API; scratch sized for every group
    mma_sync = args.batch_kernels == "mma_sync"
    progress("weights and batch plans resident")
    stream = torch.cuda.Stream()

    def enqueue_step(s, base, strm):
        for layer in range(LAYERS):
            off = base + layer * lstride
            mlp.run(stream=strm, x=xs[layer], output=y, cache=st.cache[layer], scales=st.scales[layer],
                    union_descs=off, union_count=int(unions[s, layer]), tokens=BATCH, mask=off + NGROUPS * 20,
                    residual=xs[layer], hidden_out=xs[layer + 1], norm_input=True, rms_eps=EPS,
                    mma_sync=mma_sync)

    # first calls outside capture (the call opts the kernels into their ring size)
    with torch.cuda.stream(stream):
        enqueue_step(0, img_dev[0].data_ptr(), stream)
    torch.cuda.synchronize()
    graphs, e2e_graphs = [], []
    for s in range(steps_total):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            enqueue_step(s, img_dev[s].data_ptr(), torch.cuda.current_stream())
        graphs.append(g)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            enqueue_step(s, slot_dev.data_ptr(), torch.cuda.current_stream())
        e2e_graphs.append(g)
    torch.cuda.synchronize()
    progress(f"{2 * steps_total} step graphs captured")

    # ---- value: device-resident inputs and plans
    with torch.cuda.stream(stream):
        for s in range(args.warmup):
            graphs[s].replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    clocks.mark()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for s in range(args.warmup, steps_total):
            graphs[s].replay()
        e1.record(stream)
    torch.cuda.synchronize()
    clock = clocks.stop()
    ms = e0.elapsed_time(e1)
    progress(f"timed region: {ms / args.steps:.3f} ms per step")

    # ---- e2e: the step's plans and hidden states from pinned host memory,
    # outputs back to the host, every step
    x_host = x.cpu().pin_memory()
    y_host = torch.zeros(BATCH, H, dtype=torch.float16, pin_memory=True)
    h2d = img_host[0].numel() + x_host.numel() * 2
    d2h = y_host.numel() * 2

    def e2e_step(s):
        slot_dev.copy_(img_host[s], non_blocking=True)
        x.copy_(x_host, non_blocking=True)
        e2e_graphs[s].replay()
        y_host.copy_(xs[LAYERS], non_blocking=True)

    with torch.cuda.stream(stream):
        for s in range(args.warmup):
            e2e_step(s)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for s in range(args.warmup, steps_total):
            e2e_step(s)
        f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    if not np.isfinite(y_host.numpy().astype(np.float32)).all():
        raise RuntimeError("non-finite batch output")
    progress("end-to-end timing done")

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    timed = unions[args.warmup:]
    alg_bytes = float(timed.sum()) * ALG_BYTES_PER_GROUP
    achieved = alg_bytes / (ms * 1e-3) / 1e9
    result = {
        "metric": METRIC,
        "value": BATCH * args.steps / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "us_per_layer": ms / args.steps * 1e3 / LAYERS,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int4 weights x fp16 activations, fp32 accumulate",
        "data": "synthetic (seeded INT4/fp16, BASELINE.json shapes)",
        "config": workload_config(1, args),
        "timing": "CUDA graph per step, CUDA events on the launching stream",
        "arithmetic": "w = fp16(q * s) as the reference (backends/triton/core.py:17), fp32 accumulation",
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None,
                     "kernel": ("batch_norm_kernel + batch_gateup_kernel + batch_down_kernel" if mma_sync else
                                "batch_ximg_kernel + batch_gateup_tc_kernel + batch_down_tc_kernel") +
                               " + batch_epilogue_kernel (one layer)",
                     "algorithmic_bytes_per_group": ALG_BYTES_PER_GROUP,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if peaks else "fallback"},
        "e2e": {"value": BATCH * args.steps / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        # per layer: RMSNorm + gate/up + down + epilogue (warp MMA), or x image
        # (with the RMSNorm) + gate/up (with h) + down + epilogue (tcgen05)
        "gpu_launches": 4 * LAYERS * args.steps,
        "batch_kernels": args.batch_kernels,
        "clocks": clock,
    }
    if mlp.error():
        raise RuntimeError("a tensor-core batch kernel gave up a bounded wait")
    torch.cuda.synchronize()
    for g in graphs + e2e_graphs:
        g.reset()
    progress("done")
    return result


# --------------------------------------------------------------------- CPU arm
def host_cores() -> int:
    """Threads the CPU path may use: the process's CPU affinity set (as the
    reference's ls_available_cores, predictor/predictor_cpu.cpp:128). Under
    torchrun OMP_NUM_THREADS is 1, so the OpenMP default is not used."""
    return len(os.sched_getaffinity(0))


class CpuPath:
    """The reference's CPU path for one layer of the workload, on the host
    cores: group selection by the reference's own ls_predict
    (predictor/predictor_cpu.cpp:144-204, compiled unmodified into
    oracle/_ref) followed by the sparse INT4 MLP of the oracle port
    (OpenMP over active neurons; examples/custom_pytorch/run.py:43-50
    arithmetic). The reference has no native CPU MLP kernel, so the MLP leg
    is the port. Weight values do not change the arithmetic cost: one
    seeded layer stands for every layer."""

    def __init__(self, threads: int):
        from oracle import oracle as O
        from leanstream_b200.synthetic import make_layer

        self.O, self.threads = O, threads
        self.layer = make_layer(1000, H, NGROUPS, G)
        self.pred = None
        self.pred_weights = None
        try:
            rng = np.random.default_rng(SEED)
            # one representative fp32 gate/up row pair per group
            self.pred_weights = rng.standard_normal((NGROUPS, 2, H)).astype(np.float32)
            self.pred_x = self.layer.x.astype(np.float32)
        except Exception:  # pragma: no cover
            self.pred_weights = None

    def _predict(self, k: int):
        """Top-k group IDs by ls_predict. One context ranks the most groups a
        layer can have active (ls_create is set-up, not per-layer work); a
        layer with fewer takes the prefix of that (score desc, id asc)
        ranking, which is its own top-k."""
        if self.pred_weights is None:
            return None
        if self.pred is None:
            kmax = max(int(round(FMAX * NGROUPS)), 4)
            self.pred = self.O.Predictor(NGROUPS, H, kmax, threads=self.threads)
        return self.pred.predict(self.pred_weights, self.pred_x)[:k]

    def layer_seconds(self, ids) -> float:
        """Wall time of one layer: ls_predict (k = the layer's active count)
        then the sparse MLP over those groups."""
        t0 = time.perf_counter()
        sel = self._predict(len(ids))
        d = np.zeros((len(ids), 5), np.uint32)
        d[:, 0] = d[:, 1] = d[:, 2] = np.asarray(ids if sel is None else np.sort(sel))
        d[:, 3] = np.arange(len(ids))
        self.O.mlp_omp(H, G, self.layer.x, self.layer.packed, self.layer.scales, d, threads=self.threads)
        return time.perf_counter() - t0

    def predictor_available(self) -> bool:
        try:
            self._predict(4)
            return True
        except Exception:
            self.pred_weights = None
            return False


def cpu_layers_per_step() -> int:
    """Layers in one timed step of the CPU path: a whole token for
    configuration 3 (about a second on 16 host cores); for configuration 5
    (about ten seconds per token) an 8-layer sample, so that a driver run
    of tens of steps ends within minutes."""
    return LAYERS if CONFIG == 3 else min(8, LAYERS)


def cpu_stack_rate(budget_s: float = 12.0, threads: int = 0):
    """cpu_baseline of the GPU arm: the CPU path on a bounded sample of the
    same workload (the layers of tokens 0, 1, ... in order, until `budget_s`
    of CPU work or 64 tokens)."""
    nthreads = threads or host_cores()
    path = CpuPath(nthreads)
    pred = path.predictor_available()
    done, elapsed, tokens = 0, 0.0, 0
    while elapsed < budget_s and tokens < 64:
        sets = active_sets(tokens)
        for layer in range(LAYERS):
            elapsed += path.layer_seconds(sets[layer])
            done += 1
            if elapsed >= budget_s:
                break
        tokens += 1
    per_layer = elapsed / done
    what = "ls_predict + sparse MLP port" if pred else "sparse MLP port (reference predictor library absent)"
    return {"value": 1.0 / (per_layer * LAYERS), "unit": "tokens/s", "cores": int(nthreads), "kind": "port",
            "sample": f"{done} layers of tokens 0-{tokens - 1} ({what}; same shapes and active sets), "
                      f"{elapsed:.1f} s of CPU work; tokens/s = 1/({LAYERS} x mean layer time)"}


def reference_cuda_backend() -> dict:
    """The reference's own CUDA backend (kernels/streaming_mlp.cu, compiled
    unmodified into oracle/_ref/ref_streaming_timer by `make -C oracle
    ref-cuda`) timed on this box's GPU at BASELINE.json configurations 1 and
    2: seeded inputs, an all-ready BatchCompat plan (the reference's
    static-stripe path), CUDA events over back-to-back layers; the best of
    several persistent-consumer worker counts. A GPU reference point beside
    the CPU arm, not this arm's value."""
    exe = ROOT / "oracle" / "_ref" / "ref_streaming_timer"
    if not exe.exists():
        return {"unavailable": "oracle/_ref/ref_streaming_timer not built (make -C oracle ref-cuda)"}
    out = {}
    for name, cfg in (("config1", ["1024", "64", "64", "16", "50"]), ("config2", ["4096", "64", "192", "58", "20"])):
        try:
            proc = subprocess.run([str(exe), *cfg, "16", "32", "64", "148"], capture_output=True, text=True,
                                  timeout=120)
            rows = [json.loads(l) for l in proc.stdout.splitlines() if l.startswith("{")]
        except (subprocess.SubprocessError, ValueError) as exc:
            out[name] = {"unavailable": str(exc)}
            continue
        if proc.returncode or not rows:
            out[name] = {"unavailable": f"exit {proc.returncode}: {proc.stderr.strip()[-200:]}"}
            continue
        best = min(rows, key=lambda r: r["us_per_layer"])
        out[name] = {"us_per_layer": best["us_per_layer"], "workers": best["workers"], "gb_per_s": best["gb_per_s"],
                     "sweep": {r["workers"]: r["us_per_layer"] for r in rows}}
    out["source"] = ("kernels/streaming_mlp.cu:85-93 enqueue_streaming_mlp (core kernel -> consumer -> reduction), "
                     "compiled unmodified for sm_100a; timing driver tests/native/ref_streaming_timer.cu")
    return out


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path of this workload on the
    host cores (CpuPath: its own ls_predict, then the MLP port, since the
    reference has no native CPU MLP), on rank 0 only. Each timed step runs
    cpu_layers_per_step() consecutive layers of the token stream, so
    ms_per_step is the wall time of exactly what one step did; tokens/s is
    1 / (layers x mean layer time)."""
    if rank != 0:
        return None
    threads = host_cores()
    path = CpuPath(threads)
    pred = path.predictor_available()
    lps = cpu_layers_per_step()

    def one(step):
        tok, first = divmod(step * lps, LAYERS)
        sets = active_sets(tok)
        return sum(path.layer_seconds(sets[(first + j) % LAYERS]) for j in range(lps))

    for s in range(args.warmup):
        one(s)
    t = [one(args.warmup + s) for s in range(args.steps)]
    per_step = float(np.mean(t))
    per_layer = per_step / lps
    value = 1.0 / (per_layer * LAYERS)
    what = "ls_predict + sparse MLP port" if pred else "sparse MLP port (reference predictor library absent)"
    sample = (f"each step = {lps} consecutive layers of the token stream ({what}), {threads} host threads; "
              f"tokens/s = 1/({LAYERS} x mean layer time)")
    ref_gpu = reference_cuda_backend()
    return {
        "reference_cuda_backend": ref_gpu,
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "us_per_layer": per_layer * 1e6,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4 weights x fp16 activations, fp32 accumulate",
        "data": "synthetic (seeded INT4/fp16, BASELINE.json shapes)",
        "config": workload_config(world, args),
        "timing": "host wall clock (time.perf_counter) around each step",
        "arithmetic": "the reference's rounding boundaries (w, g, u, SiLU, h in fp16; fp32 sums)",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--trace", action="store_true", help="print per-CTA phase stamps of one launch to stderr")
    p.add_argument("--config", type=int, choices=[3, 5], default=3,
                   help="BASELINE.json configuration: 3 (headline, H 4096, 36 layers) or 5 (H 8192, 80 layers)")
    p.add_argument("--batch", type=int, choices=[1, 8], default=1,
                   help="tokens per step: 1 (the default workload) or 8 (union decode, one GPU)")
    p.add_argument("--batch-kernels", choices=["tcgen05", "mma_sync"], default="tcgen05",
                   help="--batch 8 projections: tcgen05 MMAs (default) or the warp-level MMA kernels")
    p.add_argument("--headline-only", action="store_true",
                   help="skip the extra measurements printed beside the headline (per-layer enqueue path, config 5)")
    p.add_argument("--layers", type=int, default=0,
                   help="stack depth; smaller values only for profiling captures (the metric is quoted at the "
                        "configuration's depth)")
    args = p.parse_args()
    global LAYERS, METRIC, WORKLOAD
    set_config(args.config)
    if args.batch == BATCH:
        METRIC = METRIC.replace("batch-1 decode", f"batch-{BATCH} union decode")
        WORKLOAD = WORKLOAD.replace("batch 1", f"batch {BATCH} over the union of the tokens' active groups")
    if args.layers:
        if not 1 <= args.layers <= LAYERS:
            p.error(f"--layers must be in [1, {LAYERS}]")
        LAYERS = args.layers
    if args.warmup < 3:
        p.error("--warmup must be at least 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    import torch

    if world > 1:
        from datetime import timedelta

        import torch.distributed as dist

        # NCCL carries only host-side setup, the parity gather and the timing
        # reductions; a rank that dies while bound to an NVLink multicast
        # object can fault the other GPUs, so NVLS stays off.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    res = run_batch(args, rank, world, local_rank) if args.batch == BATCH else run_gpu(args, rank, world, local_rank)
    if rank == 0 and res is not None and world == 1 and not args.no_cpu_baseline:
        try:
            res["cpu_baseline"] = cpu_stack_rate()
        except Exception as exc:  # the oracle library is test infrastructure; report why it is absent
            res["cpu_baseline"] = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "port",
                                   "sample": f"unavailable: {exc}"}
    if CONFIG == 3 and args.batch == 1 and not args.headline_only and not args.layers:
        res5 = run_config5(args, rank, world, local_rank)
        if rank == 0 and res is not None:
            res.update(res5)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def _summary(r: dict) -> dict:
    keep = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "us_per_layer", "roofline",
            "e2e", "parity", "gpu_launches", "config", "clocks")
    return {k: r[k] for k in keep if k in r}


def run_config5(args, rank, world, local_rank) -> dict:
    """BASELINE.json configuration 5 beside the headline, in the same run:
    batch 1 at N GPUs (the tensor-parallel launch at N > 1) and, on one GPU,
    batch 8 over the union of the tokens' active groups. Fewer steps than
    the headline (each step is an 80-layer token of ~5.8 GB of weights)."""
    import argparse as _ap

    set_config(5)
    a = _ap.Namespace(**vars(args))
    a.steps, a.warmup, a.trace, a.batch = min(args.steps, 10), 3, False, 1
    out = {}
    r = run_gpu(a, rank, world, local_rank)
    if rank == 0:
        out["config5_batch1"] = _summary(r)
    if world == 1:
        global METRIC, WORKLOAD
        metric, workload = METRIC, WORKLOAD
        METRIC = METRIC.replace("batch-1 decode", f"batch-{BATCH} union decode")
        WORKLOAD = WORKLOAD.replace("batch 1", f"batch {BATCH} over the union of the tokens' active groups")
        a.batch = BATCH
        out["config5_batch8"] = _summary(run_batch(a, rank, world, local_rank))
        METRIC, WORKLOAD = metric, workload
    return out


if __name__ == "__main__":
    main()
