"""PyTorch attachment on the B200 backend (leanstream_b200/torch_attach.py), the
interface of leanstream/integrations/torch: contracts and model inspection on
CPU; on the GPU, a small decoder-shaped model whose dense MLP weights are the
exact dequantisation of packed INT4 groups. During batch-1 decode the
replacement SparseMLP must equal the oracle's sparse MLP over the final
groups (Progressive: launch before the final prediction; basic: after the
reads), prefill shapes must run the original module, and close() must
restore the model."""
import numpy as np
import pytest
import torch

H, G, NG = 1024, 64, 16


def _layer(seed):
    from leanstream_b200.synthetic import make_layer

    return make_layer(seed, H, NG, G)


class _MLP(torch.nn.Module):
    def __init__(self, L):
        from leanstream_b200.synthetic import dequantize

        super().__init__()
        I = NG * G
        self.gate_proj = torch.nn.Linear(H, I, bias=False)
        self.up_proj = torch.nn.Linear(H, I, bias=False)
        self.down_proj = torch.nn.Linear(I, H, bias=False)
        w = dequantize(L.q, L.scales).reshape(NG * G, 3, H)  # [neuron, gate/up/down, H]
        with torch.no_grad():
            self.gate_proj.weight.copy_(torch.from_numpy(w[:, 0, :]))
            self.up_proj.weight.copy_(torch.from_numpy(w[:, 1, :]))
            self.down_proj.weight.copy_(torch.from_numpy(np.ascontiguousarray(w[:, 2, :].T)))

    def forward(self, x):
        return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


class _Norm(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(H))

    def forward(self, x):
        v = x.float()
        return (v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-5)).to(x.dtype) * self.weight.to(x.dtype)


class _Decoder(torch.nn.Module):
    def __init__(self, L):
        super().__init__()
        self.self_attn = torch.nn.Identity()
        self.post_attention_layernorm = _Norm()
        self.mlp = _MLP(L)
        self.seen = None

    def forward(self, hidden_states):
        n = self.post_attention_layernorm(hidden_states)
        m = self.mlp(n)
        self.seen = (n, m)
        return hidden_states + m


class _Model(torch.nn.Module):
    def __init__(self, layers):
        super().__init__()
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList([_Decoder(L) for L in layers])

    def forward(self, x):
        for layer in self.model.layers:
            x = layer(x)
        return x


def _spec(tmp_path, L, idx):
    from leanstream_b200 import torch_attach as T

    gb = L.group_bytes
    path = tmp_path / f"layer{idx}.bin"
    L.packed.tofile(path)
    layout = tuple(T.GroupLayout(g, g, g * gb, gb) for g in range(NG))
    return T.WeightSpec(path, H, layout, torch.from_numpy(L.scales.copy()), group_size=G)


def test_contracts_and_inspection_on_cpu(tmp_path):
    from leanstream_b200 import torch_attach as T

    L = _layer(1)
    spec = _spec(tmp_path, L, 0)
    spec.validate()
    with pytest.raises(ValueError):
        T.WeightSpec(spec.path, H, spec.layout[:-1] + (T.GroupLayout(NG - 1, NG - 1, 1, spec.group_bytes),),
                     spec.scales, group_size=G).validate()  # overlapping extents
    with pytest.raises(ValueError):
        T.CachePolicy(resident=(0, 1), core=(2,)).validate(NG)  # core outside the resident set
    T.CachePolicy(resident=(0, 1, 2), core=(1,)).validate(NG)
    stage = T.PredictionStage(lambda *a: [0], 4, 4)
    with pytest.raises(ValueError):
        T.PredictionSchedule(final=stage).validate(NG, "progressive")  # progressive needs an early stage
    T.PredictionSchedule(final=stage, early=stage).validate(NG, "progressive")
    report = T.inspect_model(_Model([L, L]))
    assert report["compatible"] and report["points"].layers == "model.layers"
    assert [r["hidden"] for r in report["layers"]] == [H, H] and report["layers"][0]["intermediate"] == NG * G
    with pytest.raises(ValueError):
        T.checked_selection([3, 3], NG, 4)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["progressive", "basic"])
def test_attached_decode_matches_oracle(native_lib, cuda_device, tmp_path, mode):
    from leanstream_b200 import torch_attach as T
    from leanstream_b200.synthetic import descriptors
    from oracle import oracle as O

    layers = [_layer(30 + i) for i in range(2)]
    model = _Model(layers).half().cuda().eval()
    final_sets = [[0, 1, 5, 9, 12, 3], [0, 2, 7, 11, 14, 15]]  # core group 0 first; 1, 2 resident
    early_sets = [[5, 9, 13], [7, 4, 11]]

    def early(source, index, x, budget):
        return early_sets[index]

    def final(source, index, x, budget):
        return final_sets[index]

    sched = T.PredictionSchedule(final=T.PredictionStage(final, 8, 8),
                                 early=T.PredictionStage(early, 8, 8) if mode == "progressive" else None)
    specs = [_spec(tmp_path, L, i) for i, L in enumerate(layers)]
    policies = [T.CachePolicy(resident=(0, 1, 2), core=(0,)) for _ in layers]
    att = T.attach_leanstream(model, points=T.ModelPoints(), weights=specs, compute=T.ComputeSpec(check_execution=True),
                              cache_policy=policies, prediction=sched, mode=mode)
    try:
        assert isinstance(model.model.layers[0].mlp, T.SparseMLP)
        with torch.inference_mode():
            for step in range(3):
                x = (torch.randn(1, 1, H, generator=torch.Generator().manual_seed(step)) * 0.5).half().cuda()
                model(x)
                for i, layer in enumerate(model.model.layers):
                    n, m = layer.seen
                    xin = n.reshape(-1).cpu().numpy()
                    y_ref, _, _ = O.mlp(H, G, xin, layers[i].packed, layers[i].scales,
                                        descriptors(np.array(final_sets[i])))
                    got = m.reshape(-1).float().cpu().numpy()
                    ref = y_ref.astype(np.float32)
                    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max(), (step, i)
                    execs = layer.mlp.runtime.execs.cpu().numpy()
                    assert execs.sum() == len(final_sets[i]) and np.all(execs[:len(final_sets[i])] == 1)
            # prefill shape: the original module runs
            xp = torch.randn(1, 4, H, generator=torch.Generator().manual_seed(9)).half().cuda()
            layer = model.model.layers[0]
            out = layer(xp)
            n, m = layer.seen
            dense = layer.mlp.original(n)
            assert torch.equal(m, dense)
    finally:
        att.close()
    assert isinstance(model.model.layers[0].mlp, _MLP) and not hasattr(model, "_leanstream_attachment")


def test_layer_runtime_protocol_on_cpu():
    """The layer step of LayerRuntime against fakes of the queue, IO backend
    and kernel backend (weight_manager.cpp:135-205): update passes only
    non-resident EMPTY groups within the IO budget; finalize writes cached
    rows (kind 0, cache slot) and streamed rows (kind 1, slot = id) with dest
    = core count + position, appends cached and already-READY rows
    unpublished, then activates and consumes the non-resident final reads;
    a landing publishes its row only after finalize and only once."""
    from leanstream_b200 import _native as N
    from leanstream_b200 import torch_attach as T

    calls = []

    class FakeQueue:
        def reset(self, e): calls.append(("reset", e))
        def write_descriptors(self, rows): calls.append(("rows", np.array(rows).tolist()))
        def prepare(self, n): calls.append(("prepare", n))
        def append_unpublished(self, i): calls.append(("append", i))
        def activate(self): calls.append(("activate",))
        def publish(self, i): calls.append(("publish", i))
        def fail(self, e): calls.append(("fail", e))

    class FakeIO:
        def __init__(self):
            self.cb = None
        def begin(self, cb, epoch): self.cb = cb; return 0
        def update(self, ids): calls.append(("update", list(ids))); return 0
        def consume(self, ids): calls.append(("consume", list(ids))); return 0
        def retire(self): return 0
        def wait(self, ms): return 0

    class FakeEngine:
        io_states = np.zeros(9, np.uint32)

    rt = T.LayerRuntime.__new__(T.LayerRuntime)
    rt.n = 8
    rt.policy = T.CachePolicy(resident=(0, 1, 2), core=(0,))
    rt.cache_slot = np.array([0, 1, 2, -1, -1, -1, -1, -1])
    rt.physical = np.arange(8, dtype=np.uint32)[::-1].copy()
    rt.queue, rt.io, rt.engine = FakeQueue(), FakeIO(), FakeEngine()
    rt.execs = None
    rt.lock = T.threading.Lock()
    rt.epoch, rt.active, rt.finalized = 0, False, False
    rt.final_index, rt.published = {}, set()

    rt.begin()
    assert calls[0] == ("reset", 1) and rt.active
    rt.engine.io_states[5] = N.IO_READY
    rt.update([1, 3, 5, 6, 7], io_budget=2)  # 1 resident, 5 already READY
    assert calls[-1] == ("update", [3, 6])
    rt._landed(1, 6, 6, 0, 1)  # before finalize: ignored (picked up at finalize)
    assert not any(c[0] == "publish" for c in calls)
    rt.engine.io_states[6] = N.IO_READY
    calls.clear()
    rt.finalize([0, 2, 5, 6, 3])
    rows = next(c[1] for c in calls if c[0] == "rows")
    # [logical, physical, slot, dest, kind]; core group 0 is not in the queue
    assert rows == [[2, 5, 2, 1, 0], [5, 2, 5, 2, 1], [6, 1, 6, 3, 1], [3, 4, 3, 4, 1]]
    assert [c for c in calls if c[0] in ("prepare", "append", "activate", "consume")] == [
        ("prepare", 4), ("append", 0), ("append", 1), ("append", 2), ("activate",), ("consume", [5, 6, 3])]
    rt._landed(1, 3, 3, 0, 2)
    rt._landed(1, 3, 3, 0, 3)  # a repeated completion publishes nothing more
    rt._landed(0, 7, 7, 0, 4)  # a stale epoch is ignored
    assert [c for c in calls if c[0] == "publish"] == [("publish", 3)]
    with pytest.raises(ValueError):
        rt.finalize([2, 5])  # the core group must be in the final set
