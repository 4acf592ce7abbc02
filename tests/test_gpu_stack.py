"""GPU parity of the fused layer epilogue/prologue used by the stack:
x_in = RMSNorm_HF(x_l), y = MLP(x_in), x_{l+1} = fp16(x_l + y)
(examples/ministral/native/predictor_shared_input.cu:16-33;
backends/triton/reduction.py:17-20), chained over several layers."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3


def test_norm_residual_single_layer(native_lib, cuda_device):
    import torch
    from gpu_harness import LayerBuffers, make_backend, run_layer, wait_stream
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    H, G, n = 1024, 64, 32
    L = make_layer(21, H, n, G)
    x = (L.x.astype(np.float32) * 7).astype(np.float16)  # un-normalised input
    rows = descriptors(np.arange(0, n, 3))
    buf = LayerBuffers(H, G, n, L.packed, L.scales, x)
    hidden = torch.zeros(H, dtype=torch.float16, device="cuda")
    be = make_backend(H, G, n, rms_eps=1e-5)
    run_layer(be, buf, [], rows, flags=N.NORM_INPUT, residual=buf.x, hidden_out=hidden)
    wait_stream()
    assert be.status()[N.STATUS_ERROR] == 0
    xin = O.rmsnorm(x, None, 1e-5)
    y_ref, _, _ = O.mlp(H, G, xin, L.packed, L.scales, rows)
    y = buf.y.cpu().numpy().astype(np.float32)
    assert np.abs(y - y_ref.astype(np.float32)).max() <= TOL * np.abs(y_ref.astype(np.float32)).max()
    h_ref = O.residual(x, buf.y.cpu().numpy())  # same y -> exact residual arithmetic
    assert np.array_equal(hidden.cpu().numpy().view(np.uint16), h_ref.view(np.uint16))
    be.close()


@pytest.mark.parametrize("H", [1024, 4096, 8192])
def test_stack_chain(native_lib, cuda_device, H):
    import torch
    from gpu_harness import to_dev, wait_stream
    from leanstream_b200 import B200Backend, ExecutionQueue
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    G, n, layers = 64, 48, 4
    Ls = [make_layer(100 + l, H, n, G) for l in range(layers)]
    sets = [np.sort(np.random.default_rng(l).permutation(n)[: 10 + 3 * l]) for l in range(layers)]
    be = B200Backend().configure(H, G, n, max_layers=layers, rms_eps=1e-5)
    xs = [to_dev(Ls[0].x.view(np.int16), torch.float16)] + [torch.zeros(H, dtype=torch.float16, device="cuda")
                                                            for _ in range(layers)]
    y = torch.zeros(H, dtype=torch.float16, device="cuda")
    keep = []
    for l in range(layers):
        q = ExecutionQueue(n)
        q.reset(l + 1)
        q.write_descriptors(descriptors(sets[l]))
        q.prepare(len(sets[l]))
        q.publish_all()
        q.activate()
        cache = to_dev(Ls[l].packed)
        scales = to_dev(Ls[l].scales.reshape(-1).view(np.int16), torch.float16)
        keep += [q, cache, scales]
        args = be.layer_args(input=xs[l], output=y, cache=cache, scales=scales, epoch=l + 1, queue=q.view,
                             mode=N.MODE_BATCH_COMPAT, layer=l, flags=N.NORM_INPUT, residual=xs[l],
                             hidden_out=xs[l + 1])
        be.launch(args)
    wait_stream()
    assert be.status()[N.STATUS_ERROR] == 0, be.status()
    for l in range(layers):
        assert be.completed_epoch(l) == l + 1
    # oracle chain, fed with the GPU's own x_l each layer (per-layer parity)
    for l in range(layers):
        x_l = xs[l].cpu().numpy()
        assert np.isfinite(x_l.astype(np.float32)).all()
        xin = O.rmsnorm(x_l, None, 1e-5)
        y_ref, _, _ = O.mlp(H, G, xin, Ls[l].packed, Ls[l].scales, descriptors(sets[l]))
        nxt = O.residual(x_l, y_ref)
        got = xs[l + 1].cpu().numpy().astype(np.float32)
        ref = nxt.astype(np.float32)
        assert np.abs(got - ref).max() <= TOL * np.abs(ref).max() + 1e-3, (l, np.abs(got - ref).max())
    be.close()


def test_multilayer_launch_matches_per_layer(native_lib, cuda_device):
    """One persistent launch over L layers (ls_b200_launch_plans) must equal,
    bit for bit, L chained single-layer launches (same canonical arithmetic)."""
    import torch
    from gpu_harness import to_dev, wait_stream
    from leanstream_b200 import B200Backend, ExecutionQueue
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors, make_layer

    H, G, n, layers = 4096, 64, 40, 5
    Ls = [make_layer(300 + l, H, n, G) for l in range(layers)]
    sets = [np.sort(np.random.default_rng(50 + l).permutation(n)[: 8 + 4 * l]) for l in range(layers)]
    be = B200Backend().configure(H, G, n, max_layers=layers, rms_eps=1e-5)
    x0 = to_dev(Ls[0].x.view(np.int16), torch.float16)
    keep, queues = [], []
    for l in range(layers):
        q = ExecutionQueue(n)
        q.reset(l + 1)
        q.write_descriptors(descriptors(sets[l]))
        q.prepare(len(sets[l]))
        q.publish_all()
        q.activate()
        queues.append(q)
        keep += [to_dev(Ls[l].packed), to_dev(Ls[l].scales.reshape(-1).view(np.int16), torch.float16)]

    def run(multi):
        xs = [x0.clone()] + [torch.zeros(H, dtype=torch.float16, device="cuda") for _ in range(layers)]
        y = torch.zeros(H, dtype=torch.float16, device="cuda")
        args = [be.layer_args(input=xs[l], output=y, cache=keep[2 * l], scales=keep[2 * l + 1], epoch=l + 1,
                              queue=queues[l].view, mode=N.MODE_BATCH_COMPAT, layer=l, flags=N.NORM_INPUT,
                              residual=xs[l], hidden_out=xs[l + 1]) for l in range(layers)]
        if multi:
            host = torch.frombuffer(bytearray(b"".join(be.encode_plan(a) for a in args)), dtype=torch.uint8)
            dev = host.cuda()
            be.launch_plans(dev, layers, host.numpy().ctypes.data)
        else:
            for a in args:
                be.launch(a)
        wait_stream()
        assert be.status()[N.STATUS_ERROR] == 0, be.status()
        return [x.cpu().numpy().view(np.uint16).copy() for x in xs]

    single = run(False)
    multi = run(True)
    for l in range(1, layers + 1):
        assert np.array_equal(single[l], multi[l]), l
        assert np.isfinite(single[l].view(np.float16).astype(np.float32)).all()
    for l in range(layers):
        assert be.completed_epoch(l) == l + 1
    be.close()
