"""GPU importance output (ls_b200_layer_args.importance / importance_flag):
per executed destination, the sum over its group's G neurons of |h|, the
cache-retention signal of examples/ministral/native/leanstream_mapped.cu:43-47,
published with the layer's epoch (leanstream_mapped.cu:36-39).

The kernel sums |h| * 2^24 exactly in 64-bit integers (every fp16 value is
a multiple of 2^-24) and rounds once to fp32, so each entry must equal, bit
for bit, the fp32 rounding of the exact (fp64) sum of the layer's own
activation output |h|. Destinations the layer did not execute are 0, the
flag holds the epoch, and a second launch finds its sums reset."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _expected(act: np.ndarray, G: int, executed) -> np.ndarray:
    h = np.abs(act.astype(np.float64)).reshape(-1, G)
    out = h.sum(axis=1).astype(np.float32)  # exact in fp64, one rounding to fp32
    mask = np.zeros(len(out), bool)
    mask[list(executed)] = True
    out[~mask] = 0.0
    return out


def test_importance_single_layer_twice(native_lib, cuda_device):
    import torch
    from gpu_harness import LayerBuffers, make_backend, run_layer, wait_stream
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors, make_layer

    H, G, n = 1024, 64, 64
    L = make_layer(5, H, n, G)
    be = make_backend(H, G, n)
    for epoch, ids in ((1, np.arange(0, n, 4)), (2, np.arange(1, n, 3))):
        rows = descriptors(ids)  # dest = position
        buf = LayerBuffers(H, G, n, L.packed, L.scales, L.x)
        imp = torch.full((n,), -1.0, dtype=torch.float32, device="cuda")
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        run_layer(be, buf, [], rows, epoch=epoch, mode=N.MODE_BATCH_COMPAT, importance=imp, importance_flag=flag)
        wait_stream()
        assert be.status()[N.STATUS_ERROR] == 0, be.status()
        want = _expected(buf.act.cpu().numpy(), G, range(len(rows)))
        got = imp.cpu().numpy()
        assert np.array_equal(got, want), (epoch, np.abs(got - want).max())
        assert got[: len(rows)].min() > 0
        assert int(flag.item()) == epoch
    be.close()


def test_importance_multi_layer_launch(native_lib, cuda_device):
    """Three chained layers in one launch: the per-layer sums alternate
    between two buffers by layer parity, and each layer's entries match its
    own activations."""
    import torch
    from gpu_harness import to_dev, wait_stream
    from leanstream_b200 import B200Backend, ExecutionQueue
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors, make_layer

    H, G, n, layers = 4096, 64, 48, 3
    Ls = [make_layer(300 + l, H, n, G) for l in range(layers)]
    sets = [np.sort(np.random.default_rng(40 + l).permutation(n)[: 12 + 5 * l]) for l in range(layers)]
    be = B200Backend().configure(H, G, n, max_layers=layers, rms_eps=1e-5)
    xs = [to_dev(Ls[0].x.view(np.int16), torch.float16)] + [torch.zeros(H, dtype=torch.float16, device="cuda")
                                                            for _ in range(layers)]
    y = torch.zeros(H, dtype=torch.float16, device="cuda")
    acts = [torch.zeros(n * G, dtype=torch.float16, device="cuda") for _ in range(layers)]
    imps = [torch.full((n,), -1.0, dtype=torch.float32, device="cuda") for _ in range(layers)]
    flags = torch.zeros(layers, dtype=torch.int32, device="cuda")
    keep, args = [], []
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
        args.append(be.layer_args(input=xs[l], output=y, cache=cache, scales=scales, epoch=l + 1, queue=q.view,
                                  mode=N.MODE_BATCH_COMPAT, layer=l, flags=N.NORM_INPUT, residual=xs[l],
                                  hidden_out=xs[l + 1], activations=acts[l], importance=imps[l],
                                  importance_flag=flags[l:l + 1]))
    host = torch.frombuffer(bytearray(b"".join(be.encode_plan(a) for a in args)), dtype=torch.uint8)
    dev = host.cuda()
    be.launch_plans(dev, layers, host.numpy().ctypes.data)
    wait_stream()
    assert be.status()[N.STATUS_ERROR] == 0, be.status()
    for l in range(layers):
        want = _expected(acts[l].cpu().numpy(), G, range(len(sets[l])))
        assert np.array_equal(imps[l].cpu().numpy(), want), l
    assert flags.cpu().tolist() == [1, 2, 3]
    be.close()
