"""ls_b200_launch_static: the launch for callers that cannot allocate device
memory on their launch path (an engine whose pool already owns all of HBM,
a launch path where a cudaMalloc would synchronise the device). Its scratch
is a fixed set of device arrays in the library.

Checked here: the limits are rejected on the host before any CUDA call; on
the GPU, two calls in a row with different activations and active sets each
match ls_b200_launch on the same layer bit for bit (the same kernel and
arithmetic), the first one also matches the CPU oracle within the north_star
tolerance, and neither call changes the device's free memory. The file name
sorts last, so the GPU test also runs after every other test of a session
has used the device."""
import ctypes as C
import errno

import numpy as np
import pytest

TOL = 2e-3  # max|y - y_ref| <= 2e-3 * ||y_ref||_inf


def _geometry(H, G, N_groups, **kw):
    from leanstream_b200 import _native as N

    return N.Geometry(H, G, N_groups, kw.get("max_layers", 0), kw.get("cache_slots", 0), 0,
                      kw.get("physical_groups", 0), kw.get("timeout_us", 2_000_000), 1e-5)


def test_static_limits_rejected_on_host(native_lib):
    """E2BIG past the fixed scratch, EINVAL for what ls_b200_launch rejects;
    no device is touched (this runs without a GPU)."""
    from leanstream_b200 import B200Backend
    from leanstream_b200 import _native as N

    lib = N.load()
    args = B200Backend.layer_args(layer=0)
    # 4096 x ceil(64/16) x 257 groups = 4,210,688 tagged words > 2^22
    assert lib.ls_b200_launch_static(C.byref(_geometry(4096, 64, 257)), C.byref(args), None, None) == errno.E2BIG
    # H 8192 is a supported hidden size: its geometry passes and 129 groups
    # (4,227,072 words) are rejected for size, not shape
    assert lib.ls_b200_launch_static(C.byref(_geometry(8192, 64, 129)), C.byref(args), None, None) == errno.E2BIG
    big_layer = B200Backend.layer_args(layer=256)
    assert lib.ls_b200_launch_static(C.byref(_geometry(4096, 64, 256)), C.byref(big_layer), None,
                                     None) == errno.E2BIG
    for bad_hidden in (768, 1280, 16384):  # not 256 * 2^k, or above the kernel's 8192
        assert lib.ls_b200_launch_static(C.byref(_geometry(bad_hidden, 64, 8)), C.byref(args), None,
                                         None) == errno.EINVAL
    assert lib.ls_b200_launch_static(None, C.byref(args), None, None) == errno.EINVAL
    # within the limits, but args without epoch / buffers: encode rejects it
    assert lib.ls_b200_launch_static(C.byref(_geometry(4096, 64, 256)), C.byref(args), None, None) == errno.EINVAL


def _queue(rows, epoch=1):
    from leanstream_b200 import ExecutionQueue

    q = ExecutionQueue(max(len(rows), 1))
    q.reset(epoch)
    q.write_descriptors(rows)
    q.prepare(len(rows))
    for i in range(len(rows)):
        q.append_unpublished(i)
    q.activate()
    return q


def _static_args(buf, rows):
    """Queue (pinned host memory) and arguments of one static call, made
    before the free-memory snapshot."""
    from leanstream_b200 import B200Backend
    from leanstream_b200 import _native as N

    q = _queue(rows)
    args = B200Backend.layer_args(input=buf.x, output=buf.y, cache=buf.cache, staging=buf.staging,
                                  scales=buf.scales, epoch=1, queue=q.view, mode=N.MODE_PROGRESSIVE,
                                  activations=buf.act, executions=buf.execs, output_f32=buf.y32)
    return q, args


def _launch_static(geo, args, status):
    import torch
    from leanstream_b200 import _native as N

    rc = N.load().ls_b200_launch_static(C.byref(geo), C.byref(args), C.c_void_p(status.data_ptr()),
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc


@pytest.mark.gpu
@pytest.mark.parametrize("H,n_groups,n_active,seed", [(4096, 192, 58, 11), (1024, 64, 16, 0)])
def test_static_launch_matches_launch_twice(native_lib, cuda_device, H, n_groups, n_active, seed):
    """BASELINE.json configuration 2's layer (H 4096, 58 of 192 groups), then
    configuration 1's geometry (H 1024, 16 of 64), in that order, so the
    H 1024 calls find the H 4096 calls' words in the shared scratch. Each
    parametrisation makes two static calls in a row with different
    activations and active sets."""
    import torch
    from gpu_harness import LayerBuffers, make_backend, run_layer, wait_stream
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    G = 64
    L = make_layer(seed, H, n_groups, G)
    rng = np.random.default_rng(seed)
    calls = []
    for c in range(2):
        ids = np.sort(rng.permutation(n_groups)[:n_active - 3 * c])  # a different set each call
        x = (rng.standard_normal(H) * (1.0 + 0.5 * c)).astype(np.float16)
        calls.append((descriptors(ids), x))

    lib = N.load()
    assert lib.ls_b200_launch_static(None, None, None,
                                     C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0  # set-up only
    # references from the allocating entry point, and every buffer, first
    refs, bufs = [], []
    for rows, x in calls:
        ref = LayerBuffers(H, G, n_groups, L.packed, L.scales, x)
        be = make_backend(H, G, n_groups, cache_slots=n_groups, physical_groups=n_groups)
        run_layer(be, ref, [], rows, mode=N.MODE_PROGRESSIVE)
        wait_stream()
        assert be.status()[N.STATUS_ERROR] == 0, be.status()
        be.close()
        refs.append(ref)
        bufs.append(LayerBuffers(H, G, n_groups, L.packed, L.scales, x))
    statuses = [torch.zeros(N.STATUS_WORDS, dtype=torch.int32, device=cuda_device) for _ in calls]
    prepared = [_static_args(bufs[c], rows) for c, (rows, _) in enumerate(calls)]
    geo = _geometry(H, G, n_groups, cache_slots=n_groups, physical_groups=n_groups)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]

    for c in range(len(calls)):
        _launch_static(geo, prepared[c][1], statuses[c])
        wait_stream()
    free_after = torch.cuda.mem_get_info()[0]
    assert free_after == free_before, (free_before, free_after)

    for c, (rows, x) in enumerate(calls):
        st = statuses[c].cpu().numpy()
        assert st[N.STATUS_ERROR] == 0, (c, st)
        assert st[N.STATUS_LAUNCHES] != 0, (c, st)
        buf, ref = bufs[c], refs[c]
        # the same kernel on the same inputs: identical bits
        assert torch.equal(buf.y, ref.y), c
        assert torch.equal(buf.y32, ref.y32), c
        assert torch.equal(buf.act, ref.act), c
        sel = np.asarray([r[3] for r in rows])
        execs = buf.execs.cpu().numpy()
        assert np.all(execs[sel] == 1) and execs.sum() == len(rows), c
        if c == 0:  # and the reference math (CPU oracle) within the tolerance
            y_ref, _, _ = O.mlp(H, G, x, L.packed, L.scales, rows)
            y_ref = y_ref.astype(np.float32)
            got = buf.y.cpu().numpy().astype(np.float32)
            assert np.abs(got - y_ref).max() <= TOL * np.abs(y_ref).max()
