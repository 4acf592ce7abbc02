"""ls_b200_launch_static: the launch that allocates nothing, its scratch a
fixed set of device arrays in the library. Its output must match
ls_b200_launch on the same layer, on two calls in a row (the second one
meets the first one's tagged scratch), and its limits are checked on the
host before any CUDA call. The file name sorts last so that the GPU test
also runs after every other test of the session has used the device."""
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
    big_layer = B200Backend.layer_args(layer=256)
    assert lib.ls_b200_launch_static(C.byref(_geometry(4096, 64, 256)), C.byref(big_layer), None,
                                     None) == errno.E2BIG
    assert lib.ls_b200_launch_static(C.byref(_geometry(768, 64, 8)), C.byref(args), None, None) == errno.EINVAL
    assert lib.ls_b200_launch_static(C.byref(_geometry(8192, 64, 8)), C.byref(args), None, None) == errno.EINVAL
    assert lib.ls_b200_launch_static(None, C.byref(args), None, None) == errno.EINVAL
    # within the limits, but args without epoch / buffers: encode rejects it
    assert lib.ls_b200_launch_static(C.byref(_geometry(4096, 64, 256)), C.byref(args), None, None) == errno.EINVAL


def _static_layer(geo, buf, rows, status, epoch=1):
    import torch
    from leanstream_b200 import B200Backend, ExecutionQueue
    from leanstream_b200 import _native as N

    q = ExecutionQueue(max(len(rows), 1))
    q.reset(epoch)
    q.write_descriptors(rows)
    q.prepare(len(rows))
    for i in range(len(rows)):
        q.append_unpublished(i)
    q.activate()
    args = B200Backend.layer_args(input=buf.x, output=buf.y, cache=buf.cache, staging=buf.staging,
                                  scales=buf.scales, epoch=epoch, queue=q.view, mode=N.MODE_PROGRESSIVE,
                                  activations=buf.act, executions=buf.execs, output_f32=buf.y32)
    rc = N.load().ls_b200_launch_static(C.byref(geo), C.byref(args), C.c_void_p(status.data_ptr()),
                                        C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    return q


@pytest.mark.gpu
@pytest.mark.parametrize("H,n_groups,n_active,seed", [(4096, 192, 58, 11), (1024, 64, 16, 0)])
def test_static_launch_matches_launch_twice(native_lib, cuda_device, H, n_groups, n_active, seed):
    """Config 1 (H 4096, 58 of 192 groups) and config 0 (H 1024, 16 of 64),
    in that order, so the H 1024 calls find the H 4096 calls' words in the
    shared scratch."""
    import torch
    from gpu_harness import LayerBuffers, make_backend, run_layer, wait_stream
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors, make_layer

    G = 64
    L = make_layer(seed, H, n_groups, G)
    ids = np.sort(np.random.default_rng(seed).permutation(n_groups)[:n_active])
    rows = descriptors(ids)

    ref = LayerBuffers(H, G, n_groups, L.packed, L.scales, L.x)
    be = make_backend(H, G, n_groups, cache_slots=n_groups, physical_groups=n_groups)
    run_layer(be, ref, [], rows, mode=N.MODE_PROGRESSIVE)
    wait_stream()
    assert be.status()[N.STATUS_ERROR] == 0, be.status()
    be.close()
    y_ref = ref.y.cpu().numpy().astype(np.float32)
    y32_ref = ref.y32.cpu().numpy()
    assert np.abs(y_ref).max() > 0

    geo = _geometry(H, G, n_groups, cache_slots=n_groups, physical_groups=n_groups)
    sel = np.asarray([r[3] for r in rows])
    for call in range(2):
        buf = LayerBuffers(H, G, n_groups, L.packed, L.scales, L.x)
        status = torch.zeros(N.STATUS_WORDS, dtype=torch.int32, device=cuda_device)
        _static_layer(geo, buf, rows, status)
        wait_stream()
        st = status.cpu().numpy()
        assert st[N.STATUS_ERROR] == 0, (call, st)
        assert st[N.STATUS_LAUNCHES] != 0, (call, st)
        y = buf.y.cpu().numpy().astype(np.float32)
        bound = TOL * np.abs(y_ref).max()
        assert np.abs(y - y_ref).max() <= bound, (call, np.abs(y - y_ref).max(), bound)
        assert np.abs(buf.y32.cpu().numpy() - y32_ref).max() <= TOL * np.abs(y32_ref).max(), call
        execs = buf.execs.cpu().numpy()
        assert np.all(execs[sel] == 1) and execs.sum() == len(rows), call
