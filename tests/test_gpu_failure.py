"""Failure detection of the fused kernel without a GPU fault. Every device-side
wait has a short limit here (timeout_us = 50 ms); a test makes one wait run
out (a queue word nothing sets, a descriptor nothing publishes) or sets the
ExecutionQueue's error word from the host (execution_queue.cpp:44-46), then
reads the error status the kernel recorded (LS_B200_STATUS_*) and checks that
the context stays usable: the same backend then runs a normal layer. The
reference's CUDA backend exits its consumer on QueueControl.error and on its
own timeouts in the same way (streaming_mlp.cu:49-56,63-75)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, G, N_GROUPS = 1024, 64, 12
TIMEOUT_US = 50_000


def _setup():
    from gpu_harness import LayerBuffers, make_backend
    from leanstream_b200.synthetic import make_layer

    L = make_layer(41, H, N_GROUPS, G)
    buf = LayerBuffers(H, G, N_GROUPS, L.packed, L.scales, L.x)
    be = make_backend(H, G, N_GROUPS, timeout_us=TIMEOUT_US)
    return L, buf, be


def _launch(be, buf, q, epoch):
    from leanstream_b200 import _native as N

    args = be.layer_args(input=buf.x, output=buf.y, cache=buf.cache, staging=buf.staging, scales=buf.scales,
                         epoch=epoch, queue=q.view, mode=N.MODE_PROGRESSIVE, executions=buf.execs,
                         output_f32=buf.y32)
    be.launch(args)


def _still_usable(be, buf, L):
    """After clearing the status, the same backend computes a normal layer."""
    from gpu_harness import run_layer, wait_stream
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors
    from oracle import oracle as O

    be.clear_status()
    assert be.status()[N.STATUS_ERROR] == 0
    buf.execs.zero_()
    rows = descriptors(np.array([2, 7, 9]))
    run_layer(be, buf, [], rows, epoch=77)
    wait_stream()
    assert be.status()[N.STATUS_ERROR] == 0, be.status()
    y_ref, _, _ = O.mlp(H, G, L.x, L.packed, L.scales, rows)
    ref = y_ref.astype(np.float32)
    y = buf.y.cpu().numpy().astype(np.float32)
    assert np.abs(y - ref).max() <= 2e-3 * np.abs(ref).max()


def test_queue_never_activated_times_out(native_lib, cuda_device):
    from gpu_harness import wait_stream
    from leanstream_b200 import ExecutionQueue
    from leanstream_b200 import _native as N

    L, buf, be = _setup()
    q = ExecutionQueue(N_GROUPS)
    q.reset(5)  # the epoch word is published only by activate(), which never comes
    _launch(be, buf, q, 5)
    wait_stream(timeout_s=10.0)
    st = be.status()
    assert st[N.STATUS_ERROR] == N.DEV_TIMEOUT_EPOCH, st
    assert st[N.STATUS_ERROR_EPOCH] == 5
    _still_usable(be, buf, L)
    be.close()


def test_queue_error_word_ends_the_launch(native_lib, cuda_device):
    from gpu_harness import wait_stream
    from leanstream_b200 import ExecutionQueue
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors

    L, buf, be = _setup()
    q = ExecutionQueue(N_GROUPS)
    q.reset(6)
    q.write_descriptors(descriptors(np.array([1, 3, 4])))
    q.prepare(3)
    q.activate()
    q.fail(5)  # EIO from a failed read, published before any descriptor
    _launch(be, buf, q, 6)
    wait_stream(timeout_s=10.0)
    st = be.status()
    assert st[N.STATUS_ERROR] == N.DEV_QUEUE_ERROR, st
    assert int(buf.execs.sum().item()) == 0  # nothing was computed
    _still_usable(be, buf, L)
    be.close()


def test_descriptor_never_published_times_out(native_lib, cuda_device):
    from gpu_harness import wait_stream
    from leanstream_b200 import ExecutionQueue
    from leanstream_b200 import _native as N
    from leanstream_b200.synthetic import descriptors

    L, buf, be = _setup()
    q = ExecutionQueue(N_GROUPS)
    q.reset(8)
    q.write_descriptors(descriptors(np.array([0, 5, 10])))
    q.prepare(3)
    q.activate()
    _launch(be, buf, q, 8)
    q.publish(0)  # positions 1 and 2 are never published
    wait_stream(timeout_s=10.0)
    st = be.status()
    assert st[N.STATUS_ERROR] == N.DEV_TIMEOUT_READY, st
    _still_usable(be, buf, L)
    be.close()
