"""C ABI of libleanstream_b200.so without a GPU: every symbol declared in
include/leanstream_b200.h is exported, struct layouts match the reference
types, the kernel selector follows src/runtime/kernel_selector.cpp and
tests/kernel_selector_test.cpp, and the host producer follows
src/runtime/execution_queue.cpp. No compute call is made."""
import ctypes as C
import errno
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "leanstream_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(ls_b200_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_every_declared_symbol_is_exported(native_lib):
    from leanstream_b200 import _native as N

    names = declared_functions()
    assert len(names) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIBRARY)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (ls_b200_[a-z0-9_]+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # and the Python binding declares a signature for each of them
    assert set(names) == set(N.SIGNATURES), set(names) ^ set(N.SIGNATURES)
    for n in names:
        getattr(native_lib, n)


def test_struct_layouts_match_reference_types():
    from leanstream_b200 import _native as N

    assert C.sizeof(N.ExecDesc) == 20  # types.h:20
    assert C.sizeof(N.QueueControl) == 128  # execution_queue.h:12
    assert N.QueueControl.epoch.offset == 12 and N.QueueControl.claim_count.offset == 64
    assert N.QueueControl.error.offset == 20
    assert C.sizeof(N.DeviceExecQueue) == 32
    assert N.ComputeBackend.cancel.offset == 5 * C.sizeof(C.c_void_p)
    assert N.LayerArgs.queue.offset == 56 and N.LayerArgs.flags.offset == 92


def test_quantize_io_load(native_lib):
    """tests/kernel_selector_test.cpp:20-25."""
    q = native_lib.ls_b200_quantize_io_load
    assert q(1, 1, 8) == 7 and q(10, 8, 8) == 7
    assert q(0, 0, 8) == 0 and q(1, 0, 8) == 0
    assert q(1, 8, 0) == 0 and q(0, 8, 8) == 0
    for i in range(8):
        assert q(i, 8, 8) == i
    assert q(2**32 - 2, 2**32 - 1, 8) == 7
    assert q(2**32 - 2, 2**32 - 1, 2**32 - 1) == 2**32 - 2


def test_catalog_and_fallback(native_lib):
    from leanstream_b200 import _native as N

    lib = native_lib
    assert lib.ls_b200_catalog_size() == 6
    default = lib.ls_b200_default_candidate()
    assert default == 4
    c = N.KernelCandidate()
    for cid, ctas in enumerate([4, 8, 16, 32]):  # triton_backend.h:5-8 geometry kept
        assert lib.ls_b200_candidate(None, cid, C.byref(c)) == 0
        assert c.id == cid and c.cta_count == ctas and c.workers == ctas and c.available and c.entry_point == 1
    assert lib.ls_b200_candidate(None, 5, C.byref(c)) == 0 and c.id == 5 and c.entry_point == 0
    assert lib.ls_b200_candidate(None, 99, C.byref(c)) == 0 and c.id == default
    assert lib.ls_b200_candidate(None, 255, C.byref(c)) == 0 and c.id == default


def test_lut_selection_matches_table(native_lib):
    """kernel_selector.cpp:17-22: direct row-major LUT, invalid -> fallback."""
    from leanstream_b200 import B200Backend

    table = [[3, 3, 2, 2, 1, 1, 0, 0], [4, 3, 3, 2, 2, 1, 1, 0], [2, 2, 2, 2, 1, 1, 0, 0]]
    be = B200Backend(table)
    for l in range(3):
        for b in range(8):
            assert be.select(l, b) == table[l][b]
    assert be.select(3, 0) == 4 and be.select(0, 8) == 4  # out of range -> fallback
    be.close()
    bad = B200Backend([[255, 0, 1, 2, 3, 4]])
    assert [bad.select(0, i) for i in range(6)] == [4, 0, 1, 2, 3, 4]
    bad.close()
    assert B200Backend().select(0, 0) == 4


def test_selector_allocation_free_and_fast(native_lib):
    """kernel_selector_test.cpp:44-50 asserts zero allocations in 240k
    lookups; here: 240k lookups through the C ABI, constant results."""
    from leanstream_b200 import B200Backend

    be = B200Backend([[0, 1, 2, 3]])
    sel = native_lib.ls_b200_select
    ctx = be.context
    res = [sel(ctx, 0, i % 4) for i in range(240000)]
    assert res[:4] == [0, 1, 2, 3] and len(set(res)) == 4
    be.close()


def _host_queue(capacity):
    from leanstream_b200 import _native as N

    desc = np.zeros(capacity * 5, np.uint32)
    idx = np.zeros(capacity, np.uint32)
    ctl = np.zeros(32, np.uint32)
    view = N.DeviceExecQueue(desc.ctypes.data, idx.ctypes.data, ctl.ctypes.data, capacity)
    q = N.Queue()
    N.load().ls_b200_queue_bind(C.byref(q), view)
    return q, desc, idx, ctl


def test_queue_protocol_matches_execution_queue(native_lib):
    """execution_queue.cpp:4-46 on plain host memory."""
    lib = native_lib
    q, desc, idx, ctl = _host_queue(8)
    ctl[:] = 7
    assert lib.ls_b200_queue_reset(C.byref(q), 5) == 0
    assert ctl[0] == 0 and ctl[2] == 0 and ctl[3] == 0 and ctl[5] == 0 and ctl[16] == 0  # claim_count zeroed
    assert lib.ls_b200_queue_prepare(C.byref(q), 4) == 0 and ctl[2] == 4
    assert lib.ls_b200_queue_append_unpublished(C.byref(q), 2) == 0
    assert lib.ls_b200_queue_append_unpublished(C.byref(q), 2) != 0  # duplicate rejected
    assert lib.ls_b200_queue_activate(C.byref(q)) == 0
    assert ctl[0] == 1 and ctl[3] == 5 and ctl[4] == 0  # partial plan: no batch epoch
    for i in (0, 3):
        assert lib.ls_b200_queue_publish(C.byref(q), i) == 0
    assert ctl[0] == 3 and ctl[4] == 0
    assert lib.ls_b200_queue_publish(C.byref(q), 1) == 0
    assert ctl[0] == 4 and ctl[4] == 5  # complete -> batch epoch
    assert idx[:4].tolist() == [2, 0, 3, 1]
    assert lib.ls_b200_queue_publish(C.byref(q), 1) != 0  # full
    assert lib.ls_b200_queue_fail(C.byref(q), 5) == 0 and ctl[5] == 5
    assert lib.ls_b200_queue_fail(C.byref(q), 9) == 0 and ctl[5] == 5  # single-shot CAS
    assert lib.ls_b200_queue_reset(C.byref(q), 0) != 0  # epoch must be nonzero
    assert lib.ls_b200_queue_prepare(C.byref(q), 9) != 0  # above capacity


def test_queue_publish_all_and_seal(native_lib):
    lib = native_lib
    q, desc, idx, ctl = _host_queue(6)
    assert lib.ls_b200_queue_reset(C.byref(q), 2) == 0
    assert lib.ls_b200_queue_prepare(C.byref(q), 6) == 0
    assert lib.ls_b200_queue_publish_all(C.byref(q)) == 0
    assert idx.tolist() == list(range(6)) and ctl[0] == 6 and ctl[4] == 2 and ctl[3] == 0
    assert lib.ls_b200_queue_activate(C.byref(q)) == 0 and ctl[3] == 2
    assert lib.ls_b200_queue_reset(C.byref(q), 3) == 0
    assert lib.ls_b200_queue_seal(C.byref(q), 0) == 0  # empty plan is complete at once
    assert ctl[3] == 3 and ctl[4] == 3 and ctl[0] == 0


def test_view_and_unconfigured_errors(native_lib):
    from leanstream_b200 import B200Backend
    from leanstream_b200 import _native as N

    be = B200Backend()
    v = be.view()
    assert v.context == be.context and v.enqueue and v.complete and v.commit and v.cancel
    assert not v.defer_commit
    # launching on an unconfigured backend is refused on the host, before any CUDA call
    args = be.layer_args(input=1 << 20, output=1 << 21, cache=1 << 22, scales=1 << 23, epoch=1,
                         queue=N.DeviceExecQueue(1 << 24, 1 << 25, 1 << 26, 4))
    assert be.launch_rc(args, 0) != 0
    assert native_lib.ls_b200_status(be.context, (C.c_uint32 * 4)(), 4) != 0
    # tensor-parallel setup needs a configured backend; connect needs a setup
    handle = (C.c_uint8 * N.TP_HANDLE_BYTES)()
    assert native_lib.ls_b200_tp_setup(be.context, 0, 2, handle) == errno.EINVAL
    assert native_lib.ls_b200_tp_connect(be.context, handle) == errno.EINVAL
    assert native_lib.ls_b200_tp_setup(None, 0, 2, handle) == errno.EINVAL
    be.close()


def test_geometry_validation_before_device_use(native_lib):
    from leanstream_b200 import _native as N

    lib = native_lib
    ctx = lib.ls_b200_create()
    for h, g, n in [(0, 64, 8), (1000, 64, 8), (768, 64, 8), (8448, 64, 8), (1024, 0, 8), (1024, 512, 8),
                    (1024, 64, 0)]:
        geo = N.Geometry(h, g, n, 0, 0, 0, 0, 0, 1e-5)
        assert lib.ls_b200_configure(ctx, C.byref(geo)) != 0
    lib.ls_b200_destroy(ctx)


def test_build_info(native_lib):
    assert b"sm_100a" in native_lib.ls_b200_build_info()


def test_batch_argument_validation_without_gpu(native_lib):
    """ls_b200_batch_mlp rejects bad arguments before any CUDA call."""
    from leanstream_b200 import _native as N

    lib = native_lib
    need = lib.ls_b200_batch_scratch_bytes(1024, 64, 10)
    assert need >= 8 * 640 * 2 + 4 * 8 * 1024 * 4
    good = dict(hidden=1024, group_size=64, union_count=10, tokens=8, x=1 << 20, output=1 << 21, output_f32=None,
                residual=None, hidden_out=None, cache=1 << 22, staging=None, scales=1 << 23, union_descs=1 << 24,
                mask=None, scratch=1 << 25, scratch_bytes=need)
    for key, bad in [("tokens", 9), ("tokens", 0), ("hidden", 1000), ("hidden", 16384), ("union_count", 0),
                     ("x", None), ("cache", None), ("scratch", None), ("hidden_out", 1 << 26), ("x", (1 << 20) + 8),
                     ("scales", (1 << 23) + 2), ("staging", (1 << 27) + 8), ("scratch", (1 << 25) + 4)]:
        a = N.BatchArgs(**{**good, key: bad})
        assert lib.ls_b200_batch_mlp(C.byref(a), None) == errno.EINVAL, key
    # G * union_count beyond 2^30 neurons is refused (32-bit neuron indices)
    a = N.BatchArgs(**{**good, "union_count": (1 << 30) // 64 + 1, "scratch_bytes": 1 << 62})
    assert lib.ls_b200_batch_mlp(C.byref(a), None) == errno.EINVAL
    a = N.BatchArgs(**{**good, "scratch_bytes": need - 1})
    assert lib.ls_b200_batch_mlp(C.byref(a), None) == errno.ENOSPC
    # a wait bound above 60 s is refused
    a = N.BatchArgs(**{**good, "timeout_ns": 60_000_000_001})
    assert lib.ls_b200_batch_mlp(C.byref(a), None) == errno.EINVAL
    assert lib.ls_b200_batch_mlp(None, None) == errno.EINVAL


def test_selection_path_has_no_timing_or_search():
    """tests/check_selector_contract.py:1-13: the kernel choice is a table
    lookup, never timed or searched at run time. The files of the selection
    and enqueue path here carry none of the timing or tuning calls."""
    files = [ROOT / "leanstream_b200" / "csrc" / "ls_backend.cu", ROOT / "leanstream_b200" / "csrc" / "ls_internal.h",
             ROOT / "leanstream_b200" / "backend.py"]
    forbidden = ("cudaevent", "autotune", "onlineprofiler", "runtimetuner", "autotuner", "benchmark", "cupti")
    for f in files:
        text = f.read_text().lower()
        for word in forbidden:
            assert word not in text, (f.name, word)
