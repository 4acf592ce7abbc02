"""Streaming IO (ls_b200_stream_*): the IOBackend of
include/leanstream/weight_manager.h:14-24 over pinned host memory -> HBM
staging. CPU tests check the boundary without a GPU; GPU tests drive the
engine through its IOBackend table (the calls a WeightManager makes,
weight_manager.cpp:124-205) and, with the reference's own runtime compiled
into oracle/_ref, a whole config-4 layer step (tests/native/runtime_driver.cpp):
weights in pinned host memory, predicted groups copied on a side stream and
published in a seeded random order (exponential delays, mean 20 us), a
mid-step prediction update, the persistent consumer at 4/8/16/32 CTAs through
the KernelSelector LUT."""
import ctypes as C
import errno
import json
import os
import subprocess
import threading
import time
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
DRIVER = ROOT / "oracle" / "_ref" / "runtime_driver"
TOL = 2e-3


def test_stream_config_validation_without_gpu(native_lib):
    from leanstream_b200 import _native as N

    lib = native_lib
    states = np.zeros(5, np.uint32)
    offs = np.arange(4, dtype=np.uint64) * 1024
    good = dict(host_base=1 << 20, host_offsets=offs.ctypes.data, staging=1 << 30, staging_stride=1024,
                group_bytes=1024, io_states=states.ctypes.data, group_count=4, queue_depth=8, device=0,
                delay_mean_us=0.0, delay_seed=0)
    for key, bad in [("host_base", None), ("staging", None), ("io_states", None), ("group_count", 0),
                     ("queue_depth", 0), ("queue_depth", 33), ("group_bytes", 0), ("group_bytes", 2048),
                     ("delay_mean_us", -1.0), ("host_offsets", None)]:
        cfg = N.StreamConfig(**{**good, key: bad})
        assert not lib.ls_b200_stream_create(C.byref(cfg)), key
        assert C.get_errno() == errno.EINVAL, key
    assert lib.ls_b200_stream_view(None, C.byref(N.IOBackend())) == errno.EINVAL
    assert lib.ls_b200_stream_stats(None, C.byref(N.StreamStats())) == errno.EINVAL
    assert lib.ls_b200_stream_issue_log(None, None, 0) == 0
    lib.ls_b200_stream_destroy(None)


@pytest.mark.gpu
def test_engine_priority_order_reorder_and_bytes(native_lib, cuda_device):
    """update -> admissions follow the priority order; a second update
    reorders the reads not yet started (a started read is never repeated);
    consume adds the committed final reads; every committed group lands
    byte-exact before its READY word and its completion (stream_io.cpp:62-73,
    weight_manager.cpp:135-151,190-205)."""
    import torch

    from leanstream_b200 import _native as N
    from leanstream_b200.stream import IOBackendView, StreamEngine

    n, gb = 48, 4 << 20  # 4 MB groups, one copy in flight: reads stay pending long enough to reorder
    rng = np.random.default_rng(4)
    host = torch.from_numpy(rng.integers(0, 256, n * gb, dtype=np.uint8)).pin_memory()
    staging = torch.zeros(n * gb, dtype=torch.uint8, device="cuda")
    eng = StreamEngine(host.data_ptr(), [g * gb for g in range(n)], staging.data_ptr(), gb, gb, queue_depth=1,
                       delay_mean_us=20.0, delay_seed=7)
    io = IOBackendView(eng.view())
    done, lock = [], threading.Lock()

    def on_done(epoch, group, slot, error, seq):
        assert eng.io_states[group] == N.IO_READY  # READY is published before the callback
        with lock:
            done.append((epoch, group, slot, error, seq))

    assert io.begin(on_done, 5) == 0
    assert io.begin(on_done, 6) == errno.EBUSY
    perm = [int(g) for g in rng.permutation(n)]
    p0 = perm[:20]
    p1 = p0[4:][::-1] + perm[20:24]
    assert io.update(p0) == 0
    assert io.update(p1) == 0
    deadline = time.monotonic() + 10
    while not set(p1) <= set(eng.issue_log()):
        assert time.monotonic() < deadline, "the engine did not admit the second priority list"
        time.sleep(0.001)
    final = sorted(set(p0[:2]) | set(p1[:3]) | {perm[30], perm[31]})
    assert io.consume(final) == 0
    assert io.wait(10000) == 0
    issued = eng.issue_log()
    assert len(issued) == len(set(issued)), "a group is read at most once per session"
    k = 0
    while k < len(issued) and issued[k] == p0[k]:
        k += 1
    assert k <= 4, issued[:6]  # the first update started at most a few reads (none if the second came first)
    second = [g for g in p1 if g not in issued[:k]]
    assert issued[k:k + len(second)] == second
    third = [g for g in final if g not in issued[:k + len(second)]]
    assert issued[k + len(second):] == third
    assert io.retire() == 0
    assert io.ready_slot(3) == 3 and io.ready_slot(n) == -1
    assert io.requests() == len(issued)
    st = eng.stats()
    assert st["error"] == 0 and st["bytes"] == len(issued) * gb and st["completions"] == len(issued)
    got = staging.cpu().numpy().reshape(n, gb)
    ref = host.numpy().reshape(n, gb)
    for g in issued:
        assert np.array_equal(got[g], ref[g]), g
    assert sorted(d[1] for d in done) == sorted(issued)
    assert all(d[0] == 5 and d[2] == d[1] and d[3] == 0 for d in done)
    assert sorted(d[4] for d in done) == list(range(1, len(done) + 1))
    # a new session starts from EMPTY
    assert io.begin(on_done, 6) == 0
    assert int(eng.io_states[issued[0]]) == N.IO_EMPTY
    assert io.retire() == 0
    eng.close()


@pytest.mark.gpu
@pytest.mark.parametrize("o_direct", [True, False])
def test_engine_reads_groups_from_a_file(native_lib, cuda_device, tmp_path, o_direct):
    """The SSD leg (src/io/stream_io.cpp:75-148): groups are read from a file
    (pread by the reader pool, O_DIRECT when the file system allows it) into
    their pinned host slots, then copied to HBM staging. The layout is
    config 1's groups (101,376 B) at 4 KB-aligned file offsets, host slots
    rounded up to the alignment; every committed group lands byte-exact, and
    the counters report the bytes read and whether O_DIRECT was in effect."""
    import torch

    from leanstream_b200 import _native as N
    from leanstream_b200.stream import IOBackendView, StreamEngine

    n, gb, align = 24, 64 * 3 * 1024 // 2, 4096
    slot = (gb + align - 1) // align * align
    rng = np.random.default_rng(12)
    data = rng.integers(0, 256, (n, gb), dtype=np.uint8)
    file_offsets = [align + g * (slot + align) for g in range(n)]  # gaps between groups, as a packed layout may have
    path = tmp_path / "groups.bin"
    blob = np.zeros(file_offsets[-1] + slot, np.uint8)
    for g in range(n):
        blob[file_offsets[g]:file_offsets[g] + gb] = data[g]
    blob.tofile(path)
    host = torch.zeros(n * slot + align, dtype=torch.uint8).pin_memory()
    base = (host.data_ptr() + align - 1) // align * align  # 4 KB-aligned host slots
    staging = torch.zeros(n * gb, dtype=torch.uint8, device="cuda")
    eng = StreamEngine(base, [g * slot for g in range(n)], staging.data_ptr(), gb, gb, queue_depth=8,
                       file_path=str(path), file_offsets=file_offsets, read_workers=4, o_direct=o_direct)
    io = IOBackendView(eng.view())
    landed = []
    assert io.begin(lambda e, g, s_, err, seq: landed.append((g, err)), 1) == 0
    prio = [int(g) for g in rng.permutation(n)[:10]]
    final = sorted(set(prio[:6]) | {int(rng.integers(n))})
    assert io.update(prio) == 0
    assert io.consume(final) == 0
    assert io.wait(20000) == 0
    assert io.retire() == 0
    st = eng.stats()
    issued = eng.issue_log()
    assert st["error"] == 0 and st["completions"] == len(issued) and set(final) <= set(issued)
    assert st["read_bytes"] >= len(issued) * gb and st["read_ns"] > 0
    assert st["direct"] in (0, 1) and (o_direct or st["direct"] == 0)
    got = staging.cpu().numpy().reshape(n, gb)
    for g in issued:
        assert np.array_equal(got[g], data[g]), g
        assert int(eng.io_states[g]) == N.IO_READY
    assert sorted(g for g, _ in landed) == sorted(issued) and all(err == 0 for _, err in landed)
    eng.close()


def test_engine_file_source_errors_on_host(native_lib, tmp_path):
    """A file source that cannot be opened is refused at creation (errno of
    open, here ENOENT), and one without file offsets is EINVAL -- before any
    read is issued. Needs no GPU when none is visible: creation then fails
    with ENODEV first, which is checked instead."""
    from leanstream_b200 import _native as N

    lib = native_lib
    states = np.zeros(3, np.uint32)
    offs = np.zeros(2, np.uint64)
    cfg = N.StreamConfig(1 << 20, offs.ctypes.data, 1 << 30, 4096, 4096, states.ctypes.data, 2, 4, 0, 0.0, 0,
                         str(tmp_path / "missing.bin").encode(), offs.ctypes.data, 2, 1, 4096)
    assert not lib.ls_b200_stream_create(C.byref(cfg))
    assert C.get_errno() in (errno.ENOENT, errno.ENODEV)


def _config4_inputs(tmp_path, H=1024, G=64, N=64, seed=0):
    from leanstream_b200.synthetic import make_layer

    L = make_layer(seed, H, N, G)
    rng = np.random.default_rng(100 + seed)
    perm = rng.permutation(N)
    p0 = perm[:24]
    p1 = np.concatenate([perm[8:24][::-1], perm[24:28]])
    final = np.concatenate([perm[:6], perm[10:16], perm[24:28]])  # 16 groups (25%), mixed prediction ranks
    L.packed.tofile(tmp_path / "packed.bin")
    L.scales.reshape(-1).tofile(tmp_path / "scales.bin")
    L.x.tofile(tmp_path / "x.bin")
    (tmp_path / "plan.txt").write_text("\n".join(" ".join(str(int(v)) for v in a) for a in (p0, p1, final)) + "\n")
    return L, final


@pytest.mark.gpu
@pytest.mark.parametrize("delay_us", [0, 20])
@pytest.mark.parametrize("candidate", [0, 1, 2, 3, 4])
def test_reference_runtime_streams_config4(native_lib, cuda_device, tmp_path, candidate, delay_us):
    from leanstream_b200.synthetic import descriptors
    from oracle import oracle as O

    if not DRIVER.exists():
        pytest.fail(f"{DRIVER} is missing: build it with `make -C oracle ref` where the reference is mounted")
    H, G, N = 1024, 64, 64
    L, final = _config4_inputs(tmp_path, H, G, N)
    out = subprocess.run([str(DRIVER), str(tmp_path), str(H), str(G), str(N), "8", str(delay_us), str(candidate), "8"],
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    rep = json.loads(out.stdout.strip().splitlines()[-1])
    print("config4", json.dumps(rep))  # timings of the step, shown with pytest -s
    assert rep["final_groups"] == len(final) and rep["h2d_bytes"] >= len(final) * G * 3 * H // 2
    y = np.fromfile(tmp_path / "y.bin", dtype=np.float16).astype(np.float32)
    y_ref, _, _ = O.mlp(H, G, L.x, L.packed, L.scales, descriptors(final))
    ref = y_ref.astype(np.float32)
    assert np.abs(y - ref).max() <= TOL * np.abs(ref).max()
