"""Host logic of the streaming IO engine (leanstream_b200/csrc/ls_stream.cu)
without a GPU: the same source is compiled against a host-only stand-in of
the few CUDA runtime calls it makes (tests/native/stub_cuda: a copy is a
memcpy that has landed when its event is queried), and driven through its
IOBackend table the way a WeightManager does (weight_manager.cpp:124-205).
Checked: admission follows the priority list, then the next list for reads
not yet started, then the committed final reads (stream_io.cpp:62-73); a
group is read once per session; READY is published before each completion;
completions carry the session epoch and consecutive sequence numbers;
emulated delays (seeded exponential) still complete every read; a refused
second begin leaves the running session intact; retire, then a new session
starting from EMPTY; argument errors."""
import ctypes as C
import errno
import shutil
import subprocess
import threading
import time
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def host_engine_lib(tmp_path_factory):
    from leanstream_b200 import _native as N

    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ is not available")
    d = tmp_path_factory.mktemp("stream_host")
    # the engine source beside the stand-in internal header (quoted includes
    # resolve in the source's directory first)
    shutil.copy(ROOT / "leanstream_b200" / "csrc" / "ls_stream.cu", d / "ls_stream.cpp")
    shutil.copy(ROOT / "tests" / "native" / "stub_cuda" / "ls_internal.h", d / "ls_internal.h")
    out = d / "libstream_host.so"
    subprocess.run([gxx, "-std=c++17", "-O1", "-fPIC", "-shared", "-pthread",
                    "-I", str(ROOT / "tests" / "native" / "stub_cuda"), "-I", str(ROOT / "include"),
                    str(d / "ls_stream.cpp"), "-o", str(out)], check=True, capture_output=True)
    lib = C.CDLL(str(out), use_errno=True)
    for name in ("ls_b200_stream_create", "ls_b200_stream_view", "ls_b200_stream_stats",
                 "ls_b200_stream_issue_log", "ls_b200_stream_destroy"):
        res, args = N.SIGNATURES[name]
        f = getattr(lib, name)
        f.restype, f.argtypes = res, args
    return lib


@pytest.fixture
def engine(host_engine_lib, monkeypatch):
    from leanstream_b200 import stream as S

    monkeypatch.setattr(S.N, "load", lambda: host_engine_lib)
    made = []

    def make(n=40, gb=256, qd=4, delay_us=0.0, seed=1):
        host = np.random.default_rng(seed).integers(0, 256, n * gb, dtype=np.uint8)
        staging = np.zeros(n * gb, np.uint8)
        eng = S.StreamEngine(host.ctypes.data, [g * gb for g in range(n)], staging.ctypes.data, gb, gb,
                             queue_depth=qd, delay_mean_us=delay_us, delay_seed=seed)
        made.append(eng)
        return eng, S.IOBackendView(eng.view()), host.reshape(n, gb), staging.reshape(n, gb)

    yield make
    for eng in made:
        eng.close()


def _wait_issued(eng, ids, timeout=5.0):
    deadline = time.monotonic() + timeout
    while not set(ids) <= set(eng.issue_log()):
        assert time.monotonic() < deadline, "engine did not admit the list"
        time.sleep(0.0005)


def test_admission_order_reorder_and_commit(engine):
    from leanstream_b200 import _native as N

    eng, io, host, staging = engine()
    done, lock = [], threading.Lock()

    def on_done(epoch, group, slot, error, seq):
        assert eng.io_states[group] == N.IO_READY  # READY before the completion
        with lock:
            done.append((epoch, group, slot, error, seq))

    assert io.begin(on_done, 7) == 0
    p0 = [3, 17, 5, 29, 11]
    assert io.update(p0) == 0
    _wait_issued(eng, p0)
    p1 = [5, 22, 3, 8, 31]  # 5 and 3 already read: never read again
    assert io.update(p1) == 0
    _wait_issued(eng, p1)
    final = [8, 3, 36, 12]
    assert io.consume(final) == 0
    assert io.wait(5000) == 0
    issued = eng.issue_log()
    assert issued == p0 + [22, 8, 31] + [36, 12]
    assert io.retire() == 0
    for g in issued:
        assert np.array_equal(staging[g], host[g])
    untouched = [g for g in range(len(host)) if g not in issued]
    assert not staging[untouched].any()
    assert sorted(d[1] for d in done) == sorted(issued)
    assert all(d[0] == 7 and d[2] == d[1] and d[3] == 0 for d in done)
    assert sorted(d[4] for d in done) == list(range(1, len(issued) + 1))
    st = eng.stats()
    assert st["admissions"] == st["completions"] == len(issued) and st["bytes"] == len(issued) * 256
    assert io.requests() == len(issued) and io.ready_slot(8) == 8 and io.ready_slot(40) == -1


def test_delays_complete_every_read_and_sessions_restart(engine):
    from leanstream_b200 import _native as N

    eng, io, host, staging = engine(qd=8, delay_us=30.0, seed=5)
    seen = []
    assert io.begin(lambda *a: seen.append(a[1]), 1) == 0
    ids = list(range(0, 40, 2))
    assert io.update(ids[:10]) == 0
    assert io.consume(ids) == 0
    assert io.wait(5000) == 0
    assert all(eng.io_states[g] == N.IO_READY for g in ids)
    assert io.retire() == 0
    assert sorted(seen) == ids
    # a new session starts from EMPTY and reads again
    seen.clear()
    assert io.begin(lambda *a: seen.append(a[1]), 2) == 0
    assert all(eng.io_states[g] == N.IO_EMPTY for g in range(40))
    assert io.consume([1, 2]) == 0
    assert io.wait(5000) == 0
    assert io.retire() == 0
    assert sorted(seen) == [1, 2]


def test_refused_begin_and_argument_errors(engine):
    eng, io, host, staging = engine()
    assert io.update([1]) == errno.EINVAL       # no session
    assert io.retire() == errno.EINVAL
    hits = []
    assert io.begin(lambda *a: hits.append(a[1]), 3) == 0
    # a refused begin must leave the running session's callback in place
    assert io.begin(lambda *a: None, 4) == errno.EBUSY
    assert io.update([40]) == errno.EINVAL      # out of range
    assert io.update([-1]) == errno.EINVAL
    assert io.consume([6]) == 0
    assert io.wait(5000) == 0
    assert io.retire() == 0
    assert hits == [6]
