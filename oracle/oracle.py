"""CPU ORACLE bindings -- test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, as the checker or the timed CPU baseline. The product package
(leanstream_b200/) never imports it.

Two libraries:
  * libls_oracle.so  -- ls_oracle.c, the C restatement of the reference math;
  * _ref/libls_predictor_ref.so -- the reference's own predictor/predictor_cpu.cpp
    compiled unmodified from the reference tree (REFERENCE_ROOT) by
    oracle/Makefile (`make ref`), which also builds the reference runtime
    and the integration driver of tests/native.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "libls_oracle.so"
REF_DIR = HERE / "_ref"
PREDICTOR_LIB = REF_DIR / "libls_predictor_ref.so"
# The reference checkout: $LEANSTREAM_REFERENCE, else the directory
# `reference` beside this repository's root. It is only read to build the
# reference objects of _ref/ (absent on machines without the checkout).
REFERENCE_ROOT = Path(os.environ.get("LEANSTREAM_REFERENCE") or (HERE.parents[1] / "reference")).resolve()

_oracle = None
_predictor = None


def build(reference: bool = True) -> None:
    """Compiles the oracle; the reference objects too when the reference is mounted."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    if reference and REFERENCE_ROOT.exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", "ref-cuda", f"REF={REFERENCE_ROOT}"], check=True)


def _u16(a):
    return np.ascontiguousarray(a).view(np.uint16)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def lib() -> C.CDLL:
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists():
            build(reference=False)
        L = C.CDLL(str(ORACLE_LIB))
        vp, u32 = C.c_void_p, C.c_uint32
        L.ls_oracle_mlp.argtypes = [u32, u32, vp, vp, vp, vp, vp, u32, vp, vp, vp]
        L.ls_oracle_mlp_f64.argtypes = [u32, u32, vp, vp, vp, vp, vp, u32, vp]
        L.ls_oracle_mlp_omp.argtypes = [u32, u32, vp, vp, vp, vp, vp, u32, vp, C.c_int]
        L.ls_oracle_neuron.argtypes = [u32, vp, vp, vp, vp, vp, vp]
        L.ls_oracle_rmsnorm.argtypes = [u32, vp, vp, C.c_float, vp]
        L.ls_oracle_residual.argtypes = [u32, vp, vp, vp]
        L.ls_oracle_f2h.argtypes = [C.c_float]
        L.ls_oracle_f2h.restype = C.c_uint16
        L.ls_oracle_h2f.argtypes = [C.c_uint16]
        L.ls_oracle_h2f.restype = C.c_float
        L.ls_oracle_max_threads.restype = C.c_int
        _oracle = L
    return _oracle


def mlp(hidden, group_size, x, cache, scales, descs, staging=None, h_out_groups=0):
    """Sparse MLP (ls_oracle_mlp). Returns (y16 float16 [H], y32 float32 [H], h or None)."""
    L = lib()
    x = _u16(np.asarray(x, dtype=np.float16))
    scales = _u16(np.asarray(scales, dtype=np.float16).reshape(-1))
    cache = np.ascontiguousarray(cache, dtype=np.uint8)
    staging = cache if staging is None else np.ascontiguousarray(staging, dtype=np.uint8)
    d = np.ascontiguousarray(np.asarray(descs, dtype=np.uint32).reshape(-1, 5))
    y32 = np.zeros(hidden, dtype=np.float32)
    y16 = np.zeros(hidden, dtype=np.uint16)
    h = np.zeros(h_out_groups * group_size, dtype=np.uint16) if h_out_groups else None
    rc = L.ls_oracle_mlp(hidden, group_size, _ptr(x), _ptr(cache), _ptr(staging), _ptr(scales), _ptr(d),
                         len(d), _ptr(y32), _ptr(y16), _ptr(h))
    if rc:
        raise ValueError("ls_oracle_mlp rejected its arguments")
    return y16.view(np.float16), y32, (None if h is None else h.view(np.float16))


def mlp_f64(hidden, group_size, x, cache, scales, descs, staging=None):
    L = lib()
    x = _u16(np.asarray(x, dtype=np.float16))
    scales = _u16(np.asarray(scales, dtype=np.float16).reshape(-1))
    cache = np.ascontiguousarray(cache, dtype=np.uint8)
    staging = cache if staging is None else np.ascontiguousarray(staging, dtype=np.uint8)
    d = np.ascontiguousarray(np.asarray(descs, dtype=np.uint32).reshape(-1, 5))
    y = np.zeros(hidden, dtype=np.float64)
    if L.ls_oracle_mlp_f64(hidden, group_size, _ptr(x), _ptr(cache), _ptr(staging), _ptr(scales), _ptr(d),
                           len(d), _ptr(y)):
        raise ValueError("ls_oracle_mlp_f64 rejected its arguments")
    return y


def mlp_omp(hidden, group_size, x, cache, scales, descs, threads=0, staging=None):
    """OpenMP CPU baseline; returns y16."""
    L = lib()
    x = _u16(np.asarray(x, dtype=np.float16))
    scales = _u16(np.asarray(scales, dtype=np.float16).reshape(-1))
    cache = np.ascontiguousarray(cache, dtype=np.uint8)
    staging = cache if staging is None else np.ascontiguousarray(staging, dtype=np.uint8)
    d = np.ascontiguousarray(np.asarray(descs, dtype=np.uint32).reshape(-1, 5))
    y16 = np.zeros(hidden, dtype=np.uint16)
    if L.ls_oracle_mlp_omp(hidden, group_size, _ptr(x), _ptr(cache), _ptr(staging), _ptr(scales), _ptr(d),
                           len(d), _ptr(y16), int(threads)):
        raise ValueError("ls_oracle_mlp_omp rejected its arguments")
    return y16.view(np.float16)


def neuron(hidden, record, scale_row, x):
    L = lib()
    g, u, h = C.c_float(), C.c_float(), C.c_float()
    rec = np.ascontiguousarray(record, dtype=np.uint8)
    srow = _u16(np.asarray(scale_row, dtype=np.float16))
    xx = _u16(np.asarray(x, dtype=np.float16))
    if L.ls_oracle_neuron(hidden, _ptr(rec), _ptr(srow), _ptr(xx), C.byref(g), C.byref(u), C.byref(h)):
        raise ValueError("ls_oracle_neuron rejected its arguments")
    return g.value, u.value, h.value


def rmsnorm(x, weight=None, eps=1e-5):
    L = lib()
    xx = _u16(np.asarray(x, dtype=np.float16))
    w = None if weight is None else _u16(np.asarray(weight, dtype=np.float16))
    out = np.zeros(len(xx), dtype=np.uint16)
    L.ls_oracle_rmsnorm(len(xx), _ptr(xx), _ptr(w), eps, _ptr(out))
    return out.view(np.float16)


def residual(res, y):
    L = lib()
    r = _u16(np.asarray(res, dtype=np.float16))
    yy = _u16(np.asarray(y, dtype=np.float16))
    out = np.zeros(len(r), dtype=np.uint16)
    L.ls_oracle_residual(len(r), _ptr(r), _ptr(yy), _ptr(out))
    return out.view(np.float16)


def f2h(v: float) -> np.float16:
    return np.uint16(lib().ls_oracle_f2h(float(v))).view(np.float16)


def max_threads() -> int:
    return int(lib().ls_oracle_max_threads())


# ------------------------------------------------------------------ predictor
def predictor() -> C.CDLL:
    """The reference's own ls_create/ls_predict (predictor/predictor_cpu.cpp)."""
    global _predictor
    if _predictor is None:
        if not PREDICTOR_LIB.exists():
            if not REFERENCE_ROOT.exists():
                raise RuntimeError(f"{PREDICTOR_LIB} missing and the reference is not mounted to build it")
            build(reference=True)
        L = C.CDLL(str(PREDICTOR_LIB))
        L.ls_create.restype = C.c_void_p
        L.ls_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.ls_destroy.argtypes = [C.c_void_p]
        L.ls_available_cores.restype = C.c_int
        L.ls_predict.restype = C.c_int
        L.ls_predict.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_int,
                                 C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        _predictor = L
    return _predictor


def available_cores() -> int:
    return int(predictor().ls_available_cores())


class Predictor:
    """ls_create/ls_predict context. ls_create pins its OpenMP workers
    (predictor_cpu.cpp:132-139); the calling thread's affinity is restored."""

    def __init__(self, rows, stride, k, threads=1, precision=32):
        self.L = predictor()
        saved = os.sched_getaffinity(0)
        self.ctx = self.L.ls_create(rows, stride, k, threads, precision)
        os.sched_setaffinity(0, saved)
        if not self.ctx:
            raise ValueError("ls_create rejected its arguments")
        self.rows, self.stride, self.k = rows, stride, k

    def predict(self, weights, inputs, keep=None, skip=0, scales=None, input_scale=1.0, return_scores=False):
        w = np.ascontiguousarray(weights)
        x = np.ascontiguousarray(inputs)
        out = np.zeros(self.k, dtype=np.int32)
        keep_arr = None if keep is None else np.ascontiguousarray(keep, dtype=np.int32)
        sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
        scores = np.zeros(self.rows, dtype=np.float32) if return_scores else None
        rc = self.L.ls_predict(self.ctx, _ptr(w), _ptr(sc), _ptr(x), float(input_scale), _ptr(keep_arr),
                               0 if keep_arr is None else len(keep_arr), int(skip), _ptr(out), None, None,
                               _ptr(scores))
        if rc:
            raise ValueError(f"ls_predict returned {rc}")
        return (out, scores) if return_scores else out

    def close(self):
        if self.ctx:
            self.L.ls_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
