"""Pins the CPU oracle (oracle/ls_oracle.c) before it is trusted as the checker:
against the reference's closed forms, the outputs of the reference's own
host implementation (examples/custom_pytorch/run.py reference(), fixtures in
tests/golden/), and the reference predictor's known answers."""
import json
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def _half(z):
    return float(np.float16(z))


def _uniform_case(H, G, groups, byte, scale=0.05, x=0.1):
    cache = np.full(groups * G * 3 * H // 2, byte, np.uint8)
    scales = np.full(groups * G * 3 * H // 128, scale, np.float16)
    xs = np.full(H, x, np.float16)
    d = np.array([[i, i, i, i, 0] for i in range(groups)], np.uint32).reshape(-1, 5)
    return cache, scales, xs, d


@pytest.mark.parametrize("q,byte", [(1, 0x11), (-1, 0xFF)])
@pytest.mark.parametrize("count", [0, 1, 2, 16, 37])
def test_persistent_mlp_closed_form(count, q, byte):
    """tests/persistent_mlp_test.cu:15-16,52-56 (H=256, G=2, 1 core + count)."""
    H, G = 256, 2
    groups = count + 1
    cache, scales, x, d = _uniform_case(H, G, groups, byte)
    y16, _, _ = O.mlp(H, G, x, cache, scales, d)
    gate = _half(H * _half(0.1) * _half(0.05) * q)
    act = _half(_half(gate / (1 + math.exp(-gate))) * gate)
    expected = _half(groups * G * act * _half(0.05) * q)
    assert np.all(np.abs(y16.astype(np.float32) - expected) < 0.002)


def test_triton_smoke_closed_form():
    """tests/triton_smoke.py:19,74-77: H=256, G=2, CORE 2 + TOTAL 4."""
    H, G, CORE, TOTAL = 256, 2, 2, 4
    cache, scales, x, _ = _uniform_case(H, G, CORE + TOTAL, 0x11)
    d = np.array([[i, i, i, i, 0] for i in range(CORE + TOTAL)], np.uint32)
    y16, _, _ = O.mlp(H, G, x, cache, scales, d)
    gate = _half(H * _half(0.1) * _half(0.05))
    silu = _half(gate / (1 + math.exp(-gate)))
    expected = _half((CORE + TOTAL) * G * _half(silu * gate) * _half(0.05))
    assert np.all(np.abs(y16.astype(np.float32) - expected) <= 0.002)


def test_end_to_end_closed_form():
    """examples/end_to_end/main.cu:42,75-79: H=512, G=2, 4 final groups, tol .005."""
    H, G = 512, 2
    cache, scales, x, _ = _uniform_case(H, G, 8, 0x11)
    final = [0, 6, 2, 4]
    d = np.array([[g, g, g, i, 0] for i, g in enumerate(final)], np.uint32)
    y16, _, _ = O.mlp(H, G, x, cache, scales, d)
    gate = _half(H * _half(0.1) * _half(0.05))
    silu = _half(gate / (1 + math.exp(-gate)))
    expected = _half(4 * G * _half(silu * gate) * _half(0.05))
    assert np.all(np.abs(y16.astype(np.float32) - expected) < 0.005)


def test_custom_triton_gate_value():
    """docs/custom_triton.md:26: H=512, q=1, scale .05, x=.1 -> gate ~ 2.56."""
    H = 512
    rec = np.full(3 * H // 2, 0x11, np.uint8)
    srow = np.full(3 * H // 128, 0.05, np.float16)
    g, u, h = O.neuron(H, rec, srow, np.full(H, 0.1, np.float16))
    assert abs(g - 2.56) < 0.01 and g == u
    assert h == _half(_half(g / (1 + math.exp(-g))) * u)


@pytest.mark.parametrize("case", ["toy_mult1", "toy_mult2", "full_range", "negative_heavy"])
def test_reference_host_vectors(case):
    """Oracle == examples/custom_pytorch/run.py reference() on the same inputs.
    The multiplier of run.py scales decoded weights after fp16 rounding; a
    power-of-two multiplier equals the same multiple of the fp16 scale."""
    from leanstream_b200.synthetic import pack_int4

    z = np.load(GOLDEN / "reference_mlp.npz")
    q, x, sel, mult, y = (z[f"{case}/{k}"] for k in ("q", "x", "selected", "multiplier", "y"))
    H, G = 512, 2
    packed = pack_int4(q).reshape(-1)  # [8 groups][2 neurons][3][H/2], slot = logical
    scales = np.full(8 * G * 3 * H // 128, np.float16(0.05) * np.float16(mult), np.float16)
    d = np.array([[g, g, g, i, 0] for i, g in enumerate(sel)], np.uint32)
    y16, _, _ = O.mlp(H, G, x, packed, scales, d)
    ref = y.astype(np.float32)
    assert np.abs(y16.astype(np.float32) - ref).max() <= 0.002  # run.py:76 tolerance
    # the two fp32 summation orders agree to within one fp16 ulp everywhere
    ulp = np.spacing(np.abs(y.astype(np.float16))).astype(np.float32)
    assert np.all(np.abs(y16.astype(np.float32) - ref) <= ulp)


def test_fp64_cross_check_of_sum_order():
    from leanstream_b200.synthetic import descriptors, make_layer

    L = make_layer(4, 1024, 12, 64)
    d = descriptors([1, 5, 7, 11])
    _, y32, _ = O.mlp(1024, 64, L.x, L.packed, L.scales, d)
    y64 = O.mlp_f64(1024, 64, L.x, L.packed, L.scales, d)
    assert np.abs(y32 - y64).max() <= 1e-4 * np.abs(y64).max()


def test_omp_baseline_matches_oracle():
    from leanstream_b200.synthetic import descriptors, make_layer

    L = make_layer(6, 1024, 16, 64)
    d = descriptors([3, 1, 4, 15, 9])
    y16, _, _ = O.mlp(1024, 64, L.x, L.packed, L.scales, d)
    yomp = O.mlp_omp(1024, 64, L.x, L.packed, L.scales, d, threads=4)
    assert np.abs(y16.astype(np.float32) - yomp.astype(np.float32)).max() <= 2e-3 * np.abs(y16).max()


def test_fp16_conversion_exhaustive():
    lib = O.lib()
    halves = np.arange(65536, dtype=np.uint16)
    finite = np.isfinite(halves.view(np.float16))
    back = np.array([lib.ls_oracle_h2f(int(h)) for h in halves[finite]], np.float32)
    assert np.array_equal(back, halves[finite].view(np.float16).astype(np.float32))
    r = np.random.default_rng(0).standard_normal(20000).astype(np.float32) * np.float32(300)
    r = np.concatenate([r, np.float32([65504, 65519.9, 65520, 1e-8, 6e-8, 3e-5, -0.0])])
    ours = np.array([lib.ls_oracle_f2h(float(v)) for v in r], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(ours, r.astype(np.float16).view(np.uint16))


def test_rmsnorm_hf_rounding():
    x = (np.random.default_rng(2).standard_normal(4096) * 13).astype(np.float16)
    w = np.random.default_rng(3).uniform(0.5, 1.5, 4096).astype(np.float16)
    got = O.rmsnorm(x, w, 1e-5).astype(np.float32)
    xf = x.astype(np.float32)
    inv = np.float32(1) / np.sqrt(np.float32((xf * xf).sum(dtype=np.float32)) / np.float32(4096) + np.float32(1e-5))
    ref = (w.astype(np.float32) * (xf * inv).astype(np.float16).astype(np.float32)).astype(np.float16)
    assert np.abs(got - ref.astype(np.float32)).max() <= np.spacing(np.abs(ref)).max()


def test_predictor_known_answer():
    """examples/predictor/main.cpp:5-12: 4 rows -> IDs 3, 2."""
    p = O.Predictor(4, 32, 2, 1, 32)
    w = np.zeros((4, 2, 32), np.float32)
    for r in range(4):
        w[r] = (r + 1) / 32
    assert p.predict(w, np.ones(32, np.float32)).tolist() == [3, 2]
    p.close()


def test_predictor_order_and_exclusions():
    """predictor_cpu.cpp:152-201: score desc, ties by ascending ID; keep+skip."""
    p = O.Predictor(6, 32, 3, 1, 32)
    w = np.zeros((6, 2, 32), np.float32)
    for r, v in enumerate([1, 3, 3, 2, 3, 0.5]):
        w[r] = v / 32
    ids = p.predict(w, np.ones(32, np.float32))
    assert ids.tolist() == [1, 2, 4]
    ids = p.predict(w, np.ones(32, np.float32), keep=np.array([2], np.int32), skip=1)
    assert ids.tolist() == [1, 4, 3]
    p.close()


def test_config1_selection_golden():
    """Config 1 (seed 0): the generator reproduces the fixture's inputs and the
    reference ls_predict reproduces the committed IDs; the oracle y too."""
    import hashlib

    from leanstream_b200.synthetic import descriptors, make_layer, representative_rows

    g = json.loads((GOLDEN / "config1.json").read_text())
    L = make_layer(g["seed"], g["hidden"], g["groups"], g["group_size"])
    digest = hashlib.sha256(L.packed.tobytes() + L.scales.tobytes() + L.x.tobytes()).hexdigest()
    assert digest == g["input_sha256"]
    p = O.Predictor(64, 1024, 16, 1, 32)
    ids = p.predict(representative_rows(L), L.x.astype(np.float32))
    p.close()
    assert ids.tolist() == g["ids"]
    y16, _, _ = O.mlp(1024, 64, L.x, L.packed, L.scales, descriptors(ids))
    assert y16.view(np.uint16).tobytes().hex() == g["y_oracle_f16_hex"]
