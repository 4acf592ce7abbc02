"""Index arithmetic of the batched union kernels (leanstream_b200/csrc/ls_batch.cu)
on CPU, bit for bit: the lane mappings that file states, restated here in
numpy, feed an emulated m16n8k16 MMA (A row-major 16x16, B 16x8, fragments as
the PTX ISA defines them for .f16 operands), and the products must equal the
plain matrix products of the dequantised weights.

Checked:
- the exact int4 -> fp16 conversion (nibble XOR 8 in the mantissa of 1024.0,
  minus 1032, times the scale) equals fp16(q * s) for every q and a spread of
  scales;
- gate/up: lane t of a quad holds coordinates c = 16t + 8w .. +7 of a
  64-coordinate block; MMA m of word w pairs coordinates c + 2m, c + 2m + 4
  (k 2t, 2t+1) and c + 2m + 1, c + 2m + 5 (k 2t+8, 2t+9); x is permuted into B
  with byte permutes 0x5410 / 0x7632; rows 0-7 gate, 8-15 up;
- down: lane group g holds columns 16g .. +15 of a 128-column half; the words
  of neurons (2t, 2t+1) and (2t+8, 2t+9) are interleaved by byte permutes so
  that nibbles i, i + 4 are one column of two neurons; tile T has row g =
  column 16g + 2T and row g + 8 = column 16g + 2T + 1.
No GPU is used; the CUDA source itself is checked by tests/test_gpu_batch.py."""
import numpy as np
import pytest


def byte_perm(x, y, s):
    b = [(x >> (8 * i)) & 0xFF for i in range(4)] + [(y >> (8 * i)) & 0xFF for i in range(4)]
    return sum(b[(s >> (4 * i)) & 7] << (8 * i) for i in range(4))


def u2h(v):
    return np.array([v & 0xFFFF, v >> 16], np.uint16).view(np.float16)


def h2u(a):
    a = np.asarray(a, np.float16).view(np.uint16).astype(np.uint64)
    return int(a[0]) | (int(a[1]) << 16)


def deq(w, i, s):
    """fp16(q * s) of nibbles i and i + 4 of the 32-bit word w."""
    biased = ((w >> (4 * i)) & 0x000F000F) ^ 0x64086408
    v = (u2h(biased) - np.float16(1032)).astype(np.float16)
    return h2u((v * np.asarray(s, np.float16)).astype(np.float16))


def mma(acc, A, B):
    """m16n8k16, fp32 accumulate: A[lane] = 4 regs, B[lane] = 2 regs."""
    Am = np.zeros((16, 16), np.float64)
    Bm = np.zeros((16, 8), np.float64)
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        a = [u2h(r).astype(np.float64) for r in A[lane]]
        Am[g, 2 * t:2 * t + 2], Am[g + 8, 2 * t:2 * t + 2] = a[0], a[1]
        Am[g, 2 * t + 8:2 * t + 10], Am[g + 8, 2 * t + 8:2 * t + 10] = a[2], a[3]
        b = [u2h(r).astype(np.float64) for r in B[lane]]
        Bm[2 * t:2 * t + 2, g], Bm[2 * t + 8:2 * t + 10, g] = b[0], b[1]
    D = Am @ Bm
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        acc[lane] += [D[g, 2 * t], D[g, 2 * t + 1], D[g + 8, 2 * t], D[g + 8, 2 * t + 1]]


def pack(q):
    """Signed nibbles, low nibble = even coordinate."""
    q = np.asarray(q) & 15
    return (q[0::2] | (q[1::2] << 4)).astype(np.uint8)


def word(b, off):
    return int(np.frombuffer(b[off:off + 4].tobytes(), np.uint32)[0])


def test_two_nibble_conversion_is_exact():
    scales = np.array([0.005, 0.0071, 0.0123, 0.02, 1.0, -0.013, 3.1e-5], np.float16)
    for s in scales:
        for q0 in range(-8, 8):
            for q4 in (-8, -1, 0, 7):
                w = ((q0 & 15) | ((q4 & 15) << 16))
                got = u2h(deq(w, 0, (s, s)))
                want = (np.array([q0, q4], np.float16) * s).astype(np.float16)
                assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), (q0, q4, s)


@pytest.mark.parametrize("seed", [0, 1])
def test_gateup_fragment_mapping(seed):
    rng = np.random.default_rng(seed)
    qg, qu = rng.integers(-8, 8, (8, 64)), rng.integers(-8, 8, (8, 64))
    sg, su = np.float16(0.011), np.float16(0.017)
    x = rng.standard_normal((8, 64)).astype(np.float16)
    gb, ub = [pack(r) for r in qg], [pack(r) for r in qu]
    acc = np.zeros((32, 4))
    for w in range(2):
        for m in range(2):
            A, B = [], []
            for lane in range(32):
                g, t = lane >> 2, lane & 3
                c = 16 * t + 8 * w
                gw, uw = word(gb[g], c // 2), word(ub[g], c // 2)
                X = [int(x[g, c + 2 * i:c + 2 * i + 2].view(np.uint32)[0]) for i in range(4)]
                xa, xb = (X[1], X[3]) if m else (X[0], X[2])
                B.append([byte_perm(xa, xb, 0x5410), byte_perm(xa, xb, 0x7632)])
                A.append([deq(gw, 2 * m, (sg, sg)), deq(uw, 2 * m, (su, su)), deq(gw, 2 * m + 1, (sg, sg)),
                          deq(uw, 2 * m + 1, (su, su))])
            mma(acc, A, B)
    wg = (qg.astype(np.float16) * sg).astype(np.float64)
    wu = (qu.astype(np.float16) * su).astype(np.float64)
    ref_g, ref_u = wg @ x.astype(np.float64).T, wu @ x.astype(np.float64).T  # [row][token]
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        for j in range(2):
            assert acc[lane, j] == pytest.approx(ref_g[g, 2 * t + j], abs=1e-9)
            assert acc[lane, 2 + j] == pytest.approx(ref_u[g, 2 * t + j], abs=1e-9)


@pytest.mark.parametrize("seed", [0, 1])
def test_down_fragment_mapping(seed):
    rng = np.random.default_rng(seed)
    qd = rng.integers(-8, 8, (16, 128))  # 16 neurons x one 128-column half
    sd = rng.uniform(0.005, 0.02, 16).astype(np.float16)
    h = rng.standard_normal((8, 16)).astype(np.float16)
    db = [pack(r) for r in qd]
    acc = np.zeros((8, 32, 4))
    lanes = []
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        nn = [2 * t, 2 * t + 1, 2 * t + 8, 2 * t + 9]
        wv = [(word(db[n], 8 * g), word(db[n], 8 * g + 4)) for n in nn]  # columns 16g .. +15
        b0 = int(h[g, 2 * t:2 * t + 2].view(np.uint32)[0])
        b1 = int(h[g, 2 * t + 8:2 * t + 10].view(np.uint32)[0])
        lanes.append((wv, [sd[n] for n in nn], b0, b1))
    for T in range(8):
        wi, T4 = T // 4, T % 4
        A, B = [], []
        for wv, s, b0, b1 in lanes:
            wa, wb, wc, wd = (wv[k][wi] for k in range(4))
            sel = 0x5410 if T4 < 2 else 0x7632
            z01, z23 = byte_perm(wa, wb, sel), byte_perm(wc, wd, sel)
            q = 2 * (T4 & 1)
            A.append([deq(z01, q, (s[0], s[1])), deq(z01, q + 1, (s[0], s[1])), deq(z23, q, (s[2], s[3])),
                      deq(z23, q + 1, (s[2], s[3]))])
            B.append([b0, b1])
        mma(acc[T], A, B)
    wd = (qd.astype(np.float16) * sd[:, None]).astype(np.float64)
    ref = h.astype(np.float64) @ wd  # [token][column]
    for T in range(8):
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            col = 16 * g + 2 * T
            for j in range(2):
                assert acc[T, lane, j] == pytest.approx(ref[2 * t + j, col], abs=1e-9)
                assert acc[T, lane, 2 + j] == pytest.approx(ref[2 * t + j, col + 1], abs=1e-9)
