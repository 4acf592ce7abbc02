/*
 * ls_oracle.c -- CPU ORACLE (test infrastructure only).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this file's library, and only as the checker or the timed CPU baseline.
 * The product (leanstream_b200/) never links, loads or calls it.
 *
 * It restates the reference's host-side math for the sparse INT4 SwiGLU MLP:
 *   examples/custom_pytorch/run.py:43-50 (reference())  -- the independent
 *     FP32 dequantisation/reduction with explicit FP16 rounding boundaries;
 *   backends/triton/core.py:10-17 (weight()) and :49-52  -- w = fp16(q*s),
 *     g,u -> fp16, SiLU -> fp16, h = fp16(s*u);
 *   kernels/streaming_mlp.cu:11-15,21-43                 -- same arithmetic,
 *     nibble decode (low nibble = even coordinate, q >= 8 -> q - 16);
 *   backends/triton/reduction.py:14-20                    -- y = fp16(sum),
 *     hidden = fp16(fp32(residual) + fp32(y));
 *   examples/ministral/native/predictor_shared_input.cu:16-33 -- HF RMSNorm:
 *     inv = rsqrt(sum(x^2)/H + eps), x' = fp16(w * fp16(x * inv)).
 * Sums are sequential fp32 in descriptor/neuron/coordinate order; a
 * compensated fp64 variant is provided as a cross-check of the fp32 order.
 * Pinned against the reference's closed forms (tests/persistent_mlp_test.cu
 * :52-56, tests/triton_smoke.py:74-77, examples/end_to_end/main.cu:75-79) and
 * against vectors produced by run.py's own reference() (tests/golden/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------ fp16 <-> fp32 */
/* IEEE binary16, round to nearest even (the rounding of __float2half_rn,
 * numpy float16 and torch .half()). */
uint16_t ls_oracle_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) return (uint16_t)(sign | (absx > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (absx < 0x38800000u) {                                      /* subnormal or zero in fp16 */
        if (absx < 0x33000000u) return (uint16_t)sign;             /* < 2^-25 -> +-0 */
        const uint32_t e = absx >> 23;
        const uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e; /* value = m * 2^(e-150); fp16 ulp = 2^-24 */
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 112u; /* rebias 127 -> 15 */
    uint32_t m = absx & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

float ls_oracle_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: normalise */
            int shift = 0;
            uint32_t mm = m;
            while (!(mm & 1024u)) { mm <<= 1; ++shift; }
            x = sign | ((uint32_t)(113 - shift) << 23) | ((mm & 1023u) << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline float r16(float v) { return ls_oracle_h2f(ls_oracle_f2h(v)); }

/* weight() of backends/triton/core.py:10-17 / streaming_mlp.cu:11-15. */
static inline float weight(const uint8_t* row, const uint16_t* scale_row, uint32_t c) {
    int q = (row[c / 2] >> ((c % 2) * 4)) & 15;
    if (q >= 8) q -= 16;
    return r16((float)q * ls_oracle_h2f(scale_row[c / 128]));
}

/* Descriptor as five uint32 (include/leanstream/types.h:16-20). */
typedef struct { uint32_t logical_group, physical_group, source_slot, dest_slot, source_kind; } oracle_desc;

/* h of one neuron (core.py:45-52). */
static float neuron_h(uint32_t H, const uint8_t* rec, const uint16_t* srow, const uint16_t* x, float* g_out,
                      float* u_out) {
    float g = 0.f, u = 0.f;
    for (uint32_t c = 0; c < H; ++c) {
        const float xv = ls_oracle_h2f(x[c]);
        g += weight(rec, srow, c) * xv;
        u += weight(rec + H / 2, srow + H / 128, c) * xv;
    }
    const float g16 = r16(g), u16 = r16(u);
    const float s = r16(g16 / (1.f + expf(-g16)));
    if (g_out) *g_out = g16;
    if (u_out) *u_out = u16;
    return r16(s * u16);
}

/*
 * Sparse MLP over `count` descriptors (core descriptors first, then queue
 * descriptors in their final order). Packed groups are slot-major with
 * group_bytes = G*3H/2; scales are fp16 [physical][G][3][H/128].
 * y32: fp32 sum (optional); y16: fp16 output (optional);
 * h_out: fp16 h at dest_slot*G+n (optional, core.py:53).
 * Returns 0, or -1 on invalid arguments.
 */
int ls_oracle_mlp(uint32_t H, uint32_t G, const uint16_t* x, const uint8_t* cache, const uint8_t* staging,
                  const uint16_t* scales, const void* descs, uint32_t count, float* y32, uint16_t* y16,
                  uint16_t* h_out) {
    if (!H || H % 256 || !G || !x || !scales || (count && !descs)) return -1;
    const oracle_desc* d = (const oracle_desc*)descs;
    const size_t rec = (size_t)3 * H / 2, gbytes = rec * G, srec = (size_t)3 * H / 128;
    float* acc = (float*)calloc(H, sizeof(float));
    if (!acc) return -1;
    for (uint32_t i = 0; i < count; ++i) {
        const uint8_t* base = (d[i].source_kind == 0 ? cache : staging);
        if (!base || d[i].source_kind > 1) { free(acc); return -1; }
        base += (size_t)d[i].source_slot * gbytes;
        for (uint32_t n = 0; n < G; ++n) {
            const uint8_t* r = base + n * rec;
            const uint16_t* s = scales + ((size_t)d[i].physical_group * G + n) * srec;
            const float h = neuron_h(H, r, s, x, NULL, NULL);
            if (h_out) h_out[(size_t)d[i].dest_slot * G + n] = ls_oracle_f2h(h);
            for (uint32_t c = 0; c < H; ++c) acc[c] += h * weight(r + H, s + 2 * H / 128, c);
        }
    }
    for (uint32_t c = 0; c < H; ++c) {
        if (y32) y32[c] = acc[c];
        if (y16) y16[c] = ls_oracle_f2h(acc[c]);
    }
    free(acc);
    return 0;
}

/* Same selection, down-projection summed in fp64 with Neumaier compensation
 * (cross-check of the fp32 sequential order; h keeps its fp16 boundaries). */
int ls_oracle_mlp_f64(uint32_t H, uint32_t G, const uint16_t* x, const uint8_t* cache, const uint8_t* staging,
                      const uint16_t* scales, const void* descs, uint32_t count, double* y64) {
    if (!H || H % 256 || !G || !x || !scales || !y64 || (count && !descs)) return -1;
    const oracle_desc* d = (const oracle_desc*)descs;
    const size_t rec = (size_t)3 * H / 2, gbytes = rec * G, srec = (size_t)3 * H / 128;
    double* comp = (double*)calloc(H, sizeof(double));
    if (!comp) return -1;
    for (uint32_t c = 0; c < H; ++c) y64[c] = 0.0;
    for (uint32_t i = 0; i < count; ++i) {
        const uint8_t* base = (d[i].source_kind == 0 ? cache : staging);
        if (!base) { free(comp); return -1; }
        base += (size_t)d[i].source_slot * gbytes;
        for (uint32_t n = 0; n < G; ++n) {
            const uint8_t* r = base + n * rec;
            const uint16_t* s = scales + ((size_t)d[i].physical_group * G + n) * srec;
            const double h = neuron_h(H, r, s, x, NULL, NULL);
            for (uint32_t c = 0; c < H; ++c) {
                const double v = h * (double)weight(r + H, s + 2 * H / 128, c);
                const double t = y64[c] + v;
                comp[c] += fabs(y64[c]) >= fabs(v) ? (y64[c] - t) + v : (v - t) + y64[c];
                y64[c] = t;
            }
        }
    }
    for (uint32_t c = 0; c < H; ++c) y64[c] += comp[c];
    free(comp);
    return 0;
}

/* Gate/up/h of one neuron, for white-box tests. */
int ls_oracle_neuron(uint32_t H, const uint8_t* record, const uint16_t* scale_row, const uint16_t* x, float* g16,
                     float* u16, float* h16) {
    if (!H || H % 256 || !record || !scale_row || !x) return -1;
    const float h = neuron_h(H, record, scale_row, x, g16, u16);
    if (h16) *h16 = h;
    return 0;
}

/* HF RMSNorm of predictor_shared_input.cu:16-33 (weight NULL = ones). */
int ls_oracle_rmsnorm(uint32_t H, const uint16_t* x, const uint16_t* w, float eps, uint16_t* out) {
    if (!H || !x || !out) return -1;
    float sum = 0.f;
    for (uint32_t c = 0; c < H; ++c) {
        const float v = ls_oracle_h2f(x[c]);
        sum += v * v;
    }
    const float inv = 1.f / sqrtf(sum / (float)H + eps);
    for (uint32_t c = 0; c < H; ++c) {
        const uint16_t n = ls_oracle_f2h(ls_oracle_h2f(x[c]) * inv);
        out[c] = w ? ls_oracle_f2h(ls_oracle_h2f(w[c]) * ls_oracle_h2f(n)) : n;
    }
    return 0;
}

/* hidden = fp16(fp32(residual) + fp32(y)) (reduction.py:17-20). */
int ls_oracle_residual(uint32_t H, const uint16_t* residual, const uint16_t* y, uint16_t* out) {
    if (!H || !residual || !y || !out) return -1;
    for (uint32_t c = 0; c < H; ++c) out[c] = ls_oracle_f2h(ls_oracle_h2f(residual[c]) + ls_oracle_h2f(y[c]));
    return 0;
}

/*
 * CPU baseline: the same MLP parallelised over descriptors with OpenMP,
 * each thread accumulating a private fp32 partial, partials reduced in
 * thread order. `threads` <= 0 uses the OpenMP default.
 */
int ls_oracle_mlp_omp(uint32_t H, uint32_t G, const uint16_t* x, const uint8_t* cache, const uint8_t* staging,
                      const uint16_t* scales, const void* descs, uint32_t count, uint16_t* y16, int threads) {
    if (!H || H % 256 || !G || !x || !scales || !y16 || (count && !descs)) return -1;
    const oracle_desc* d = (const oracle_desc*)descs;
    const size_t rec = (size_t)3 * H / 2, gbytes = rec * G, srec = (size_t)3 * H / 128;
    int nt = 1;
#ifdef _OPENMP
    nt = threads > 0 ? threads : omp_get_max_threads();
#endif
    float* part = (float*)calloc((size_t)nt * H, sizeof(float));
    if (!part) return -1;
    int bad = 0;
#ifdef _OPENMP
#pragma omp parallel num_threads(nt) reduction(| : bad)
#endif
    {
        int t = 0;
#ifdef _OPENMP
        t = omp_get_thread_num();
#endif
        float* acc = part + (size_t)t * H;
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t j = 0; j < (int64_t)count * G; ++j) {
            const uint32_t i = (uint32_t)(j / G), n = (uint32_t)(j % G);
            const uint8_t* base = (d[i].source_kind == 0 ? cache : staging);
            if (!base) { bad = 1; continue; }
            const uint8_t* r = base + (size_t)d[i].source_slot * gbytes + n * rec;
            const uint16_t* s = scales + ((size_t)d[i].physical_group * G + n) * srec;
            const float h = neuron_h(H, r, s, x, NULL, NULL);
            for (uint32_t c = 0; c < H; ++c) acc[c] += h * weight(r + H, s + 2 * H / 128, c);
        }
    }
    for (uint32_t c = 0; c < H; ++c) {
        float v = 0.f;
        for (int t = 0; t < nt; ++t) v += part[(size_t)t * H + c];
        y16[c] = ls_oracle_f2h(v);
    }
    free(part);
    return bad ? -1 : 0;
}

int ls_oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
