// Batched decode over the union of the tokens' active groups (up to 8
// tokens): every weight byte of the union is read once for all tokens, and
// the tokens form the N dimension of the tensor-core MMAs. A per-token mask
// restricts token b to its own active groups (its h is zero elsewhere), so
// each token's result is the batch-1 MLP over its own set; without a mask
// every token uses the whole union.
//
// Arithmetic of the reference path (backends/triton/core.py:17,49-52,
// reduction.py:15): w = fp16(q * s), g and u fp32 sums rounded to fp16,
// s = fp16(silu(g)), h = fp16(s * u), down partials in fp32, y rounded once.
//
// Exact int4 -> fp16: a signed nibble u (q = u as two's complement) XOR 8 is
// q + 8 in [0, 15]; placed in the mantissa of 1024.0 (exponent field 0x64,
// where the fp16 step is 1) it reads 1024 + q + 8, and subtracting 1032 gives
// q exactly. One mask-and-xor of a 32-bit word yields nibbles i and i + 4 as
// the two halves of a half2, so the MMA's K (gate/up) or M (down) order is
// chosen to pair coordinates i and i + 4 of each 8-coordinate word. The
// product with the scale is then the one fp16 rounding of q * s.
//
// Two implementations of the same arithmetic. The default runs the union
// GEMMs on the 5th-generation tensor cores (tcgen05.mma, accumulators in
// tensor memory; the "tcgen05" section below, four launches per call). The
// warp-level MMA kernels described next stay behind LS_B200_BATCH_MMA_SYNC
// for comparison.
//
// Warp-level MMA kernels: three, each with a fixed summation order
// (deterministic). The two weight kernels stream their rows through a
// 4-stage shared-memory ring filled with cp.async (completion by
// cp.async.wait_group: no spin loop), so three stages of loads are in flight
// while one is multiplied.
//   gate/up  -- one CTA per 16 union neurons (two octets), 8 warps splitting
//               each 1024-coordinate stage in 64-coordinate blocks, two
//               blocks per warp. A rows 0-7 are the octet's gate rows, 8-15
//               its up rows; B columns are the tokens (x read from L2), shared
//               by both octets. Lane t of a quad holds coordinates
//               c = 64kb + 16t + 8w .. +7 (w = 0, 1); MMA m of a word takes
//               k 2t, 2t+1 = coordinates c + 2m, c + 2m + 4 and k 2t+8, 2t+9 =
//               c + 2m + 1, c + 2m + 5. h is stored token-major.
//   down     -- one CTA per 256 output columns (128 contiguous bytes of each
//               down row) and thirteenth of the union's neurons; each stage
//               holds four 16-neuron units with their scales and h. Warp
//               (unit slot, half) computes 128 columns: A rows are output
//               columns, K the neurons, B = h (neurons x tokens). Lane group g
//               holds columns 16g .. +15 of the half; in tile T row g is
//               column 16g + 2T and row g + 8 column 16g + 2T + 1.
//   epilogue -- y = sum of the splits in split order, fp16 rounding, the
//               optional residual.
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>
#include <cerrno>

#include "ls_internal.h"

namespace lsb {
namespace {

constexpr int kBatchTokens = 8;
constexpr int kBatchThreads = 256;  // 8 warps
constexpr int kOctets = 2;  // gate/up octets per CTA, sharing each x fragment
constexpr uint32_t kGateUpNeurons = 8 * kOctets;
constexpr uint32_t kDownCols = 256;
constexpr uint32_t kDownSplits = 13;

struct BatchParams {
    uint32_t H, G, U, B, NT, NTP;  // NT union neurons, NTP padded row length of hT
    const __half* x;
    __half* y;
    float* y32;
    const __half* residual;
    __half* hidden_out;
    const uint8_t* cache;
    const uint8_t* staging;
    const __half* scales;
    const ls_exec_desc* desc;
    const uint8_t* mask;
    __half* hT;      // [8][NTP] h, token-major (warp-MMA path)
    float* partial;  // [dn_splits][B][H]
    // tensor-core path
    const uint8_t* ximg;  // x image [H / 8][8 tokens][8] fp16, K-major core matrices
    float* gpart;         // gate/up split sums [gu_splits][rows_total][8]
    uint32_t* gcnt;       // [tiles][4] stored splits per gate/up tile and lane quarter
    __half* hB;           // h image [NT64 / 8][8 tokens][8] fp16
    uint32_t gu_splits, dn_splits, rows_total;
    uint64_t timeout_ns;  // bound of the tensor-core kernels' waits
};

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 u2h(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// fp16(q * s) of nibbles i and i + 4 of w (low and high half)
__device__ __forceinline__ uint32_t deq(uint32_t w, int i, __half2 s) {
    const uint32_t biased = ((w >> (4 * i)) & 0x000F000Fu) ^ 0x64086408u;  // 1024 + q + 8
    return h2u(__hmul2(__hsub2(u2h(biased), __float2half2_rn(1032.f)), s));
}

struct Row {
    const uint8_t* src;  // neuron record [gate H/2 | up H/2 | down H/2]
    const __half* sc;    // its scales [3][H/128]
};

__device__ __forceinline__ Row neuron_row(const BatchParams& p, uint32_t n) {
    const uint32_t u = n / p.G, nl = n % p.G;
    const ls_exec_desc d = p.desc[u];
    const uint8_t* base = d.source_kind == LS_SOURCE_STAGING ? p.staging : p.cache;
    Row r;
    r.src = base + size_t(d.source_slot) * p.G * (3 * p.H / 2) + size_t(nl) * (3 * p.H / 2);
    r.sc = p.scales + (size_t(d.physical_group) * p.G + nl) * 3 * (p.H / 128);
    return r;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Gate/up stage: 16 blocks of 64 coordinates = 512 B of each of the CTA's
// 16 * kOctets rows (row 16o + 8gu + g: octet o, gate (gu 0) or up (gu 1),
// neuron g), at a 544-B row stride so that a warp's 8-row fragment load takes
// the minimum two shared-memory wavefronts.
constexpr uint32_t kGuStageBlocks = 16;
constexpr uint32_t kGuRowBytes = kGuStageBlocks * 32;
constexpr uint32_t kGuRowStride = kGuRowBytes + 32;
constexpr uint32_t kGuRows = 16 * kOctets;
constexpr uint32_t kGuStageBytes = kGuRows * kGuRowStride;
constexpr int kGuStages = 4;
constexpr uint32_t kGuSmem = kGuStages * kGuStageBytes;
static_assert(8 * 4 * kOctets * 32 * sizeof(float) <= kGuSmem, "reduction fits the ring");

__global__ void __launch_bounds__(kBatchThreads) batch_gateup_kernel(const BatchParams p) {
    extern __shared__ __align__(16) uint8_t gu_ring[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t n_base = blockIdx.x * kGateUpNeurons;
    const uint32_t half_bytes = p.H / 2, KB = p.H / 64;
    // copy role: 16-B chunk `lane` of the gate and up rows of neuron n_base + 8o + warp
    const uint8_t* csrc[kOctets];
#pragma unroll
    for (int o = 0; o < kOctets; ++o) {
        const uint32_t n = n_base + 8 * o + warp;
        csrc[o] = n < p.NT ? neuron_row(p, n).src : nullptr;
    }
    // compute role: gate row g, up row g + 8 of octet o = neuron n_base + 8o + g
    bool valid[kOctets];
    const __half* sc[kOctets];
#pragma unroll
    for (int o = 0; o < kOctets; ++o) {
        const uint32_t n = n_base + 8 * o + g;
        valid[o] = n < p.NT;
        sc[o] = valid[o] ? neuron_row(p, n).sc : nullptr;
    }
    const bool tok = uint32_t(g) < p.B;  // this lane's B column (token g)
    const __half* xrow = p.x + size_t(g) * p.H + 16 * t;
    const uint32_t nst = (half_bytes + kGuRowBytes - 1) / kGuRowBytes;

    auto issue = [&](uint32_t s) {
        uint8_t* buf = gu_ring + (s % kGuStages) * kGuStageBytes;
        const uint32_t off = s * kGuRowBytes + 16 * lane;
        if (off >= half_bytes) return;
#pragma unroll
        for (int o = 0; o < kOctets; ++o) {
            if (!csrc[o]) continue;
            cp_async16(buf + (16 * o + warp) * kGuRowStride + 16 * lane, csrc[o] + off);
            cp_async16(buf + (16 * o + 8 + warp) * kGuRowStride + 16 * lane, csrc[o] + half_bytes + off);
        }
    };

    float acc[kOctets][4];
#pragma unroll
    for (int o = 0; o < kOctets; ++o) acc[o][0] = acc[o][1] = acc[o][2] = acc[o][3] = 0.f;
#pragma unroll
    for (int s = 0; s < kGuStages - 1; ++s) {
        if (uint32_t(s) < nst) issue(s);
        cp_async_commit();
    }
    for (uint32_t s = 0; s < nst; ++s) {
        const uint32_t blocks = min(kGuStageBlocks, KB - s * kGuStageBlocks);
        // this warp's blocks warp and warp + 8 of the stage: x and scales
        // (L2-resident) are requested before waiting for the stage
        __half2 sg[2][kOctets], su[2][kOctets];
        uint4 xv[2][2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t kbl = warp + 8 * j, kb = s * kGuStageBlocks + kbl;
            const bool inb = kbl < blocks;
#pragma unroll
            for (int o = 0; o < kOctets; ++o) {
                sg[j][o] = su[j][o] = __float2half2_rn(0.f);
                if (inb && valid[o]) {
                    sg[j][o] = __half2half2(sc[o][kb / 2]);
                    su[j][o] = __half2half2(sc[o][p.H / 128 + kb / 2]);
                }
            }
            xv[j][0] = xv[j][1] = make_uint4(0u, 0u, 0u, 0u);
            if (inb && tok) {
                const uint4* xp = reinterpret_cast<const uint4*>(xrow + kb * 64);
                xv[j][0] = xp[0];
                xv[j][1] = xp[1];
            }
        }
        cp_async_wait<kGuStages - 2>();
        __syncthreads();  // stage s visible; every warp is done with stage s - 1
        if (s + kGuStages - 1 < nst) issue(s + kGuStages - 1);
        cp_async_commit();
        const uint8_t* buf = gu_ring + (s % kGuStages) * kGuStageBytes;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t kbl = warp + 8 * j;
            if (kbl >= blocks) continue;  // warp-uniform
            uint2 wg[kOctets], wu[kOctets];
#pragma unroll
            for (int o = 0; o < kOctets; ++o) {
                wg[o] = wu[o] = make_uint2(0u, 0u);
                if (valid[o]) {
                    wg[o] = *reinterpret_cast<const uint2*>(buf + (16 * o + g) * kGuRowStride + kbl * 32 + 8 * t);
                    wu[o] = *reinterpret_cast<const uint2*>(buf + (16 * o + 8 + g) * kGuRowStride + kbl * 32 + 8 * t);
                }
            }
#pragma unroll
            for (int w = 0; w < 2; ++w) {
                const uint4 X = xv[j][w];  // x[c .. c+7] as (c, c+1) (c+2, c+3) (c+4, c+5) (c+6, c+7)
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    const uint32_t xa = m ? X.y : X.x, xb = m ? X.w : X.z;
                    const uint32_t b0 = __byte_perm(xa, xb, 0x5410);  // x[c + 2m], x[c + 2m + 4]
                    const uint32_t b1 = __byte_perm(xa, xb, 0x7632);  // x[c + 2m + 1], x[c + 2m + 5]
#pragma unroll
                    for (int o = 0; o < kOctets; ++o) {
                        const uint32_t gw = w ? wg[o].y : wg[o].x, uw = w ? wu[o].y : wu[o].x;
                        mma_f16(acc[o], deq(gw, 2 * m, sg[j][o]), deq(uw, 2 * m, su[j][o]),
                                deq(gw, 2 * m + 1, sg[j][o]), deq(uw, 2 * m + 1, su[j][o]), b0, b1);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // the ring is free: reuse it for the cross-warp sums
    float (*red)[4 * kOctets][32] = reinterpret_cast<float (*)[4 * kOctets][32]>(gu_ring);  // [warp][4o + d][lane]
#pragma unroll
    for (int o = 0; o < kOctets; ++o)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][4 * o + e][lane] = acc[o][e];
    __syncthreads();
    if (warp >= kOctets) return;
    const int o = warp;  // warp o finishes octet o
    float gs[2] = {0.f, 0.f}, us[2] = {0.f, 0.f};
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        gs[0] += red[w][4 * o + 0][lane];
        gs[1] += red[w][4 * o + 1][lane];
        us[0] += red[w][4 * o + 2][lane];
        us[1] += red[w][4 * o + 3][lane];
    }
    const uint32_t nrow = n_base + 8 * o + g;
    if (nrow >= p.NT) return;
    const uint32_t u = nrow / p.G;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint32_t b = 2 * t + j;  // token of D column 2t + j
        if (b >= p.B) continue;
        const float g16 = __half2float(__float2half_rn(gs[j])), u16 = __half2float(__float2half_rn(us[j]));
        const float sl = __half2float(__float2half_rn(g16 / (1.f + expf(-g16))));
        __half h = __float2half_rn(sl * u16);
        if (p.mask && !p.mask[size_t(b) * p.U + u]) h = __float2half_rn(0.f);
        p.hT[size_t(b) * p.NTP + nrow] = h;
    }
}

// one 16-neuron unit's down inputs of a lane: neurons 2t, 2t+1, 2t+8, 2t+9
struct DownIn {
    uint2 w[4];       // 16 columns of the lane's column group
    __half s[4];      // their down scale (one 128-column block)
    uint32_t b0, b1;  // h of token g: neurons (2t, 2t+1), (2t+8, 2t+9)
};

__device__ __forceinline__ void down_mma(float (&acc)[8][4], const DownIn& v) {
    const __half2 s01 = __halves2half2(v.s[0], v.s[1]), s23 = __halves2half2(v.s[2], v.s[3]);
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
        // neuron pairs interleaved per byte pair: nibbles i, i + 4 = the same
        // column of neurons 2t and 2t+1 (resp. 2t+8, 2t+9)
        const uint32_t wa = wi ? v.w[0].y : v.w[0].x, wb = wi ? v.w[1].y : v.w[1].x;
        const uint32_t wc = wi ? v.w[2].y : v.w[2].x, wd = wi ? v.w[3].y : v.w[3].x;
        const uint32_t zlo01 = __byte_perm(wa, wb, 0x5410), zhi01 = __byte_perm(wa, wb, 0x7632);
        const uint32_t zlo23 = __byte_perm(wc, wd, 0x5410), zhi23 = __byte_perm(wc, wd, 0x7632);
#pragma unroll
        for (int T4 = 0; T4 < 4; ++T4) {  // tile T = 4wi + T4: columns 8wi + 2T4, +1 of the lane's 16
            const uint32_t z01 = T4 < 2 ? zlo01 : zhi01, z23 = T4 < 2 ? zlo23 : zhi23;
            const int q = 2 * (T4 & 1);
            mma_f16(acc[4 * wi + T4], deq(z01, q, s01), deq(z01, q + 1, s01), deq(z23, q, s23),
                    deq(z23, q + 1, s23), v.b0, v.b1);
        }
    }
}

// Down stage: kDnUnits 16-neuron units, one per warp pair. Per neuron the
// CTA's 256 columns are 128 contiguous bytes of its down row (stride 144 B:
// a warp's four-neuron fragment load takes the minimum two wavefronts), its
// two down scales (one per 128-column half) and, per unit, h of the 8 tokens.
constexpr uint32_t kDnUnits = 4;
constexpr uint32_t kDnNeuronStride = 144;
constexpr uint32_t kDnW = kDnUnits * 16 * kDnNeuronStride;
constexpr uint32_t kDnS = kDnUnits * 16 * 2 * sizeof(__half);
constexpr uint32_t kDnHT = kDnUnits * kBatchTokens * 16 * sizeof(__half);
constexpr uint32_t kDnStageBytes = kDnW + kDnS + kDnHT;
constexpr int kDnStages = 6;
constexpr uint32_t kDnSmem = kDnStages * kDnStageBytes;
static_assert(kDnW % 16 == 0 && kDnS % 16 == 0 && kDnStageBytes % 16 == 0, "16-B aligned stage parts");
static_assert(kDnUnits * 2 * 32 * 32 * sizeof(float) <= kDnSmem, "reduction fits the ring");

// one stage's unit `un` (slot nw) for the lane's 128-column half ch
__device__ __forceinline__ void down_unit(float (&acc)[8][4], const BatchParams& p, const uint8_t* buf, uint32_t un,
                                          int nw, int ch, int g, int t, bool tok) {
    const uint32_t n0 = un * 16;
    const uint32_t kk[4] = {2u * t, 2u * t + 1, 2u * t + 8, 2u * t + 9};
    DownIn v;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        v.w[q] = make_uint2(0u, 0u);
        v.s[q] = __float2half_rn(0.f);
        if (n0 + kk[q] < p.NT) {  // never-copied slots stay zero here
            const uint32_t slot = nw * 16 + kk[q];
            v.w[q] = *reinterpret_cast<const uint2*>(buf + slot * kDnNeuronStride + 64 * ch + 8 * g);
            v.s[q] = reinterpret_cast<const __half*>(buf + kDnW)[2 * slot + ch];
        }
    }
    v.b0 = v.b1 = 0u;
    if (tok) {
        // h of neurons past the union is never written: zero it (a zero
        // weight times a stale NaN pattern would still poison the sum)
        const uint32_t* hb = reinterpret_cast<const uint32_t*>(buf + kDnW + kDnS + (nw * kBatchTokens + g) * 32);
        if (n0 + kk[0] < p.NT) v.b0 = hb[t];      // neurons 2t, 2t+1
        if (n0 + kk[2] < p.NT) v.b1 = hb[t + 4];  // neurons 2t+8, 2t+9
        if (n0 + kk[1] >= p.NT) v.b0 &= 0xffffu;
        if (n0 + kk[3] >= p.NT) v.b1 &= 0xffffu;
    }
    down_mma(acc, v);
}

__global__ void __launch_bounds__(kBatchThreads) batch_down_kernel(const BatchParams p) {
    extern __shared__ __align__(16) uint8_t dn_ring[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int nw = warp >> 1, ch = warp & 1;  // unit slot of the stage, 128-column half
    const uint32_t c0 = blockIdx.x * kDownCols, split = blockIdx.y;
    const uint32_t units = (p.NT + 15) / 16;
    const uint32_t u_begin = uint32_t(uint64_t(units) * split / kDownSplits);
    const uint32_t u_end = uint32_t(uint64_t(units) * (split + 1) / kDownSplits);
    const uint32_t nst = (u_end - u_begin + kDnUnits - 1) / kDnUnits;
    const bool tok = uint32_t(g) < p.B;

    auto issue = [&](uint32_t s) {
        uint8_t* buf = dn_ring + (s % kDnStages) * kDnStageBytes;
        const uint32_t u0 = u_begin + s * kDnUnits;
#pragma unroll
        for (int m = 0; m < 2; ++m) {  // 2 x 256 chunks: unit, neuron, 16-B part
            const uint32_t c = threadIdx.x + 256 * m, us = c >> 7, k = (c >> 3) & 15, j = c & 7;
            const uint32_t un = u0 + us, n = un * 16 + k;
            if (un >= u_end || n >= p.NT) continue;
            const Row r = neuron_row(p, n);
            cp_async16(buf + (us * 16 + k) * kDnNeuronStride + 16 * j, r.src + p.H + c0 / 2 + 16 * j);
            if (j == 0) cp_async4(buf + kDnW + (us * 16 + k) * 4, r.sc + 2 * (p.H / 128) + c0 / 128);
        }
        if (threadIdx.x < kDnUnits * kBatchTokens * 2) {  // h: unit, token, 8-neuron half
            const uint32_t us = threadIdx.x >> 4, b = (threadIdx.x >> 1) & 7, hf = threadIdx.x & 1;
            const uint32_t un = u0 + us;
            if (un < u_end && b < p.B)
                cp_async16(buf + kDnW + kDnS + (us * kBatchTokens + b) * 32 + 16 * hf,
                           p.hT + size_t(b) * p.NTP + un * 16 + 8 * hf);
        }
    };

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
    for (int s = 0; s < kDnStages - 1; ++s) {
        if (uint32_t(s) < nst) issue(s);
        cp_async_commit();
    }
    for (uint32_t s = 0; s < nst; ++s) {
        cp_async_wait<kDnStages - 2>();
        __syncthreads();  // stage s visible; every warp is done with stage s - 1
        const uint32_t un = u_begin + s * kDnUnits + nw;
        if (un < u_end) down_unit(acc, p, dn_ring + (s % kDnStages) * kDnStageBytes, un, nw, ch, g, t, tok);
        // refill the buffer of stage s - 1 after the MMAs: its descriptor
        // loads then do not delay this stage's compute
        if (s + kDnStages - 1 < nst) issue(s + kDnStages - 1);
        cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();  // the ring is free: reuse it for the cross-warp sums
    float (*red)[2][32][32] = reinterpret_cast<float (*)[2][32][32]>(dn_ring);  // [nw][ch][4T + d][lane]
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[nw][ch][4 * i + e][lane] = acc[i][e];
    __syncthreads();
    // warp (pair, ch) sums tiles 2 pair, 2 pair + 1 of half ch over the unit slots in order
    float* out = p.partial + size_t(split) * p.B * p.H;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int T = 2 * nw + i;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (uint32_t w = 0; w < kDnUnits; ++w)
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] += red[w][ch][4 * T + e][lane];
        const uint32_t col = c0 + 128 * ch + 16 * g + 2 * T;  // row g; row g+8 is col + 1
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t b = 2 * t + j;
            if (b >= p.B) continue;
            *reinterpret_cast<float2*>(out + size_t(b) * p.H + col) = make_float2(v[j], v[2 + j]);
        }
    }
}

__global__ void batch_epilogue_kernel(const BatchParams p) {
    const uint32_t total = p.B * p.H;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        float y = 0.f;
        for (uint32_t s = 0; s < p.dn_splits; ++s) y += p.partial[size_t(s) * total + i];
        const __half y16 = __float2half_rn(y);
        if (p.y32) p.y32[i] = y;
        if (p.y) p.y[i] = y16;
        if (p.hidden_out) p.hidden_out[i] = __float2half_rn(__half2float(p.residual[i]) + __half2float(y16));
    }
}

// Optional prologue (LS_B200_NORM_INPUT): the HF RMSNorm of every token,
// one CTA per token, as the batch-1 kernel's stage_x applies it
// (examples/ministral/native/predictor_shared_input.cu:16-33):
// inv = rsqrt(sum(x^2) / H + eps), x' = fp16(w * fp16(x * inv)) (w = 1 when
// no weight is given). The sum of squares runs in a fixed order (per thread
// strided, then a shuffle tree, then the warps in order), so two calls give
// identical bits. x' goes to the scratch row of the token, which the gate/up
// kernel reads in place of x.
__global__ void __launch_bounds__(256) batch_norm_kernel(const __half* x, const __half* w, float eps, uint32_t H,
                                                         __half* xn) {
    __shared__ float part[8];
    const __half* row = x + size_t(blockIdx.x) * H;
    __half* out = xn + size_t(blockIdx.x) * H;
    float ss = 0.f;
    for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) {
        const float v = __half2float(row[c]);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += part[i];
    const float inv = rsqrtf(tot / float(H) + eps);
    for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) {
        __half v = __float2half_rn(__half2float(row[c]) * inv);
        if (w) v = __hmul(w[c], v);
        out[c] = v;
    }
}

// ------------------------------------------------------------------ tcgen05
// The union GEMMs on the 5th-generation tensor cores. Both kernels are
// warp-specialised: a producer warp streams the raw int4 rows of the union
// into a shared-memory ring with cp.async.bulk (completion on mbarriers),
// eight converter warps turn them into w = fp16(q * s) (deq, the exact
// conversion above), and one thread issues tcgen05.mma with the fp32
// accumulator in tensor memory; tcgen05.commit releases every buffer an MMA
// has read. Per 16-coordinate (gate/up) or 16-neuron (down) step the tensor
// core does what 8 to 16 warp-level MMAs did, so the converter warps spend
// their issue slots on the conversion alone, and the ring keeps several
// stages of HBM reads in flight per SM.
//
// gate/up (batch_gateup_tc_kernel): CTA = tile of 64 union neurons (128 A
// rows: row 2j the gate row, 2j + 1 the up row of neuron j) x one of S
// splits of the hidden dimension. A lives in TENSOR memory: each converter
// thread owns one row (tcgen05.st.32x32b, lane = row), so the fp16 weights
// never pass through shared memory. B is the stage's slice of the x image
// (batch_ximg_kernel: 8 tokens, K-major core matrices, one 4 KB bulk copy
// per stage). The form with A in tensor memory takes N >= 16 at M = 128:
// B rows 8..15 alias rows 0..7 (zero stride between the two 8-row groups)
// and D columns 8..15 are never read. Each split stores its fp32 sums; the
// epilogue warp that stores the last split of a tile's lane quarter (a
// counter per tile and quarter) adds that quarter's splits in split order,
// applies the SiLU chain and writes the h image. The per-stage scales (two
// per row) are copied by the producer.
//
// down (batch_down_tc_kernel): CTA = 256 output columns (two M = 128 tiles,
// two accumulators) x one split of the union's neurons. The MMA's A is the
// down rows (M = output columns, K = neurons), which only shared memory can
// hold in that orientation: the converters write M-major core matrices into
// a double-buffered A area; B = h from the K-major image the gate/up kernel
// writes (one 1 KB bulk copy per 64 neurons).
//
// Core-matrix layouts (8 rows x 16 bytes, no swizzle):
//   x image / h image, K-major: coordinate k of token n at
//     (k / 8) * 128 + n * 16 + pos(k % 8) * 2 (x) or + (k % 8) * 2 (h);
//   down A, M-major: output column m, neuron k of the stage at
//     (m / 128) * 16384 + ((m % 128) / 8) * 1024 + (k / 8) * 128 + (k % 8) * 16
//     + pos(m % 8) * 2.
// pos() is the order deq produces within 8 coordinates (0, 4, 1, 5, 2, 6, 3,
// 7). Along K (gate/up) the tensor-memory A and the x image share it, so the
// dot products are those of the natural order; along M (down) it permutes
// the accumulator rows, which the epilogue undoes (row 8g + p holds column
// 8g + (p >> 1) + 4 (p & 1)).
//
// Every wait is bounded (ls_b200_batch_args.timeout_ns, 2 s by default): on
// expiry the waiting role sets bit 0 of the caller's error word
// (ls_b200_batch_args.error) and leaves its loop; the producer then waits for
// the copies it issued and the MMA thread for the MMAs it issued (bounded by
// a further kTcGraceNs), and the tensor memory is freed before the CTA ends.
constexpr uint64_t kTcTimeoutNs = 2000000000ull;        // default bound of every wait
constexpr uint64_t kTcMaxTimeoutNs = 60000000000ull;
constexpr uint64_t kTcGraceNs = 1000000000ull;          // drains of own copies / MMAs after a timeout
// kind::f16 instruction descriptor: D fp32 (bits 4-5 = 1), A and B fp16 (0),
// K-major unless bit 15 (A M-major) is set, N >> 3 in bits 17-22, M >> 4 in
// bits 24-28.
constexpr uint32_t kIdescGateUp = (1u << 4) | ((16u >> 3) << 17) | ((128u >> 4) << 24);   // M 128 N 16
constexpr uint32_t kIdescDown = (1u << 4) | (1u << 15) | ((8u >> 3) << 17) | ((128u >> 4) << 24);  // M 128 N 8

// gate/up geometry. A ring stage is 256 coordinates of the tile's 128 rows
// (128 B of each row); an A chunk is 128 of them (one scale block, 64
// tensor-memory columns, 8 MMAs), converted by one of two warp groups in
// turn, which also copies the chunk's x slice next to the A buffer. Each
// wait of the MMA thread drains the MMA pipeline (measured: a few hundred
// cycles, and even a plain shared-memory load of the issuing thread stalls
// behind its MMAs), so it waits once per chunk (A ready); with two CTAs
// per SM the other CTA's MMAs keep the tensor core busy meanwhile, and the
// sixteen converter warps of the SM hide each other's latency. (Measured
// alternative, slower: one CTA per SM waiting once per 16 MMAs.)
constexpr uint32_t kGtK = 256;                          // coordinates per ring stage
constexpr uint32_t kGtChunk = 128;                      // coordinates per tensor-memory A buffer
constexpr uint32_t kGtChunks = kGtK / kGtChunk;         // 2: converter group g takes chunk g of each stage
constexpr uint32_t kGtRowPitch = kGtK / 2 + 16;         // int4 of a row + 16 (conflict-free reads)
constexpr uint32_t kGtW = 128 * kGtRowPitch;            // 18432
constexpr uint32_t kGtX = kGtK * kBatchTokens * 2;      // 4096: the stage's x image
constexpr uint32_t kGtS = 128 * (kGtK / 128) * 2;       // 512: the rows' two fp16 scales
constexpr uint32_t kGtStage = kGtW + kGtX + kGtS;       // 23040
constexpr uint32_t kGtStages = 4;
constexpr uint32_t kGtABufs = 3;                        // A buffers of kGtChunk / 2 columns, in rotation
constexpr uint32_t kGtDCol = kGtABufs * kGtChunk / 2;   // two accumulators (consecutive units) of 16 columns
constexpr uint32_t kGtTmemCols = 256;
constexpr uint32_t kGtXC = kGtChunk * kBatchTokens * 2;  // 2048: a chunk's x slice, copied next to its A buffer
constexpr uint32_t kGtXCopy = kGtStages * kGtStage;     // the x copies [kGtABufs][kGtXC]
constexpr uint32_t kGtBars = 2 * kGtStages + 2 * kGtABufs + 4;  // full, empty, afull, aempty, dfull[2], dempty[2]
constexpr uint32_t kGtSmem = kGtXCopy + kGtABufs * kGtXC + 256;
constexpr uint32_t kGtCtasPerSm = 2;
constexpr uint32_t kGtThreads = 448;                    // producer, MMA, 8 converter, 4 epilogue warps
static_assert(kGtStage % 128 == 0 && kGtW % 16 == 0 && (kGtW + kGtX) % 16 == 0, "stage alignment");
static_assert(kGtBars * 8 + 4 <= 256 && kGtSmem * kGtCtasPerSm <= 227 * 1024, "barrier area, shared memory");
static_assert(kGtDCol + 2 * 16 <= kGtTmemCols, "tensor-memory budget");

// down geometry. Two CTAs per SM, each with stages of 64 neurons: 8 MMAs
// (two M tiles x 4 K steps) per wait of a CTA's MMA thread. A wait drains
// the issuing thread's MMAs (a stage timeline of one CTA per SM with
// 128-neuron stages: ~1,565 cycles of MMAs, then ~430 of drain, per
// ~2,000-cycle stage); with two CTAs the other CTA's MMAs keep the tensor
// core busy meanwhile. The converters also copy the stage's h slice next to
// A, so that one barrier (A ready) covers both operands.
constexpr uint32_t kDtK = 64;                           // neurons per ring stage
constexpr uint32_t kDtCols = 256;                       // output columns per CTA
constexpr uint32_t kDtRowPitch = 144;                   // 128 B of int4 per neuron + 16
constexpr uint32_t kDtW = kDtK * kDtRowPitch;           // 9216
constexpr uint32_t kDtH = kDtK * kBatchTokens * 2;      // 1024: the stage's h image
constexpr uint32_t kDtS = kDtK * 4;                     // two fp16 scales per neuron
constexpr uint32_t kDtRaw = kDtW + kDtH + kDtS;         // 10496
constexpr uint32_t kDtRawStages = 4;
constexpr uint32_t kDtMTile = 128 * kDtK * 2;           // 16384: one M tile of A
constexpr uint32_t kDtMGroup = kDtK * 16;               // 1024: between 8-column groups of an M tile
constexpr uint32_t kDtA = 2 * kDtMTile + kDtH;          // two M tiles + the h copy
constexpr uint32_t kDtABufs = 2;
constexpr uint32_t kDtBars = 2 * kDtRawStages + 2 * kDtABufs + 4;  // rfull, rempty, afull, aempty, dfull[2], dempty[2]
constexpr uint32_t kDtDescCache = 256;                  // union groups cached by the producer
constexpr uint32_t kDtProducers = 1;                    // producer warps, 64 neurons of each stage apiece
constexpr uint32_t kDtConverters = 4;                   // converter warps: thread = (neuron, 128-column half)
constexpr uint32_t kDtSmem = kDtABufs * kDtA + kDtRawStages * kDtRaw + 256 + kDtProducers * kDtDescCache * 8;
constexpr uint32_t kDtThreads = 32 * (2 + kDtConverters + 4);  // producer, MMA, converter, 4 epilogue warps
constexpr uint32_t kDtCtasPerSm = 2;
constexpr uint32_t kDtTmemCols = 32;                    // [2 units][2 M tiles] x 8 columns
constexpr uint32_t kMaxDownSplits = 32;
static_assert(kDtRaw % 128 == 0 && kDtA % 1024 == 0 && kDtCtasPerSm * (kDtSmem + 1024) <= 228 * 1024,
              "stage alignment, budget");
static_assert(32 * kDtConverters == 2 * kDtK && kDtK == 64 * kDtProducers, "one converter thread per neuron and half");
static_assert(kDtK == 64, "the gate/up tiles (64 neurons) write the h image of whole down stages");
static_assert(kDtBars * 8 + 4 <= 256, "barrier area");
static_assert(kMaxDownSplits >= kDownSplits, "partials sized for both paths");

__device__ __forceinline__ uint32_t sm_u32(const void* q) { return uint32_t(__cvta_generic_to_shared(q)); }
__device__ __forceinline__ uint64_t tc_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Shared-memory matrix descriptor, no swizzle, version 1 (bit 46): start,
// leading-dimension byte offset (between core matrices along K for K-major
// operands), stride-dimension byte offset (between 8-row groups along M/N).
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
__device__ __forceinline__ void tc_mbar_init(uint32_t bar, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}
__device__ __forceinline__ bool tc_mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the completion of phase `parity`; false at the deadline.
__device__ __noinline__ bool tc_wait(uint32_t bar, uint32_t parity, uint64_t deadline) {
    for (;;) {
        if (tc_mbar_try(bar, parity)) return true;
        if (tc_now() > deadline) return false;  // %globaltimer: a few cycles beside the try
    }
}
__device__ __forceinline__ void tc_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// global -> shared bulk copy completing on `bar` (no multicast)
__device__ __forceinline__ void tc_bulk(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
template <uint32_t kCols>
__device__ __forceinline__ void tc_alloc(uint32_t slot) {  // warp-wide
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "n"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
template <uint32_t kCols>
__device__ __forceinline__ void tc_dealloc(uint32_t taddr) {  // warp-wide, the allocating warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "n"(kCols) : "memory");
}
// D (tensor memory) += A (shared memory) x B (shared memory)
__device__ __forceinline__ void tc_mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// D (tensor memory) += A (tensor memory) x B (shared memory)
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Lanes 32w..32w+31 (w = warp % 4), columns 0..7 of the accumulator at taddr.
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// The 8 fp16 of a 16-byte chunk of consecutive values x0..x7, reordered to
// the deq order (x0, x4, x1, x5, x2, x6, x3, x7).
__device__ __forceinline__ uint4 to_pos(uint4 w) {
    return make_uint4(__byte_perm(w.x, w.z, 0x5410), __byte_perm(w.x, w.z, 0x7632), __byte_perm(w.y, w.w, 0x5410),
                      __byte_perm(w.y, w.w, 0x7632));
}
// 8 weights of one packed word as fp16(q * s), in the deq order: the same
// values as deq(w, 0..3, s) with one shift instead of three. Pairs (0, 4)
// and (2, 6) are the low nibbles of w and w >> 8 as in deq; pairs (1, 5) and
// (3, 7) stay in place in mantissa bits 4..7 (mask 0x00F000F0), where the
// biased nibble reads 1024 + 16 (q + 8), and v / 16 - 72 = q exactly (one
// fma of exact operands); the product with s is the one rounding.
__device__ __forceinline__ uint4 deq8(uint32_t w, __half2 s2) {
    const uint32_t w8 = w >> 8;
    const __half2 bias = __float2half2_rn(1032.f), sixteenth = __float2half2_rn(0.0625f),
                  m72 = __float2half2_rn(-72.f);
    const __half2 q0 = __hsub2(u2h((w & 0x000F000Fu) ^ 0x64086408u), bias);
    const __half2 q1 = __hfma2(u2h((w & 0x00F000F0u) ^ 0x64806480u), sixteenth, m72);
    const __half2 q2 = __hsub2(u2h((w8 & 0x000F000Fu) ^ 0x64086408u), bias);
    const __half2 q3 = __hfma2(u2h((w8 & 0x00F000F0u) ^ 0x64806480u), sixteenth, m72);
    return make_uint4(h2u(__hmul2(q0, s2)), h2u(__hmul2(q1, s2)), h2u(__hmul2(q2, s2)), h2u(__hmul2(q3, s2)));
}
__device__ __forceinline__ void tc_fail(uint32_t* err) {
    if (err) atomicOr(err, 1u);
}
// Every lane waits (each acquires the phase); the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, uint64_t deadline) {
    return __all_sync(0xffffffffu, tc_wait(bar, parity, deadline)) != 0;
}
// Arrives on `bar` once every cp.async this thread issued so far has landed
// (counted among the barrier's expected arrivals).
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
// Producer exit: wait (bounded) for the last ring stages it filled, so no
// copy lands after the CTA has ended.
__device__ void drain_ring(const uint64_t* full, uint32_t stages, uint32_t issued, uint64_t deadline) {
    const uint32_t first = issued > stages ? issued - stages : 0u;
    for (uint32_t s = first; s < issued; ++s)
        if (!tc_wait(sm_u32(full + s % stages), (s / stages) & 1u, deadline)) return;
}

// h of union neuron n for token b from its split sums: the reference's
// rounding chain (fp16 g and u, s = fp16(silu(g)), h = fp16(s * u)), zero
// where the token's mask excludes the neuron's group.
__device__ __forceinline__ __half h_value(const BatchParams& p, float gs, float us, uint32_t n, uint32_t b) {
    const float g16 = __half2float(__float2half_rn(gs)), u16 = __half2float(__float2half_rn(us));
    const float sl = __half2float(__float2half_rn(g16 / (1.f + expf(-g16))));
    __half h = __float2half_rn(sl * u16);
    if (p.mask && !p.mask[size_t(b) * p.U + n / p.G]) h = __float2half_rn(0.f);
    return h;
}

// x image of the gate/up kernel (and the HF RMSNorm of LS_B200_NORM_INPUT,
// the arithmetic of batch_norm_kernel: inv = rsqrt(sum(x^2) / H + eps),
// x' = fp16(w * fp16(x * inv))): CTA b writes token b's coordinates in
// K-major core matrices, zeros for b >= B. Each thread holds up to four
// 8-coordinate blocks (H <= 8192) in registers; the sum of squares runs in a
// fixed order (per thread, a shuffle tree, then the warps in order). It also
// zeroes the gate/up kernel's split counters.
__global__ void __launch_bounds__(256) batch_ximg_kernel(const __half* x, const __half* w, float eps, uint32_t H,
                                                         uint32_t B, uint32_t norm, uint8_t* img, uint32_t* cnt,
                                                         uint32_t ncnt) {
    __shared__ float part[8];
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < ncnt; i += gridDim.x * blockDim.x)
        cnt[i] = 0u;  // the gate/up kernel's split counters
    const uint32_t b = blockIdx.x, nkg = H / 8;
    const __half* row = x + size_t(b) * H;
    uint4 v[4];
    float ss = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
        const uint32_t kg = threadIdx.x + 256 * j;
        v[j] = make_uint4(0u, 0u, 0u, 0u);
        if (b < B && kg < nkg) v[j] = *reinterpret_cast<const uint4*>(row + 8 * kg);
        const __half* e = reinterpret_cast<const __half*>(&v[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(__half2float(e[i]), __half2float(e[i]), ss);
    }
    float inv = 1.f;
    if (norm) {
#pragma unroll
        for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) tot += part[i];
        inv = rsqrtf(tot / float(H) + eps);
    }
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
        const uint32_t kg = threadIdx.x + 256 * j;
        if (kg >= nkg) continue;
        if (norm && b < B) {
            __half* e = reinterpret_cast<__half*>(&v[j]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                __half t = __float2half_rn(__half2float(e[i]) * inv);
                if (w) t = __hmul(w[8 * kg + i], t);
                e[i] = t;
            }
        }
        *reinterpret_cast<uint4*>(img + size_t(kg) * 128 + b * 16) = to_pos(v[j]);
    }
}

// Persistent: CTA c takes work units c, c + grid, ... (unit = tile x split,
// tile-major); the ring, the tensor-memory A buffers and two accumulators
// run on across units, so a CTA's set-up is paid once.
__global__ void __launch_bounds__(kGtThreads, kGtCtasPerSm) batch_gateup_tc_kernel(const BatchParams p,
                                                                                  uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kGtSmem - 256);
    uint64_t* full = bars;                    // [kGtStages] producer -> converters
    uint64_t* empty = bars + kGtStages;       // [kGtStages] converters -> producer
    uint64_t* afull = bars + 2 * kGtStages;   // [kGtABufs] converters -> MMA
    uint64_t* aempty = afull + kGtABufs;      // [kGtABufs] MMA -> converters
    uint64_t* dfull = aempty + kGtABufs;      // [2] MMA -> epilogue
    uint64_t* dempty = dfull + 2;             // [2] epilogue -> MMA
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + kGtBars);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp == 1) tc_alloc<kGtTmemCols>(sm_u32(tslot));
    if (tid == 0) {
        for (uint32_t i = 0; i < kGtStages; ++i) {
            tc_mbar_init(sm_u32(full + i), 32);  // the producer's 32 lanes (+ the x copy's bytes)
            tc_mbar_init(sm_u32(empty + i), 8);  // the eight converter warps, once they have read the stage
        }
        for (uint32_t i = 0; i < kGtABufs; ++i) {
            tc_mbar_init(sm_u32(afull + i), 4);   // one converter warp per tensor-memory lane quarter
            tc_mbar_init(sm_u32(aempty + i), 1);  // tcgen05.commit
        }
        for (uint32_t i = 0; i < 2; ++i) {
            tc_mbar_init(sm_u32(dfull + i), 1);
            tc_mbar_init(sm_u32(dempty + i), 4);  // the four epilogue warps
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint64_t deadline = tc_now() + p.timeout_ns, grace = deadline + kTcGraceNs;
    const uint32_t S = p.gu_splits, units = ((p.NT + 63) / 64) * S, stages_all = p.H / kGtK;
    auto unit_stages = [&](uint32_t split, uint32_t& st0, uint32_t& st1) {
        st0 = stages_all * split / S;
        st1 = stages_all * (split + 1) / S;
    };
    bool ok = true;

    if (warp == 0) {
        // producer: 16-byte cp.async, one instruction = 4 rows x 128 B (lanes
        // 8i .. 8i + 7 take row i of the four); lane l holds the source of
        // rows l, l + 32, l + 64, l + 96, passed by shuffle
        uint32_t gs = 0;  // stages issued by this CTA
        const uint32_t part = lane & 7u, rsub = lane >> 3;
        for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
            const uint32_t tile = u / S;
            uint32_t st0, st1;
            unit_stages(u % S, st0, st1);
            const uint32_t rows_valid = min(128u, 2u * (p.NT - 64u * tile));
            const uint8_t* src[4];
            const __half* scp[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t row = lane + 32u * j;
                src[j] = nullptr;
                scp[j] = nullptr;
                if (row < rows_valid) {
                    const Row r = neuron_row(p, 64u * tile + row / 2);
                    src[j] = r.src + (row & 1u) * (p.H / 2);
                    scp[j] = r.sc + (row & 1u) * (p.H / 128);
                }
            }
            for (uint32_t s = st0; s < st1; ++s, ++gs) {
                const uint32_t slot = gs % kGtStages;
                if (gs >= kGtStages && !warp_wait(sm_u32(empty + slot), ((gs / kGtStages) - 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                const uint32_t bar = sm_u32(full + slot);
                uint8_t* st = sm + slot * kGtStage;
                const uint32_t k0 = s * kGtK;  // first coordinate of the stage
                if (lane == 0) {
                    tc_expect_tx(bar, kGtX);
                    tc_bulk(sm_u32(st + kGtW), p.ximg + size_t(k0) * 16, kGtX, bar);
                }
#pragma unroll
                for (uint32_t i = 0; i < 32; ++i) {
                    const uint32_t row = 4 * i + rsub;  // rows of one instruction share row / 32
                    const uint8_t* rs = reinterpret_cast<const uint8_t*>(
                        __shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(src[i / 8]), row & 31u));
                    if (row < rows_valid) cp_async16(st + row * kGtRowPitch + 16 * part, rs + k0 / 2 + 16 * part);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j)  // scales of the stage's two 128-blocks
                    if (scp[j]) cp_async4(st + kGtW + kGtX + 4 * (lane + 32u * j), scp[j] + k0 / 128);
                cp_async_arrive(bar);  // arrives once this lane's copies have landed
            }
        }
        if (!ok) tc_fail(err);
        if (lane == 0) drain_ring(full, kGtStages, gs, grace);
        __syncwarp();
    } else if (warp == 1) {
        // MMA issuer: one wait and 8 MMAs per chunk
        if (lane == 0) {
            uint32_t gq = 0, ui = 0;
            for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x, ++ui) {
                uint32_t st0, st1;
                unit_stages(u % S, st0, st1);
                const uint32_t nch = (st1 - st0) * kGtChunks;
                const uint32_t d = ui & 1u, dcol = tmem + kGtDCol + 16 * d;
                if (ui >= 2 && !tc_wait(sm_u32(dempty + d), ((ui / 2) - 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (uint32_t q = 0; q < nch; ++q, ++gq) {
                    const uint32_t a = gq % kGtABufs;
                    if (!tc_wait(sm_u32(afull + a), (gq / kGtABufs) & 1u, deadline)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xb = sm_u32(sm + kGtXCopy + a * kGtXC);
#pragma unroll
                    for (uint32_t kk = 0; kk < kGtChunk / 16; ++kk)
                        tc_mma_ts(dcol, tmem + a * (kGtChunk / 2) + kk * 8, tc_desc(xb + 256 * kk, 128, 0),
                                  kIdescGateUp, (q | kk) ? 1u : 0u);
                    tc_commit(sm_u32(aempty + a));
                }
                tc_commit(sm_u32(dfull + d));  // arrives when every MMA so far has completed
            }
            // every MMA of this CTA complete before the tensor memory is freed
            if (ui && !tc_wait(sm_u32(dfull + ((ui - 1) & 1u)), ((ui - 1) / 2) & 1u, grace)) ok = false;
            if (!ok) tc_fail(err);
        }
        __syncwarp();
    } else if (warp < 10) {
        // converters: warp group g = (warp - 2) / 4 takes chunk g of each
        // stage (coordinates 128 g .. 128 g + 127, one scale block), lane
        // quarter = warp % 4 the rows
        const uint32_t g = (warp - 2) / 4, quarter = warp & 3, row = 32 * quarter + lane;
        const uint32_t lanebits = (32 * quarter) << 16;
        uint32_t gq = 0;
        for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
            const uint32_t tile = u / S;
            uint32_t st0, st1;
            unit_stages(u % S, st0, st1);
            const uint32_t nch = (st1 - st0) * kGtChunks;
            const bool valid = row < min(128u, 2u * (p.NT - 64u * tile));
            for (uint32_t q = g; q < nch; q += kGtChunks) {
                const uint32_t Q = gq + q, gsi = Q / kGtChunks, c = Q % kGtChunks, slot = gsi % kGtStages,
                               a = Q % kGtABufs;
                if (!warp_wait(sm_u32(full + slot), (gsi / kGtStages) & 1u, deadline) ||
                    (Q >= kGtABufs && !warp_wait(sm_u32(aempty + a), ((Q / kGtABufs) - 1) & 1u, deadline))) {
                    ok = false;
                    break;
                }
                const uint8_t* st = sm + slot * kGtStage;
                const __half2 s2 = valid ? __half2half2(reinterpret_cast<const __half*>(st + kGtW + kGtX)[2 * row + c])
                                         : __float2half2_rn(0.f);
                uint4 w4[4];
#pragma unroll
                for (uint32_t i = 0; i < 4; ++i)
                    w4[i] = valid ? *reinterpret_cast<const uint4*>(st + row * kGtRowPitch + 64 * c + 16 * i)
                                  : make_uint4(0u, 0u, 0u, 0u);
                // the chunk's x slice next to the A buffer (thread `row` copies 16 B)
                reinterpret_cast<uint4*>(sm + kGtXCopy + a * kGtXC)[row] =
                    reinterpret_cast<const uint4*>(st + kGtW + c * kGtXC)[row];
                __syncwarp();
                if (lane == 0) tc_arrive(sm_u32(empty + slot));  // this warp is done with the raw stage
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {  // two halves of 32 columns
                    uint32_t v[32];
                    const uint4 w0 = w4[2 * h], w1 = w4[2 * h + 1];
                    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const uint4 dq = deq8(w[i], s2);
                        v[4 * i] = dq.x;
                        v[4 * i + 1] = dq.y;
                        v[4 * i + 2] = dq.z;
                        v[4 * i + 3] = dq.w;
                    }
                    tc_st32(tmem + lanebits + a * (kGtChunk / 2) + 32 * h, v);
                }
                proxy_fence();  // the x copy (generic proxy) -> visible to the tensor core
                tc_fence_before();
                __syncwarp();
                if (lane == 0) tc_arrive(sm_u32(afull + a));
            }
            gq += nch;
        }
        if (!ok) tc_fail(err);
    } else {
        // epilogue: the unit's gate/up sums of the 32 rows of this lane quarter
        const uint32_t quarter = warp & 3, row = 32 * quarter + lane, lanebits = (32 * quarter) << 16;
        uint32_t ui = 0;
        for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x, ++ui) {
            const uint32_t tile = u / S, split = u % S, d = ui & 1u;
            if (!warp_wait(sm_u32(dfull + d), (ui / 2) & 1u, deadline)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float r[8];
            tc_ld8(tmem + lanebits + kGtDCol + 16 * d, r);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) tc_arrive(sm_u32(dempty + d));
            if (row < min(128u, 2u * (p.NT - 64u * tile))) {
                float4* out =
                    reinterpret_cast<float4*>(p.gpart + (size_t(split) * p.rows_total + 128u * tile + row) * kBatchTokens);
                out[0] = make_float4(r[0], r[1], r[2], r[3]);
                out[1] = make_float4(r[4], r[5], r[6], r[7]);
            }
            // This quarter's rows are the gate and up rows of neurons
            // 16 quarter .. +15 of the tile. The warp that stores the last of
            // the tile's S splits of them (stores, fence, then the count; the
            // counters start at zero) sums the splits in split order and
            // writes those neurons' h image: neuron n of token b at
            // (n / 8) * 64 + b * 8 + n % 8, zero past the union and for
            // tokens >= B. Lane: neuron jn = lane / 2, tokens 4 (lane & 1) .. +3.
            __threadfence();
            __syncwarp();
            uint32_t arrived = 0;
            if (lane == 0) arrived = atomicAdd(p.gcnt + 4u * tile + quarter, 1u);
            if (__shfl_sync(0xffffffffu, arrived, 0) == S - 1) {
                __threadfence();
                const uint32_t n = 64u * tile + 16u * quarter + (lane >> 1), b0 = 4u * (lane & 1u);
                float4 g = make_float4(0.f, 0.f, 0.f, 0.f), up = g;
                if (n < p.NT)
                    for (uint32_t sp = 0; sp < S; ++sp) {
                        const float* q = p.gpart + (size_t(sp) * p.rows_total + 2u * n) * kBatchTokens + b0;
                        const float4 a = __ldcg(reinterpret_cast<const float4*>(q));
                        const float4 c = __ldcg(reinterpret_cast<const float4*>(q + kBatchTokens));
                        g.x += a.x, g.y += a.y, g.z += a.z, g.w += a.w;
                        up.x += c.x, up.y += c.y, up.z += c.z, up.w += c.w;
                    }
                const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {up.x, up.y, up.z, up.w};
                __half* hb = p.hB + size_t(n / 8) * 64 + n % 8;
#pragma unroll
                for (uint32_t j = 0; j < 4; ++j) {
                    const uint32_t b = b0 + j;
                    hb[b * 8] = n < p.NT && b < p.B ? h_value(p, gv[j], uv[j], n, b) : __float2half_rn(0.f);
                }
            }
        }
        if (!ok) tc_fail(err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc<kGtTmemCols>(tmem);
    }
}

// Persistent: CTA c takes work units c, c + grid, ... (unit = split x
// column block, split-major, so that the CTAs working at one time read
// neighbouring pieces of the same down rows). The producer warp keeps the
// physical group, source slot and kind of up to kDtDescCache union groups in
// shared memory (refilled when a stage's groups fall outside), so no stage
// waits on a global load before its copies are issued.
__global__ void __launch_bounds__(kDtThreads, kDtCtasPerSm) batch_down_tc_kernel(const BatchParams p, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    uint8_t* abuf = sm;                         // [kDtABufs][kDtA]
    uint8_t* raw = sm + kDtABufs * kDtA;        // [kDtRawStages][kDtRaw]
    uint64_t* bars = reinterpret_cast<uint64_t*>(raw + kDtRawStages * kDtRaw);
    uint64_t* rfull = bars;
    uint64_t* rempty = bars + kDtRawStages;
    uint64_t* afull = bars + 2 * kDtRawStages;
    uint64_t* aempty = afull + kDtABufs;
    uint64_t* dfull = aempty + kDtABufs;   // [2]
    uint64_t* dempty = dfull + 2;          // [2]
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + kDtBars);
    uint2* dcache = reinterpret_cast<uint2*>(raw + kDtRawStages * kDtRaw + 256);  // [kDtDescCache]
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp == 1) tc_alloc<kDtTmemCols>(sm_u32(tslot));
    if (tid == 0) {
        for (uint32_t i = 0; i < kDtRawStages; ++i) {
            tc_mbar_init(sm_u32(rfull + i), 32 * kDtProducers);
            tc_mbar_init(sm_u32(rempty + i), 1);
        }
        for (uint32_t i = 0; i < kDtABufs; ++i) {
            tc_mbar_init(sm_u32(afull + i), kDtConverters);  // the converter warps
            tc_mbar_init(sm_u32(aempty + i), 1);
        }
        for (uint32_t i = 0; i < 2; ++i) {
            tc_mbar_init(sm_u32(dfull + i), 1);
            tc_mbar_init(sm_u32(dempty + i), 4);  // the four epilogue warps
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint64_t deadline = tc_now() + p.timeout_ns, grace = deadline + kTcGraceNs;
    const uint32_t CB = p.H / kDtCols, units = CB * p.dn_splits;
    // a split's stages: 64-neuron blocks [sb, se) of the union (whole h-image blocks)
    const uint32_t stages_all = (p.NT + kDtK - 1) / kDtK;
    auto split_range = [&](uint32_t split, uint32_t& sb, uint32_t& se) {
        sb = stages_all * split / p.dn_splits;
        se = stages_all * (split + 1) / p.dn_splits;
    };
    bool ok = true;

    if (warp < kDtProducers) {
        // producer pw: neurons 64 pw .. 64 pw + 63 of each stage; lane l
        // resolves neurons 64 pw + l and 64 pw + l + 32
        const uint32_t pw = warp;
        uint2* dc = dcache + pw * kDtDescCache;
        uint32_t gs = 0, cache_lo = 0xFFFFFFFFu;
        const size_t rec = size_t(p.G) * (3 * p.H / 2);
        const bool pow2 = (p.G & (p.G - 1)) == 0;
        const uint32_t gshift = uint32_t(__ffs(int(p.G)) - 1);
        auto group_of = [&](uint32_t n) { return pow2 ? n >> gshift : n / p.G; };
        for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
            const uint32_t split = u / CB, c0 = (u % CB) * kDtCols;
            uint32_t sb, se;
            split_range(split, sb, se);
            for (uint32_t s = sb; s < se; ++s, ++gs) {
                const uint32_t slot = gs % kDtRawStages;
                if (gs >= kDtRawStages &&
                    !warp_wait(sm_u32(rempty + slot), ((gs / kDtRawStages) - 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                const uint32_t k0 = s * kDtK, n_valid = min(kDtK, p.NT - k0);
                const uint32_t my0 = 64 * pw, my_valid = n_valid > my0 ? min(64u, n_valid - my0) : 0u;
                if (my_valid) {
                    const uint32_t u_first = group_of(k0 + my0), u_last = group_of(k0 + my0 + my_valid - 1);
                    if (cache_lo == 0xFFFFFFFFu || u_first < cache_lo || u_last >= cache_lo + kDtDescCache) {
                        __syncwarp();
                        cache_lo = u_first;
                        for (uint32_t i = lane; i < kDtDescCache && cache_lo + i < p.U; i += 32) {
                            const ls_exec_desc d = p.desc[cache_lo + i];
                            dc[i] = make_uint2(d.source_slot | (d.source_kind == LS_SOURCE_STAGING ? 0x80000000u : 0u),
                                               d.physical_group);
                        }
                        __syncwarp();
                    }
                }
                const uint32_t bar = sm_u32(rfull + slot);
                uint8_t* st = raw + slot * kDtRaw;
                if (pw == 0 && lane == 0) {
                    tc_expect_tx(bar, kDtH);
                    tc_bulk(sm_u32(st + kDtW), p.hB + size_t(k0) * kBatchTokens, kDtH, bar);
                }
                const uint8_t* src[2];
#pragma unroll
                for (uint32_t j = 0; j < 2; ++j) {
                    const uint32_t kl = my0 + lane + 32u * j;
                    src[j] = nullptr;
                    if (kl >= n_valid) continue;
                    const uint32_t n = k0 + kl, g = group_of(n), nl = n - g * p.G;
                    const uint2 e = dc[g - cache_lo];
                    const uint8_t* base = (e.x & 0x80000000u) ? p.staging : p.cache;
                    src[j] = base + size_t(e.x & 0x7FFFFFFFu) * rec + size_t(nl) * (3 * p.H / 2) + p.H + c0 / 2;
                    const __half* sc = p.scales + (size_t(e.y) * p.G + nl) * 3 * (p.H / 128);
                    cp_async4(st + kDtW + kDtH + 4 * kl, sc + 2 * (p.H / 128) + c0 / 128);
                }
                // 16-byte cp.async, one instruction = 4 neurons x 128 B
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) {
                    const uint32_t kr = 4 * i + (lane >> 3), part = lane & 7u;  // i / 8 = kr / 32: uniform
                    const uint8_t* rs = reinterpret_cast<const uint8_t*>(
                        __shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(src[i / 8]), kr & 31u));
                    if (my0 + kr < n_valid) cp_async16(st + (my0 + kr) * kDtRowPitch + 16 * part, rs + 16 * part);
                }
                cp_async_arrive(bar);
            }
        }
        if (!ok) tc_fail(err);
        if (lane == 0) drain_ring(rfull, kDtRawStages, gs, grace);
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t gs = 0, ui = 0;
            for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x, ++ui) {
                uint32_t sb, se;
                split_range(u / CB, sb, se);
                const uint32_t d = ui & 1u, dcol = tmem + 16 * d;
                if (ui >= 2 && !tc_wait(sm_u32(dempty + d), ((ui / 2) - 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (uint32_t s = sb; s < se; ++s, ++gs) {
                    const uint32_t slot = gs % kDtRawStages, a = gs % kDtABufs;
                    // A ready: the converters have read the raw stage, written A and copied h
                    if (!tc_wait(sm_u32(afull + a), (gs / kDtABufs) & 1u, deadline)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ab = sm_u32(abuf + a * kDtA), hb = ab + 2 * kDtMTile;
#pragma unroll
                    for (uint32_t kk = 0; kk < kDtK / 16; ++kk)
#pragma unroll
                        for (uint32_t mt = 0; mt < 2; ++mt)
                            tc_mma_ss(dcol + 8 * mt, tc_desc(ab + mt * kDtMTile + 256 * kk, 128, kDtMGroup),
                                      tc_desc(hb + 256 * kk, 128, 1024), kIdescDown, (s != sb || kk) ? 1u : 0u);
                    tc_commit(sm_u32(rempty + slot));
                    tc_commit(sm_u32(aempty + a));
                }
                tc_commit(sm_u32(dfull + d));
            }
            if (ui && !tc_wait(sm_u32(dfull + ((ui - 1) & 1u)), ((ui - 1) / 2) & 1u, grace)) ok = false;
            if (!ok) tc_fail(err);
        }
        __syncwarp();
    } else if (warp < 2 + kDtConverters) {
        // converters: thread (neuron kl, 128-column half mt) of each stage
        const uint32_t t = tid - 64, kl = t & (kDtK - 1), mt = t / kDtK;
        uint32_t gs = 0;
        for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
            uint32_t sb, se;
            split_range(u / CB, sb, se);
            for (uint32_t s = sb; s < se; ++s, ++gs) {
                const uint32_t slot = gs % kDtRawStages, a = gs % kDtABufs;
                if (!warp_wait(sm_u32(rfull + slot), (gs / kDtRawStages) & 1u, deadline) ||
                    (gs >= kDtABufs && !warp_wait(sm_u32(aempty + a), ((gs / kDtABufs) - 1) & 1u, deadline))) {
                    ok = false;
                    break;
                }
                const uint8_t* st = raw + slot * kDtRaw;
                uint8_t* A = abuf + a * kDtA;
                const bool live = s * kDtK + kl < p.NT;  // neurons past the union: zero weights
                const __half2 s2 = live ? __half2half2(reinterpret_cast<const __half*>(st + kDtW + kDtH)[2 * kl + mt])
                                        : __float2half2_rn(0.f);
                uint8_t* Ak = A + mt * kDtMTile + (kl / 8) * 128 + (kl % 8) * 16;
#pragma unroll
                for (uint32_t h = 0; h < 4; ++h) {  // 32 columns at a time
                    uint4 w0 = make_uint4(0u, 0u, 0u, 0u);
                    if (live) w0 = *reinterpret_cast<const uint4*>(st + kl * kDtRowPitch + 64 * mt + 16 * h);
                    const uint32_t w[4] = {w0.x, w0.y, w0.z, w0.w};
#pragma unroll
                    for (uint32_t q = 0; q < 4; ++q)  // columns 32h + 8q .. +7: core-matrix group 4h + q
                        *reinterpret_cast<uint4*>(Ak + (4 * h + q) * kDtMGroup) = deq8(w[q], s2);
                }
                if (t < kDtH / 16)  // the stage's h image next to A
                    reinterpret_cast<uint4*>(A + 2 * kDtMTile)[t] = reinterpret_cast<const uint4*>(st + kDtW)[t];
                proxy_fence();  // generic-proxy stores -> visible to the tensor core
                __syncwarp();
                if (lane == 0) tc_arrive(sm_u32(afull + a));
            }
        }
        if (!ok) tc_fail(err);
    } else {
        // epilogue (the last four warps): rows 32 quarter .. +31 of both M tiles of the unit
        const uint32_t quarter = warp & 3, m = 32 * quarter + lane;
        const uint32_t colm = 8 * (m / 8) + ((m % 8) >> 1) + 4 * (m & 1);
        uint32_t ui = 0;
        for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x, ++ui) {
            const uint32_t split = u / CB, c0 = (u % CB) * kDtCols, d = ui & 1u;
            uint32_t sb, se;
            split_range(split, sb, se);
            if (!warp_wait(sm_u32(dfull + d), (ui / 2) & 1u, deadline)) {
                ok = false;
                break;
            }
            float v[2][8];
            if (se > sb) {
                tc_fence_after();
                tc_ld8(tmem + ((32 * quarter) << 16) + 16 * d, v[0]);
                tc_ld8(tmem + ((32 * quarter) << 16) + 16 * d + 8, v[1]);
            } else {  // an empty split contributes zeros
#pragma unroll
                for (int i = 0; i < 8; ++i) v[0][i] = v[1][i] = 0.f;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) tc_arrive(sm_u32(dempty + d));
            float* out = p.partial + size_t(split) * p.B * p.H;
            for (uint32_t b = 0; b < p.B; ++b) {
                out[size_t(b) * p.H + c0 + colm] = v[0][b];
                out[size_t(b) * p.H + c0 + 128 + colm] = v[1][b];
            }
        }
        if (!ok) tc_fail(err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc<kDtTmemCols>(tmem);
    }
}

// Scratch (256-byte aligned parts): h [8][NTP] fp16 (warp-MMA path), the
// down partials [splits][8][H] fp32, the normalised activations [8][H] fp16
// (warp-MMA path, LS_B200_NORM_INPUT), the x image [H / 8][8][8] fp16, the
// gate/up split sums [splits][rows][8] fp32 and the h image [NT64 / 8][8][8]
// fp16 (tensor-core path).
struct ScratchLayout {
    uint64_t ht, part, xn, ximg, gpart, hb, gcnt, total;
};
constexpr uint64_t up256(uint64_t v) { return (v + 255) / 256 * 256; }
uint32_t max_gu_splits(uint32_t H) { return H >= 2048 ? H / 1024 : 1u; }  // splits of >= 1024 coordinates
ScratchLayout scratch_layout(uint32_t H, uint32_t G, uint32_t U) {
    const uint64_t nt = uint64_t(G) * U, ntp = (nt + 15) / 16 * 16 + 16, nt64 = (nt + 63) / 64 * 64;
    ScratchLayout l{};
    l.ht = 0;
    l.part = l.ht + up256(ntp * kBatchTokens * sizeof(__half));
    l.xn = l.part + up256(uint64_t(kMaxDownSplits) * kBatchTokens * H * sizeof(float));
    l.ximg = l.xn + up256(uint64_t(kBatchTokens) * H * sizeof(__half));
    l.gpart = l.ximg + up256(uint64_t(H) * kBatchTokens * sizeof(__half));
    l.hb = l.gpart + up256(uint64_t(max_gu_splits(H)) * 2 * nt64 * kBatchTokens * sizeof(float));
    l.gcnt = l.hb + up256((nt + kDtK - 1) / kDtK * kDtK * kBatchTokens * sizeof(__half));
    l.total = l.gcnt + up256((nt + 63) / 64 * 4 * sizeof(uint32_t)) + 256;
    return l;
}
uint64_t batch_scratch(uint32_t H, uint32_t G, uint32_t U) { return scratch_layout(H, G, U).total; }

// Number of splits that balances `units_per_split * splits` work units over
// `slots` persistent CTAs best (mean units per CTA / the most any CTA
// takes); a larger count must gain more than 5 % (each split adds one
// partial result per unit to write and to sum).
uint32_t pick_splits(uint32_t units_per_split, uint32_t max_splits, uint32_t slots) {
    uint32_t best = 1;
    double best_eff = 0.0;
    for (uint32_t s = 1; s <= max_splits; ++s) {
        const double x = double(units_per_split) * s / slots;
        const double eff = x / double(uint64_t(x) + (x > double(uint64_t(x)) ? 1 : 0));
        if (eff > best_eff + 0.05) {
            best = s;
            best_eff = eff;
        }
    }
    return best;
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

// dynamic shared memory above 48 KB is an opt-in per function and device
cudaError_t set_ring_attributes() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(batch_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGuSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(batch_gateup_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGtSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(batch_down_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kDtSmem));
    if (e == cudaSuccess)  // two CTAs per SM
        e = cudaFuncSetAttribute(batch_down_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 int(cudaSharedmemCarveoutMaxShared));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(batch_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kDnSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(batch_gateup_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 int(cudaSharedmemCarveoutMaxShared));
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace
}  // namespace lsb

extern "C" {

uint64_t ls_b200_batch_scratch_bytes(uint32_t hidden, uint32_t group_size, uint32_t union_count) {
    return lsb::batch_scratch(hidden, group_size, union_count);
}

int ls_b200_batch_mlp(const ls_b200_batch_args* a, void* stream) {
    using namespace lsb;
    if (!a) return EINVAL;
    const uint32_t H = a->hidden, G = a->group_size, U = a->union_count, B = a->tokens;
    if (H < 256 || H > uint32_t(kMaxHidden) || H % 256 || !G || G > uint32_t(kMaxGroupSize) || !U || !B ||
        B > uint32_t(kBatchTokens))
        return EINVAL;
    // union neurons index rows of h and the gate/up grid in 32 bits
    if (uint64_t(G) * U > (uint64_t(1) << 30)) return EINVAL;
    if (!a->x || !a->output || !a->cache || !a->scales || !a->union_descs || !a->scratch ||
        (a->hidden_out && !a->residual) ||
        (a->flags & ~uint32_t(LS_B200_NORM_INPUT | LS_B200_BATCH_MMA_SYNC)) ||
        (a->norm_weight && !(a->flags & LS_B200_NORM_INPUT)))
        return EINVAL;
    if (a->scratch_bytes < batch_scratch(H, G, U)) return ENOSPC;
    if (a->timeout_ns > kTcMaxTimeoutNs) return EINVAL;
    if (!al16(a->x) || !al16(a->cache) || (a->staging && !al16(a->staging)) || !al16(a->scratch) ||
        (reinterpret_cast<uintptr_t>(a->scales) & 3u))
        return EINVAL;
    BatchParams p{};
    p.H = H;
    p.G = G;
    p.U = U;
    p.B = B;
    p.NT = G * U;
    p.NTP = (p.NT + 15) / 16 * 16 + 16;
    p.x = static_cast<const __half*>(a->x);
    p.y = static_cast<__half*>(a->output);
    p.y32 = a->output_f32;
    p.residual = static_cast<const __half*>(a->residual);
    p.hidden_out = static_cast<__half*>(a->hidden_out);
    p.cache = a->cache;
    p.staging = a->staging ? a->staging : a->cache;
    p.scales = static_cast<const __half*>(a->scales);
    p.desc = a->union_descs;
    p.mask = a->mask;
    uint8_t* scratch = static_cast<uint8_t*>(a->scratch);
    const ScratchLayout lay = scratch_layout(H, G, U);
    p.timeout_ns = a->timeout_ns ? a->timeout_ns : kTcTimeoutNs;
    p.hT = reinterpret_cast<__half*>(scratch + lay.ht);
    p.partial = reinterpret_cast<float*>(scratch + lay.part);
    __half* xn = reinterpret_cast<__half*>(scratch + lay.xn);
    p.ximg = scratch + lay.ximg;
    p.gpart = reinterpret_cast<float*>(scratch + lay.gpart);
    p.hB = reinterpret_cast<__half*>(scratch + lay.hb);
    p.gcnt = reinterpret_cast<uint32_t*>(scratch + lay.gcnt);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (const cudaError_t e = set_ring_attributes(); e != cudaSuccess) return int(e);
    const __half* norm_w = static_cast<const __half*>(a->norm_weight);
    const bool norm = (a->flags & LS_B200_NORM_INPUT) != 0;
    if (a->flags & LS_B200_BATCH_MMA_SYNC) {
        p.dn_splits = kDownSplits;
        if (norm) {
            batch_norm_kernel<<<B, 256, 0, s>>>(p.x, norm_w, a->rms_eps, H, xn);
            p.x = xn;
        }
        batch_gateup_kernel<<<(p.NT + kGateUpNeurons - 1) / kGateUpNeurons, kBatchThreads, kGuSmem, s>>>(p);
        batch_down_kernel<<<dim3(H / kDownCols, kDownSplits), kBatchThreads, kDnSmem, s>>>(p);
    } else {
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                      cudaSuccess || sms <= 0)
            sms = 148;
        const uint32_t tiles = (p.NT + 63) / 64, dn_stages = (p.NT + kDtK - 1) / kDtK;
        p.rows_total = tiles * 128;
        const uint32_t gu_slots = kGtCtasPerSm * uint32_t(sms);
        p.gu_splits = pick_splits(tiles, max_gu_splits(H), gu_slots);
        const uint32_t dn_slots = kDtCtasPerSm * uint32_t(sms);
        p.dn_splits = pick_splits(H / kDtCols, dn_stages < kMaxDownSplits ? dn_stages : kMaxDownSplits, dn_slots);
        batch_ximg_kernel<<<kBatchTokens, 256, 0, s>>>(p.x, norm_w, a->rms_eps, H, B, norm ? 1u : 0u,
                                                       scratch + lay.ximg, p.gcnt, 4 * tiles);
        const uint32_t gu_units = tiles * p.gu_splits, dn_units = (H / kDtCols) * p.dn_splits;
        batch_gateup_tc_kernel<<<gu_units < gu_slots ? gu_units : gu_slots, kGtThreads, kGtSmem, s>>>(p, a->error);
        batch_down_tc_kernel<<<dn_units < dn_slots ? dn_units : dn_slots, kDtThreads, kDtSmem, s>>>(p, a->error);
    }
    const uint32_t total = B * H;
    batch_epilogue_kernel<<<(total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024, 256, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : int(e);
}

}  // extern "C"
