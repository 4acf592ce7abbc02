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
// Three kernels, each with a fixed summation order (deterministic). The two
// weight kernels stream their rows through a 4-stage shared-memory ring
// filled with cp.async (completion by cp.async.wait_group: no spin loop), so
// three stages of loads are in flight while one is multiplied.
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
    __half* hT;      // [8][NTP] h, token-major
    float* partial;  // [kDownSplits][B][H]
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
        for (uint32_t s = 0; s < kDownSplits; ++s) y += p.partial[size_t(s) * total + i];
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

// Scratch: h [8][NTP] fp16, then the down partials [kDownSplits][8][H] fp32,
// then the normalised activations [8][H] fp16 (LS_B200_NORM_INPUT).
// ------------------------------------------------------------------ tcgen05
// The union GEMMs on the 5th-generation tensor cores (tcgen05.mma, A and B
// from shared memory, the fp32 accumulator in tensor memory). One CTA of
// four warps per tile; the 128 threads convert the tile's int4 rows into
// fp16 w = fp16(q * s) (deq, the same exact conversion as above) in the
// canonical no-swizzle layout, one elected thread issues the MMAs
// (M 128 x N 8 x K 16 each, the 8 tokens as N), and tcgen05.commit frees a
// stage when its MMAs have read it. The accumulator comes back with
// tcgen05.ld (warp w reads tensor-memory lanes 32w..32w+31).
//
// Layouts (bytes, 8-row x 16-byte core matrices, no swizzle):
//   gate/up A, K-major:  row r, coordinate k of the stage at
//     (r / 8) * 1024 + (k / 8) * 128 + (r % 8) * 16 + pos(k % 8) * 2
//     (stride-dimension offset 1024, leading-dimension offset 128);
//   gate/up B (x), K-major: token n at (k / 8) * 128 + n * 16 + pos(k % 8) * 2;
//   down A, MN-major:  output column m, neuron k at
//     (m / 8) * 1024 + (k / 8) * 128 + (k % 8) * 16 + pos(m % 8) * 2;
//   down B (h), K-major: token n, neuron k at (k / 8) * 128 + n * 16 + (k % 8) * 2.
// pos() is the order deq produces within 8 coordinates (0, 4, 1, 5, 2, 6, 3,
// 7). Along K (gate/up) A and B share it, so the dot products are those of
// the natural order; along M (down) it permutes the accumulator rows, which
// the epilogue undoes (row 8g + p holds column 8g + (p >> 1) + 4 (p & 1)).
//
// Every wait is bounded (kTcTimeoutNs): on expiry the CTA sets bit 0 of the
// caller's error word (ls_b200_batch_args.error), waits (bounded) for the
// MMAs it issued, frees its tensor memory and returns.
constexpr uint32_t kTcRows = 128;                      // MMA M
constexpr uint32_t kTcK = 64;                          // coordinates (gate/up) or neurons (down) per stage
constexpr uint32_t kTcStages = 4;
constexpr uint32_t kTcA = kTcRows * kTcK * 2;          // 16 KB
constexpr uint32_t kTcB = kBatchTokens * kTcK * 2;     // 1 KB
constexpr uint32_t kTcStage = kTcA + kTcB;
constexpr uint32_t kTcSmem = kTcStages * kTcStage + 128;  // + mbarriers and the tensor-memory address
constexpr uint32_t kTcCols = 32;                       // tensor-memory columns allocated (8 used)
constexpr uint64_t kTcTimeoutNs = 2000000000ull;
static_assert(kTcStage % 128 == 0, "stage alignment");
// kind::f16 instruction descriptor: D fp32 (bits 4-5 = 1), A and B fp16 (0),
// both K-major, N = 8 (bits 17-22: N >> 3), M = 128 (bits 24-28: M >> 4);
// bit 15 makes A MN-major (the down projection).
constexpr uint32_t kIdescK = (1u << 4) | (1u << 17) | (8u << 24);
constexpr uint32_t kIdescMN = kIdescK | (1u << 15);

__device__ __forceinline__ uint32_t sm_u32(const void* q) { return uint32_t(__cvta_generic_to_shared(q)); }
__device__ __forceinline__ uint64_t tc_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Shared-memory matrix descriptor, no swizzle, version 1 (bit 46).
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
__device__ __forceinline__ void tc_mbar_init(uint32_t bar, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}
__device__ __forceinline__ bool tc_mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the completion of phase `parity`; false at the deadline.
__device__ bool tc_wait(uint32_t bar, uint32_t parity, uint64_t deadline) {
    uint32_t spins = 0;
    while (!tc_mbar_test(bar, parity)) {
        if ((++spins & 255u) == 0 && tc_now() > deadline) return false;
        __nanosleep(20);
    }
    return true;
}
__device__ __forceinline__ void tc_alloc(uint32_t slot) {  // warp-wide
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "n"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr) {  // warp-wide, the allocating warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "n"(kTcCols) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Lanes 32w..32w+31, columns 0..7 of the accumulator (one token each).
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// The 8 fp16 of a 16-byte chunk of consecutive values x0..x7, reordered to
// the deq order (x0, x4, x1, x5, x2, x6, x3, x7).
__device__ __forceinline__ uint4 to_pos(uint4 w) {
    return make_uint4(__byte_perm(w.x, w.z, 0x5410), __byte_perm(w.x, w.z, 0x7632), __byte_perm(w.y, w.w, 0x5410),
                      __byte_perm(w.y, w.w, 0x7632));
}
// 8 weights of one packed word as fp16(q * s), in the deq order.
__device__ __forceinline__ uint4 deq8(uint32_t w, __half2 s2) {
    return make_uint4(deq(w, 0, s2), deq(w, 1, s2), deq(w, 2, s2), deq(w, 3, s2));
}

// Shared teardown: wait (bounded) for the MMAs this CTA issued, free the
// tensor memory. `issued` commits were made; the last one was on stage
// (issued - 1) % kTcStages with parity ((issued - 1) / kTcStages) & 1.
__device__ void tc_finish(uint32_t* err, const uint64_t* mbar, uint32_t issued, uint32_t tmem, bool ok) {
    if (threadIdx.x == 0 && issued) {
        const uint32_t i = issued - 1;
        if (!tc_wait(sm_u32(mbar + i % kTcStages), (i / kTcStages) & 1u, tc_now() + kTcTimeoutNs)) ok = false;
    }
    if (!ok && err) atomicOr(err, 1u);
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) tc_dealloc(tmem);
}

// gate/up: one CTA per 64 union neurons, 128 MMA rows (row 2j the gate row,
// 2j + 1 the up row of neuron j), K = H in stages of 64 coordinates.
__global__ void __launch_bounds__(128) batch_gateup_tc_kernel(const BatchParams p, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + kTcStages * kTcStage);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(mbar + kTcStages);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp == 0) tc_alloc(sm_u32(tslot));
    if (tid == 0) {
        for (uint32_t i = 0; i < kTcStages; ++i) tc_mbar_init(sm_u32(mbar + i), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint64_t deadline = tc_now() + kTcTimeoutNs;
    // this thread's A row: neuron j = tid / 2 of the tile, gate (even) or up (odd)
    const uint32_t nrow = blockIdx.x * 64 + uint32_t(tid >> 1);
    const bool valid = nrow < p.NT;
    const uint8_t* src = nullptr;
    const __half* sc = nullptr;
    if (valid) {
        const Row r = neuron_row(p, nrow);
        src = r.src + (tid & 1) * (p.H / 2);
        sc = r.sc + (tid & 1) * (p.H / 128);
    }
    const uint32_t nst = p.H / kTcK;
    uint8_t* arow = sm + (tid / 8) * 1024 + (tid % 8) * 16;  // chunk c of this row at + c * 128
    uint4 cur0 = make_uint4(0u, 0u, 0u, 0u), cur1 = cur0;
    if (valid) {
        cur0 = __ldg(reinterpret_cast<const uint4*>(src));
        cur1 = __ldg(reinterpret_cast<const uint4*>(src) + 1);
    }
    bool ok = true;
    uint32_t issued = 0;
    for (uint32_t i = 0; i < nst; ++i) {
        const uint32_t s = i % kTcStages;
        uint8_t* stage = sm + s * kTcStage;
        if (i >= kTcStages && !tc_wait(sm_u32(mbar + s), ((i / kTcStages) - 1) & 1u, deadline)) ok = false;
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        // next stage's 32 bytes in flight while this one is converted
        uint4 nx0 = make_uint4(0u, 0u, 0u, 0u), nx1 = nx0;
        if (valid && i + 1 < nst) {
            nx0 = __ldg(reinterpret_cast<const uint4*>(src + 32 * (i + 1)));
            nx1 = __ldg(reinterpret_cast<const uint4*>(src + 32 * (i + 1)) + 1);
        }
        const __half2 s2 = __half2half2(valid ? sc[(kTcK * i) / 128] : __float2half_rn(0.f));
        const uint32_t w[8] = {cur0.x, cur0.y, cur0.z, cur0.w, cur1.x, cur1.y, cur1.z, cur1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(stage + (arow - sm) + c * 128) = deq8(w[c], s2);
        if (tid < 64) {  // x of the stage: token n = tid / 8, coordinates 8c .. 8c + 7
            const uint32_t n = tid >> 3, c = tid & 7;
            uint4 xv = make_uint4(0u, 0u, 0u, 0u);
            if (n < p.B) xv = __ldg(reinterpret_cast<const uint4*>(p.x + size_t(n) * p.H + kTcK * i + 8 * c));
            *reinterpret_cast<uint4*>(stage + kTcA + c * 128 + n * 16) = to_pos(xv);
        }
        proxy_fence();  // generic-proxy stores -> visible to the tensor core (async proxy)
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a = sm_u32(stage), b = sm_u32(stage + kTcA);
#pragma unroll
            for (uint32_t kk = 0; kk < kTcK / 16; ++kk)
                tc_mma(tmem, tc_desc(a + 256 * kk, 128, 1024), tc_desc(b + 256 * kk, 128, 1024), kIdescK,
                       (i | kk) ? 1u : 0u);
            tc_commit(sm_u32(mbar + s));
        }
        ++issued;
        cur0 = nx0;
        cur1 = nx1;
    }
    if (ok) {  // every MMA done: the accumulator rows
        const uint32_t last = issued - 1;
        if (!tc_wait(sm_u32(mbar + last % kTcStages), (last / kTcStages) & 1u, deadline)) ok = false;
    }
    if (__syncthreads_and(ok)) {
        tc_fence_after();
        float v[8];
        tc_ld8(tmem + (uint32_t(32 * warp) << 16), v);
        const uint32_t u = valid ? nrow / p.G : 0u;
#pragma unroll
        for (int b = 0; b < kBatchTokens; ++b) {
            const float up = __shfl_xor_sync(0xffffffffu, v[b], 1);  // odd lane: the up row
            if ((lane & 1) || !valid || uint32_t(b) >= p.B) continue;
            const float g16 = __half2float(__float2half_rn(v[b])), u16 = __half2float(__float2half_rn(up));
            const float sl = __half2float(__float2half_rn(g16 / (1.f + expf(-g16))));
            __half h = __float2half_rn(sl * u16);
            if (p.mask && !p.mask[size_t(b) * p.U + u]) h = __float2half_rn(0.f);
            p.hT[size_t(b) * p.NTP + nrow] = h;
        }
    }
    tc_finish(err, mbar, issued, tmem, ok);
}

// down: one CTA per 128 output columns and split of the union's neurons
// (the splits of the mma.sync kernel, summed by the epilogue).
__global__ void __launch_bounds__(128) batch_down_tc_kernel(const BatchParams p, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + kTcStages * kTcStage);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(mbar + kTcStages);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp == 0) tc_alloc(sm_u32(tslot));
    if (tid == 0) {
        for (uint32_t i = 0; i < kTcStages; ++i) tc_mbar_init(sm_u32(mbar + i), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint64_t deadline = tc_now() + kTcTimeoutNs;
    const uint32_t c0 = blockIdx.x * kTcRows, split = blockIdx.y;
    // split boundaries on 64-neuron stage boundaries (16-byte aligned h rows)
    const uint32_t k_begin = uint32_t(uint64_t(p.NT) * split / kDownSplits) / kTcK * kTcK;
    const uint32_t k_end =
        split + 1 == kDownSplits ? p.NT : uint32_t(uint64_t(p.NT) * (split + 1) / kDownSplits) / kTcK * kTcK;
    const uint32_t nst = (k_end - k_begin + kTcK - 1) / kTcK;
    // converter: neuron kl = tid % 64 of the stage, columns 64 * (tid / 64) .. +63
    const uint32_t kl = uint32_t(tid) & 63u, half = uint32_t(tid) >> 6;
    bool ok = true;
    uint32_t issued = 0;
    for (uint32_t i = 0; i < nst; ++i) {
        const uint32_t s = i % kTcStages;
        uint8_t* stage = sm + s * kTcStage;
        if (i >= kTcStages && !tc_wait(sm_u32(mbar + s), ((i / kTcStages) - 1) & 1u, deadline)) ok = false;
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        const uint32_t k = k_begin + kTcK * i + kl;
        uint4 w0 = make_uint4(0u, 0u, 0u, 0u), w1 = w0;
        __half2 s2 = __float2half2_rn(0.f);
        if (k < k_end) {
            const Row r = neuron_row(p, k);
            const uint8_t* d = r.src + p.H + (c0 + 64 * half) / 2;  // 32 bytes: 64 columns
            w0 = __ldg(reinterpret_cast<const uint4*>(d));
            w1 = __ldg(reinterpret_cast<const uint4*>(d) + 1);
            s2 = __half2half2(r.sc[2 * (p.H / 128) + c0 / 128]);
        }
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {  // columns c0 + 64 half + 8q .. +7: M group 8 half + q
            const uint32_t g = 8 * half + uint32_t(q);
            *reinterpret_cast<uint4*>(stage + g * 1024 + (kl / 8) * 128 + (kl % 8) * 16) = deq8(w[q], s2);
        }
        if (tid < 64) {  // h of the stage: token n = tid / 8, neurons 8c .. 8c + 7
            const uint32_t n = tid >> 3, c = tid & 7, k8 = k_begin + kTcK * i + 8 * c;
            uint4 hv = make_uint4(0u, 0u, 0u, 0u);
            if (n < p.B && k8 < k_end) {
                hv = *reinterpret_cast<const uint4*>(p.hT + size_t(n) * p.NTP + k8);
                // neurons past the split's end (and past the union) contribute nothing
                const uint32_t valid_n = k_end - k8;
                if (valid_n < 8) {
                    uint32_t* hw = reinterpret_cast<uint32_t*>(&hv);
#pragma unroll
                    for (uint32_t e = 0; e < 4; ++e) {
                        if (2 * e >= valid_n) hw[e] = 0u;
                        else if (2 * e + 1 >= valid_n) hw[e] &= 0xffffu;
                    }
                }
            }
            *reinterpret_cast<uint4*>(stage + kTcA + c * 128 + n * 16) = hv;
        }
        proxy_fence();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a = sm_u32(stage), b = sm_u32(stage + kTcA);
#pragma unroll
            for (uint32_t kk = 0; kk < kTcK / 16; ++kk)
                tc_mma(tmem, tc_desc(a + 256 * kk, 128, 1024), tc_desc(b + 256 * kk, 128, 1024), kIdescMN,
                       (i | kk) ? 1u : 0u);
            tc_commit(sm_u32(mbar + s));
        }
        ++issued;
    }
    if (ok && issued) {
        const uint32_t last = issued - 1;
        if (!tc_wait(sm_u32(mbar + last % kTcStages), (last / kTcStages) & 1u, deadline)) ok = false;
    }
    if (__syncthreads_and(ok)) {
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (issued) {
            tc_fence_after();
            tc_ld8(tmem + (uint32_t(32 * warp) << 16), v);
        }
        const uint32_t m = uint32_t(32 * warp + lane), col = c0 + 8 * (m / 8) + ((m % 8) >> 1) + 4 * (m & 1);
        float* out = p.partial + size_t(split) * p.B * p.H;
        for (uint32_t b = 0; b < p.B; ++b) out[size_t(b) * p.H + col] = v[b];
    }
    tc_finish(err, mbar, issued, tmem, ok);
}

uint64_t batch_scratch(uint32_t H, uint32_t G, uint32_t U) {
    const uint64_t nt = uint64_t(G) * U, ntp = (nt + 15) / 16 * 16 + 16;
    const uint64_t ht = (ntp * kBatchTokens * sizeof(__half) + 255) / 256 * 256;
    const uint64_t part = (uint64_t(kDownSplits) * kBatchTokens * H * sizeof(float) + 255) / 256 * 256;
    return ht + part + uint64_t(kBatchTokens) * H * sizeof(__half) + 256;
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
        e = cudaFuncSetAttribute(batch_gateup_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTcSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(batch_down_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kTcSmem));
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
    p.hT = static_cast<__half*>(a->scratch);
    const uint64_t ht_bytes = (uint64_t(p.NTP) * kBatchTokens * sizeof(__half) + 255) / 256 * 256;
    p.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(a->scratch) + ht_bytes);
    const uint64_t part_bytes = (uint64_t(kDownSplits) * kBatchTokens * H * sizeof(float) + 255) / 256 * 256;
    __half* xn = reinterpret_cast<__half*>(static_cast<uint8_t*>(a->scratch) + ht_bytes + part_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (const cudaError_t e = set_ring_attributes(); e != cudaSuccess) return int(e);
    if (a->flags & LS_B200_NORM_INPUT) {
        batch_norm_kernel<<<B, 256, 0, s>>>(p.x, static_cast<const __half*>(a->norm_weight), a->rms_eps, H, xn);
        p.x = xn;
    }
    if (a->flags & LS_B200_BATCH_MMA_SYNC) {
        batch_gateup_kernel<<<(p.NT + kGateUpNeurons - 1) / kGateUpNeurons, kBatchThreads, kGuSmem, s>>>(p);
        batch_down_kernel<<<dim3(H / kDownCols, kDownSplits), kBatchThreads, kDnSmem, s>>>(p);
    } else {
        batch_gateup_tc_kernel<<<(p.NT + 63) / 64, 128, kTcSmem, s>>>(p, a->error);
        batch_down_tc_kernel<<<dim3(H / kTcRows, kDownSplits), 128, kTcSmem, s>>>(p, a->error);
    }
    const uint32_t total = B * H;
    batch_epilogue_kernel<<<(total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024, 256, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : int(e);
}

}  // extern "C"
