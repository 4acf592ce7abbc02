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
// Three kernels, each with a fixed summation order (deterministic):
//   gate/up  -- one CTA per 16 union neurons (two octets), 8 warps splitting
//               K in 64-coordinate blocks, two blocks per iteration. A rows
//               0-7 are the octet's gate rows, 8-15 its up rows; B columns
//               are the tokens, shared by both octets. Lane t of a quad holds
//               coordinates c = 64kb + 16t + 8w .. +7 (w = 0, 1); MMA m of a
//               word takes k 2t, 2t+1 = coordinates c + 2m, c + 2m + 4 and
//               k 2t+8, 2t+9 = c + 2m + 1, c + 2m + 5. h is stored token-major.
//   down     -- one CTA per 128 output columns and eighth of the union's
//               neurons. A rows are output columns, K the neurons, B = h
//               (neurons x tokens). Lane group g holds columns c0 + 16g .. +15
//               of each neuron; in tile T row g is column c0 + 16g + 2T and
//               row g + 8 column c0 + 16g + 2T + 1. The next 16-neuron unit's
//               loads are issued before the current unit's MMAs.
//   epilogue -- y = sum of the splits in split order, fp16 rounding, the
//               optional residual.
#include <cuda_fp16.h>
#include <stdint.h>

#include <cerrno>

#include "ls_internal.h"

namespace lsb {
namespace {

constexpr int kBatchTokens = 8;
constexpr int kBatchThreads = 256;  // 8 warps
constexpr uint32_t kGateUpNeurons = 16;
constexpr uint32_t kDownCols = 128;
constexpr uint32_t kDownSplits = 8;

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

__global__ void __launch_bounds__(kBatchThreads) batch_gateup_kernel(const BatchParams p) {
    __shared__ float red[8][8][32];  // [warp][octet * 4 + d][lane]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    uint32_t n[2];
    bool valid[2];
    Row r[2];
#pragma unroll
    for (int o = 0; o < 2; ++o) {
        n[o] = blockIdx.x * kGateUpNeurons + 8 * o + g;  // gate row g, up row g + 8 of octet o
        valid[o] = n[o] < p.NT;
        r[o] = valid[o] ? neuron_row(p, n[o]) : Row{nullptr, nullptr};
    }
    const bool tok = uint32_t(g) < p.B;  // this lane's B column (token g)
    const uint32_t KB = p.H / 64;
    const __half* xrow = p.x + size_t(g) * p.H + 16 * t;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (uint32_t kb0 = warp; kb0 < KB; kb0 += 16) {
        uint2 wg[2][2], wu[2][2];
        __half2 sg[2][2], su[2][2];
        uint4 xv[2][2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t kb = kb0 + 8 * j;
            const bool inb = kb < KB;
#pragma unroll
            for (int o = 0; o < 2; ++o) {
                wg[j][o] = wu[j][o] = make_uint2(0u, 0u);
                sg[j][o] = su[j][o] = __float2half2_rn(0.f);
                if (inb && valid[o]) {
                    wg[j][o] = *reinterpret_cast<const uint2*>(r[o].src + kb * 32 + 8 * t);
                    wu[j][o] = *reinterpret_cast<const uint2*>(r[o].src + p.H / 2 + kb * 32 + 8 * t);
                    sg[j][o] = __half2half2(r[o].sc[kb / 2]);
                    su[j][o] = __half2half2(r[o].sc[p.H / 128 + kb / 2]);
                }
            }
            xv[j][0] = xv[j][1] = make_uint4(0u, 0u, 0u, 0u);
            if (inb && tok) {
                const uint4* xp = reinterpret_cast<const uint4*>(xrow + kb * 64);
                xv[j][0] = xp[0];
                xv[j][1] = xp[1];
            }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            if (kb0 + 8 * j >= KB) continue;  // warp-uniform
#pragma unroll
            for (int w = 0; w < 2; ++w) {
                const uint4 X = xv[j][w];  // x[c .. c+7] as (c, c+1) (c+2, c+3) (c+4, c+5) (c+6, c+7)
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    const uint32_t xa = m ? X.y : X.x, xb = m ? X.w : X.z;
                    const uint32_t b0 = __byte_perm(xa, xb, 0x5410);  // x[c + 2m], x[c + 2m + 4]
                    const uint32_t b1 = __byte_perm(xa, xb, 0x7632);  // x[c + 2m + 1], x[c + 2m + 5]
#pragma unroll
                    for (int o = 0; o < 2; ++o) {
                        const uint32_t gw = w ? wg[j][o].y : wg[j][o].x, uw = w ? wu[j][o].y : wu[j][o].x;
                        mma_f16(acc[o], deq(gw, 2 * m, sg[j][o]), deq(uw, 2 * m, su[j][o]),
                                deq(gw, 2 * m + 1, sg[j][o]), deq(uw, 2 * m + 1, su[j][o]), b0, b1);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int o = 0; o < 2; ++o)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][4 * o + e][lane] = acc[o][e];
    __syncthreads();
    if (warp >= 2) return;
    const int o = warp;  // warp 0 finishes octet 0, warp 1 octet 1
    float gs[2] = {0.f, 0.f}, us[2] = {0.f, 0.f};
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        gs[0] += red[w][4 * o + 0][lane];
        gs[1] += red[w][4 * o + 1][lane];
        us[0] += red[w][4 * o + 2][lane];
        us[1] += red[w][4 * o + 3][lane];
    }
    const uint32_t nrow = o ? n[1] : n[0];
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
    uint2 w[4];      // columns c0 + 16g .. +15
    __half s[4];     // their down scale (one 128-column block)
    uint32_t b0, b1;  // h of token g: neurons (2t, 2t+1), (2t+8, 2t+9)
};

__device__ __forceinline__ DownIn down_load(const BatchParams& p, uint32_t n0, uint32_t c0, int g, int t, bool tok) {
    DownIn v;
    const uint32_t nn[4] = {n0 + 2 * t, n0 + 2 * t + 1, n0 + 2 * t + 8, n0 + 2 * t + 9};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        v.w[k] = make_uint2(0u, 0u);
        v.s[k] = __float2half_rn(0.f);
        if (nn[k] < p.NT) {
            const Row r = neuron_row(p, nn[k]);
            v.w[k] = *reinterpret_cast<const uint2*>(r.src + p.H + c0 / 2 + 8 * g);
            v.s[k] = r.sc[2 * (p.H / 128) + c0 / 128];
        }
    }
    v.b0 = v.b1 = 0u;
    if (tok) {
        // h of neurons past the union is never written: zero it here (a zero
        // weight times a stale NaN pattern would still poison the sum)
        const __half* hb = p.hT + size_t(g) * p.NTP + n0;
        if (nn[0] < p.NT) v.b0 = *reinterpret_cast<const uint32_t*>(hb + 2 * t);
        if (nn[2] < p.NT) v.b1 = *reinterpret_cast<const uint32_t*>(hb + 2 * t + 8);
        if (nn[1] >= p.NT) v.b0 &= 0xffffu;
        if (nn[3] >= p.NT) v.b1 &= 0xffffu;
    }
    return v;
}

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

__global__ void __launch_bounds__(kBatchThreads) batch_down_kernel(const BatchParams p) {
    __shared__ float red[8][32][32];  // [warp][tile * 4 + d][lane]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t c0 = blockIdx.x * kDownCols, split = blockIdx.y;
    const uint32_t units = (p.NT + 15) / 16;
    const uint32_t u_begin = uint32_t(uint64_t(units) * split / kDownSplits);
    const uint32_t u_end = uint32_t(uint64_t(units) * (split + 1) / kDownSplits);
    const bool tok = uint32_t(g) < p.B;
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    uint32_t un = u_begin + warp;
    if (un < u_end) {
        DownIn cur = down_load(p, un * 16, c0, g, t, tok);
        for (;;) {
            const uint32_t next = un + 8;
            if (next < u_end) {
                const DownIn nxt = down_load(p, next * 16, c0, g, t, tok);
                down_mma(acc, cur);
                cur = nxt;
                un = next;
            } else {
                down_mma(acc, cur);
                break;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][4 * i + e][lane] = acc[i][e];
    __syncthreads();
    // warp T sums tile T over the 8 warps in warp order
    const int T = warp;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < 8; ++w)
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] += red[w][4 * T + e][lane];
    float* out = p.partial + size_t(split) * p.B * p.H;
    const uint32_t col = c0 + 16 * g + 2 * T;  // row g; row g+8 is col + 1
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint32_t b = 2 * t + j;
        if (b >= p.B) continue;
        *reinterpret_cast<float2*>(out + size_t(b) * p.H + col) = make_float2(v[j], v[2 + j]);
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

uint64_t batch_scratch(uint32_t H, uint32_t G, uint32_t U) {
    const uint64_t nt = uint64_t(G) * U, ntp = (nt + 15) / 16 * 16 + 16;
    return ntp * kBatchTokens * sizeof(__half) + uint64_t(kDownSplits) * kBatchTokens * H * sizeof(float) + 256;
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

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
    if (!a->x || !a->output || !a->cache || !a->scales || !a->union_descs || !a->scratch ||
        (a->hidden_out && !a->residual))
        return EINVAL;
    if (a->scratch_bytes < batch_scratch(H, G, U)) return ENOSPC;
    if (!al16(a->x) || !al16(a->cache) || (a->staging && !al16(a->staging)) || !al16(a->scratch)) return EINVAL;
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
    const uint64_t ht_bytes = uint64_t(p.NTP) * kBatchTokens * sizeof(__half);
    p.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(a->scratch) + (ht_bytes + 255) / 256 * 256);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    batch_gateup_kernel<<<(p.NT + kGateUpNeurons - 1) / kGateUpNeurons, kBatchThreads, 0, s>>>(p);
    batch_down_kernel<<<dim3(H / kDownCols, kDownSplits), kBatchThreads, 0, s>>>(p);
    const uint32_t total = B * H;
    batch_epilogue_kernel<<<(total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024, 256, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : int(e);
}

}  // extern "C"
