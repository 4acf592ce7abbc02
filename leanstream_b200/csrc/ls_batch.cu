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
// Three kernels, each with a fixed summation order (deterministic):
//   gate/up  -- one CTA per 8 union neurons, 8 warps splitting K. A fragment
//               rows 0-7 are the gate rows, 8-15 the up rows; B columns are
//               the tokens. The K index of an MMA maps to coordinates so that
//               a lane's 16 nibbles of a 64-coordinate block are 8 contiguous
//               bytes: k = 2t + j (j < 2) of step s is coordinate 16t + 4s + j,
//               k = 2t + 8 + j is 16t + 4s + 2 + j (t = lane % 4). h is stored
//               token-major for the next kernel.
//   down     -- one CTA per 64 output columns and neuron split. A rows are
//               output columns, K the neurons, B = h (neurons x tokens). In
//               tile tau, row r is column 8r + 2tau and row r + 8 column
//               8r + 2tau + 1, so a lane's 8 columns of one neuron are 4
//               contiguous bytes.
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
constexpr uint32_t kDownCols = 64;
constexpr uint32_t kDownSplits = 4;

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

// fp16(q * s) of two signed nibbles (q exact in fp16; one rounding of the product)
__device__ __forceinline__ uint32_t dq2(uint32_t lo_nib, uint32_t hi_nib, __half2 s) {
    const int ql = int(lo_nib << 28) >> 28, qh = int(hi_nib << 28) >> 28;
    return h2u(__hmul2(__halves2half2(__int2half_rn(ql), __int2half_rn(qh)), s));
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
    __shared__ float red[8][32][4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t n = blockIdx.x * 8 + g;  // this lane's neuron (gate row g, up row g + 8)
    const bool valid = n < p.NT;
    Row r{nullptr, nullptr};
    if (valid) r = neuron_row(p, n);
    const bool tok = uint32_t(g) < p.B;  // this lane's B column (token g)
    const uint32_t KB = p.H / 64;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (uint32_t kb = warp; kb < KB; kb += 8) {
        uint2 wg = make_uint2(0u, 0u), wu = make_uint2(0u, 0u);
        __half2 sg = __float2half2_rn(0.f), su = __float2half2_rn(0.f);
        if (valid) {
            wg = *reinterpret_cast<const uint2*>(r.src + kb * 32 + 8 * t);
            wu = *reinterpret_cast<const uint2*>(r.src + p.H / 2 + kb * 32 + 8 * t);
            sg = __half2half2(r.sc[kb / 2]);
            su = __half2half2(r.sc[p.H / 128 + kb / 2]);
        }
        uint4 x0 = make_uint4(0u, 0u, 0u, 0u), x1 = make_uint4(0u, 0u, 0u, 0u);
        if (tok) {
            const uint4* xp = reinterpret_cast<const uint4*>(p.x + size_t(g) * p.H + kb * 64 + 16 * t);
            x0 = xp[0];
            x1 = xp[1];
        }
        const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        const uint32_t gw[2] = {wg.x, wg.y}, uw[2] = {wu.x, wu.y};
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            // bytes 2s (coordinates 16t+4s, +1) and 2s+1 (+2, +3) of the lane's 8
            const uint32_t gb0 = (gw[s >> 1] >> (16 * (s & 1))) & 0xffu, gb1 = (gw[s >> 1] >> (16 * (s & 1) + 8)) & 0xffu;
            const uint32_t ub0 = (uw[s >> 1] >> (16 * (s & 1))) & 0xffu, ub1 = (uw[s >> 1] >> (16 * (s & 1) + 8)) & 0xffu;
            const uint32_t a0 = dq2(gb0 & 15u, gb0 >> 4, sg);  // row g (gate), k 2t, 2t+1
            const uint32_t a1 = dq2(ub0 & 15u, ub0 >> 4, su);  // row g+8 (up), k 2t, 2t+1
            const uint32_t a2 = dq2(gb1 & 15u, gb1 >> 4, sg);  // row g, k 2t+8, 2t+9
            const uint32_t a3 = dq2(ub1 & 15u, ub1 >> 4, su);  // row g+8, k 2t+8, 2t+9
            mma_f16(acc, a0, a1, a2, a3, xw[2 * s], xw[2 * s + 1]);
        }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) red[warp][lane][e] = acc[e];
    __syncthreads();
    if (warp != 0) return;
    float gs[2] = {0.f, 0.f}, us[2] = {0.f, 0.f};
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        gs[0] += red[w][lane][0];
        gs[1] += red[w][lane][1];
        us[0] += red[w][lane][2];
        us[1] += red[w][lane][3];
    }
    if (!valid) return;
    const uint32_t u = n / p.G;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint32_t b = 2 * t + j;  // token of D column 2t + j
        if (b >= p.B) continue;
        const float g16 = __half2float(__float2half_rn(gs[j])), u16 = __half2float(__float2half_rn(us[j]));
        const float sl = __half2float(__float2half_rn(g16 / (1.f + expf(-g16))));
        __half h = __float2half_rn(sl * u16);
        if (p.mask && !p.mask[size_t(b) * p.U + u]) h = __float2half_rn(0.f);
        p.hT[size_t(b) * p.NTP + n] = h;
    }
}

__global__ void __launch_bounds__(kBatchThreads) batch_down_kernel(const BatchParams p) {
    __shared__ float red[8][32][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint32_t c0 = blockIdx.x * kDownCols, split = blockIdx.y;
    const uint32_t units = (p.NT + 15) / 16;
    const uint32_t u_begin = uint32_t(uint64_t(units) * split / kDownSplits);
    const uint32_t u_end = uint32_t(uint64_t(units) * (split + 1) / kDownSplits);
    const bool tok = uint32_t(g) < p.B;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    for (uint32_t un = u_begin + warp; un < u_end; un += 8) {
        const uint32_t n0 = un * 16;
        // this lane's neurons: k 2t, 2t+1, 2t+8, 2t+9 of the unit
        const uint32_t nn[4] = {n0 + 2 * t, n0 + 2 * t + 1, n0 + 2 * t + 8, n0 + 2 * t + 9};
        uint32_t wv[4];
        __half sv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            wv[k] = 0u;
            sv[k] = __float2half_rn(0.f);
            if (nn[k] < p.NT) {
                const Row r = neuron_row(p, nn[k]);
                wv[k] = *reinterpret_cast<const uint32_t*>(r.src + p.H + c0 / 2 + 4 * g);  // columns c0+8g .. +7
                sv[k] = r.sc[2 * (p.H / 128) + c0 / 128];
            }
        }
        uint32_t b0 = 0u, b1 = 0u;
        if (tok) {
            // h of neurons past the union is never written: zero it here (a zero
            // weight times a stale NaN pattern would still poison the sum)
            const __half* hb = p.hT + size_t(g) * p.NTP + n0;
            if (nn[0] < p.NT) b0 = *reinterpret_cast<const uint32_t*>(hb + 2 * t);      // neurons 2t, 2t+1
            if (nn[2] < p.NT) b1 = *reinterpret_cast<const uint32_t*>(hb + 2 * t + 8);  // neurons 2t+8, 2t+9
            if (nn[1] >= p.NT) b0 &= 0xffffu;
            if (nn[3] >= p.NT) b1 &= 0xffffu;
        }
        const __half2 s01 = __halves2half2(sv[0], sv[1]), s23 = __halves2half2(sv[2], sv[3]);
#pragma unroll
        for (int tau = 0; tau < 4; ++tau) {
            // byte tau of each neuron's 4: columns c0 + 8g + 2tau (low nibble), +1 (high)
            const uint32_t by0 = (wv[0] >> (8 * tau)) & 0xffu, by1 = (wv[1] >> (8 * tau)) & 0xffu;
            const uint32_t by2 = (wv[2] >> (8 * tau)) & 0xffu, by3 = (wv[3] >> (8 * tau)) & 0xffu;
            const uint32_t a0 = dq2(by0 & 15u, by1 & 15u, s01);  // row g, k 2t, 2t+1
            const uint32_t a1 = dq2(by0 >> 4, by1 >> 4, s01);    // row g+8, k 2t, 2t+1
            const uint32_t a2 = dq2(by2 & 15u, by3 & 15u, s23);  // row g, k 2t+8, 2t+9
            const uint32_t a3 = dq2(by2 >> 4, by3 >> 4, s23);    // row g+8, k 2t+8, 2t+9
            mma_f16(acc[tau], a0, a1, a2, a3, b0, b1);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[warp][lane][4 * i + e] = acc[i][e];
    __syncthreads();
    if (warp != 0) return;
    float v[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = 0.f;
    for (int w = 0; w < 8; ++w)
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] += red[w][lane][e];
    float* out = p.partial + size_t(split) * p.B * p.H;
#pragma unroll
    for (int tau = 0; tau < 4; ++tau) {
        const uint32_t col = c0 + 8 * g + 2 * tau;  // row g; row g+8 is col + 1
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t b = 2 * t + j;
            if (b >= p.B) continue;
            out[size_t(b) * p.H + col] = v[4 * tau + j];
            out[size_t(b) * p.H + col + 1] = v[4 * tau + 2 + j];
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
    batch_gateup_kernel<<<(p.NT + 7) / 8, kBatchThreads, 0, s>>>(p);
    batch_down_kernel<<<dim3(H / kDownCols, kDownSplits), kBatchThreads, 0, s>>>(p);
    const uint32_t total = B * H;
    batch_epilogue_kernel<<<(total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024, 256, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : int(e);
}

}  // extern "C"
