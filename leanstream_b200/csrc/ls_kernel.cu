// Fused sparse INT4 SwiGLU MLP for sm_100a: one persistent launch runs one
// layer (the ComputeBackend path) or a whole stack of layers.
//
// It replaces the reference's three-launch chain A core_kernel -> B consumer
// -> reduction (kernels/streaming_mlp.cu:44-93; backends/triton/core.py:20-64,
// persistent.py:33-92, reduction.py:6-28), and for stacks also the per-layer
// residual + RMSNorm glue (reduction.py:17-20;
// examples/ministral/native/predictor_shared_input.cu:16-33).
//
// CTA = 8 consumer warps + 1 producer warp, one CTA per SM. The producer
// streams packed INT4 rows into a 6-stage shared-memory ring with
// cp.async.bulk (TMA bulk copies, no multicast) and fp16 scales with
// cp.async, completing one mbarrier per stage. It runs ahead across layer
// boundaries: weights do not depend on activations, so the next layer's
// rows are in flight while consumers synchronise on the current one.
//
// Work is described by "pieces" the producer writes next to each stage:
//   GATEUP: gate+up rows of up to 32 neurons -> h = fp16(fp16(SiLU(g)) * u)
//   DOWN:   rows x column range of one descriptor's down matrix -> fp32
//           partial row segment (one partial row per descriptor position)
//   LAYER:  end of a layer; carries the partial-row count
//   FINAL:  end of the launch
// Schedules:
//   fast path (all queue descriptors ready at decision time; BatchCompat):
//     static, balanced split of all neurons (GATEUP) and of all
//     (descriptor, 32-column chunk) pairs (DOWN) over the grid; a DOWN piece
//     waits on a per-descriptor counter of published h values.
//   progressive path: CTAs claim descriptor positions in ready order from a
//     device-memory counter (core descriptors first) and run all pieces of
//     each claimed descriptor.
// Canonical arithmetic, shared by both schedules (so BatchCompat and
// Progressive outputs are bit-identical, tests/persistent_mlp_test.cu:65):
//   g, u : per lane, 16-byte chunks j = lane + 32 i, 4 pair accumulators,
//          then a fixed xor-butterfly over the warp;
//   down : per column, one fp32 chain over the descriptor's neurons in order;
//   y    : per column, partial rows summed in row order.
// Rounding boundaries (core.py:17,49-52; reduction.py:15): w = fp16(q*s),
// g,u -> fp16, SiLU -> fp16, h -> fp16, fp32 partials, y -> fp16 once.
//
// Synchronisation uses counters with bounded waits only -- no named
// barriers inside loops -- so a warp that gives up can never strand the
// others. Every wait ends at a %globaltimer deadline and records an error.
#include <cuda_fp16.h>
#include <stdint.h>
#include "ls_internal.h"

namespace lsb {

enum : uint32_t { kPieceFinal = 0, kPieceGateUp = 1, kPieceDown = 2, kPieceLayer = 3 };
enum : uint32_t { kFirstRows = 1u, kLastRows = 2u, kCompletes = 4u, kLayerGood = 8u };
constexpr uint32_t kPathFast = 1, kPathProgressive = 2, kPathAbort = 3;

// Wait bounds, ordered so that a stalled launch always drains its ring:
// host-publication and data waits end at the deadline, the producer's wait
// for a free stage 1 s later, the consumers' wait for a full stage 2 s later
// and layer synchronisation 3 s later.
constexpr uint64_t kProducerGraceNs = 1000000000ull;
constexpr uint64_t kConsumerGraceNs = 2000000000ull;
constexpr uint64_t kSyncGraceNs = 3000000000ull;

struct Piece {
    uint32_t kind;
    uint32_t row;     // partial row = descriptor position (core first, then queue index)
    uint32_t dest;    // descriptor dest_slot (activation / counter index)
    uint32_t n0;      // GATEUP: first neuron; DOWN: first row of the down matrix
    uint32_t count;   // GATEUP: neurons; DOWN: rows; LAYER: partial rows of the layer
    uint32_t k0;      // DOWN: first 16-byte chunk (32 columns)
    uint32_t chunks;  // DOWN: 16-byte chunks per row
    uint32_t sb0;     // DOWN: first scale index (even) of the column range
    uint32_t nsb;     // DOWN: scale halves per row (even)
    uint32_t flags;
    uint32_t layer;   // launch-local layer index
    uint32_t pad[5];
};
static_assert(sizeof(Piece) == 64, "piece record");

struct DescView {
    const uint8_t* src;  // packed group base
    uint32_t phys, dest, row, ok;
};

struct SmemTail {
    unsigned long long full_bar[kStages];
    unsigned long long empty_bar[kStages];
    Piece piece[kStages];
    DescView dtab[32];  // producer's descriptor window
    __half hs[kConsumerWarps * kMaxGroupSize];
    alignas(16) __half xs[kMaxHidden];  // activation of the current layer, staged once per CTA
    uint32_t warps_done;     // consumer warps that finished a layer (monotonic)
    volatile uint32_t abort;
    volatile uint32_t xready;     // layers whose activation is staged in xs
    volatile uint32_t partials;   // layers whose partial rows are complete grid-wide
    uint32_t last;
    uint32_t pad[3];
};

size_t kernel_smem_bytes() { return size_t(kStages) * kStageBytes + sizeof(SmemTail); }

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t tx) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// TMA bulk copy global -> shared (no multicast), completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Mixed-precision fma: d = a*b + c with fp16 a, b (exact product) and fp32 c.
__device__ __forceinline__ float mfma(__half a, __half b, float c) {
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(__half_as_ushort(a)), "h"(__half_as_ushort(b)), "f"(c));
    return d;
}
__device__ __forceinline__ __half2 as_h2(uint32_t v) {
    __half2 h;
    *reinterpret_cast<uint32_t*>(&h) = v;
    return h;
}

// Eight signed two's-complement nibbles (low nibble = even coordinate,
// backends/triton/core.py:14-15) -> four half2 of exact integers:
// q[p] = (coord p, coord p+4), p = 0..3.
__device__ __forceinline__ void unpack8(uint32_t w, __half2 (&q)[4]) {
    const uint32_t lo = (w & 0x000F000Fu) ^ 0x64086408u;  // 1024 + (q + 8)
    const uint32_t hi = (w & 0x00F000F0u) ^ 0x64806480u;  // 1024 + 16 (q + 8)
    const uint32_t w8 = w >> 8;
    const uint32_t lo2 = (w8 & 0x000F000Fu) ^ 0x64086408u;
    const uint32_t hi2 = (w8 & 0x00F000F0u) ^ 0x64806480u;
    const __half2 k1032 = __float2half2_rn(1032.f);
    const __half2 k16 = __float2half2_rn(0.0625f);
    const __half2 k72 = __float2half2_rn(-72.f);
    q[0] = __hsub2(as_h2(lo), k1032);
    q[1] = __hfma2(as_h2(hi), k16, k72);
    q[2] = __hsub2(as_h2(lo2), k1032);
    q[3] = __hfma2(as_h2(hi2), k16, k72);
}

// gate/up accumulation of one 32-bit word (8 coordinates) against x.
__device__ __forceinline__ void dot_word(uint32_t w, __half2 s, const __half2* x, float (&acc)[4]) {
    __half2 q[4];
    unpack8(w, q);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        const __half2 v = __hmul2(q[p], s);  // == fp16(float(q) * float(s)), core.py:17
        acc[p] = mfma(__low2half(v), __low2half(x[p]), acc[p]);
        acc[p] = mfma(__high2half(v), __high2half(x[p]), acc[p]);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}
__device__ __forceinline__ float h2f(uint16_t v) { return __half2float(__ushort_as_half(v)); }
__device__ __forceinline__ float round16(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ uint32_t* ws_layer(const KernelParams& P, uint32_t l) {
    return P.ws + kWsHeader + kWsPerLayer * l;  // [0] path [1] claim [2] partials-done CTAs [3] reduced blocks
}
__device__ __forceinline__ uint32_t* done_h(const KernelParams& P, uint32_t l) {
    return P.ws + kWsHeader + kWsPerLayer * P.max_layers + size_t(l) * P.N;
}
__device__ __forceinline__ void trace(const KernelParams& P, uint32_t word) {
    if (P.trace) P.trace[size_t(blockIdx.x) * LS_B200_TRACE_WORDS + word] = gtimer();
}
// Per-layer stamps after the launch-level block: [grid][nlayers][LS_B200_LAYER_TRACE_WORDS].
__device__ __forceinline__ void trace_layer(const KernelParams& P, uint32_t l, uint32_t word) {
    if (P.trace)
        P.trace[size_t(gridDim.x) * LS_B200_TRACE_WORDS +
                (size_t(blockIdx.x) * P.nlayers + l) * LS_B200_LAYER_TRACE_WORDS + word] = gtimer();
}
// Records the first error of this launch and asks the CTA to stop.
__device__ __forceinline__ void raise_error(const KernelParams& P, SmemTail* t, uint32_t code, uint32_t detail) {
    if (atomicCAS(P.ws + kWsErr, 0u, code) == 0u) P.ws[kWsDetail] = detail;
    t->abort = 1;
}
// Plan of launch-local layer l, read in place (kernel parameter or device array).
__device__ __forceinline__ const LayerPlan& plan_at(const KernelParams& P, uint32_t l) {
    return P.plans ? P.plans[l] : P.first;
}

// ------------------------------------------------------------ descriptors
// Descriptor at canonical position d: core[d] for d < core_count, else the
// queue descriptor published at ready position d - core_count
// (streaming_mlp.cu:60, persistent.py:80). Partial row: d for core, else
// core_count + descriptor index (custom_triton.md:54).
__device__ DescView load_desc(const KernelParams& P, const LayerPlan& L, uint32_t d) {
    const uint32_t* c;
    uint32_t row;
    if (d < L.core_count) {
        c = reinterpret_cast<const uint32_t*>(L.core + d);
        row = d;
    } else {
        const uint32_t idx = ld_relaxed_sys(L.q.ready_indices + (d - L.core_count));
        if (idx >= L.q.capacity) return DescView{nullptr, 0, 0, 0, 0};
        c = reinterpret_cast<const uint32_t*>(L.q.descriptors + idx);
        row = L.core_count + idx;
    }
    const uint32_t phys = ld_relaxed_sys(c + 1), slot = ld_relaxed_sys(c + 2);
    const uint32_t dest = ld_relaxed_sys(c + 3), kind = ld_relaxed_sys(c + 4);
    DescView v;
    v.ok = kind <= 1u && dest < P.N && row < P.N && (P.phys_groups == 0 || phys < P.phys_groups) &&
           (kind == 0 ? (P.cache_slots == 0 || slot < P.cache_slots)
                      : (P.staging_slots == 0 || slot < P.staging_slots));
    v.src = (kind == 0 ? L.cache : L.staging) + size_t(slot) * P.group_bytes;
    v.phys = phys;
    v.dest = dest;
    v.row = row;
    return v;
}

// ------------------------------------------------------------ producer side
struct Producer {
    uint32_t idx;   // pieces issued so far (stage = idx % kStages)
    uint32_t lane;
    uint8_t* stages;
    SmemTail* t;
    uint64_t deadline;
    uint32_t wbase;  // first descriptor position held in t->dtab
    uint32_t wlayer;
};

// Waits until the next stage is free; lane 0 polls, the warp learns the result.
__device__ bool producer_acquire_stage(Producer& pr, const KernelParams& P) {
    const uint32_t s = pr.idx % kStages;
    const uint32_t parity = ((pr.idx / kStages) & 1u) ^ 1u;
    uint32_t ok = 1;
    if (pr.lane == 0) {
        const uint32_t bar = smem_u32(&pr.t->empty_bar[s]);
        uint32_t spins = 0;
        while (!mbar_try_wait(bar, parity)) {
            if ((++spins & 255u) == 0 && gtimer() > pr.deadline + kProducerGraceNs) {
                raise_error(P, pr.t, LS_B200_DEV_TIMEOUT_SYNC, 1);
                ok = 0;
                break;
            }
        }
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// A data-less piece (LAYER or FINAL marker).
__device__ bool producer_marker(Producer& pr, const KernelParams& P, uint32_t kind, uint32_t layer, uint32_t rows,
                                uint32_t flags) {
    if (!producer_acquire_stage(pr, P)) return false;
    const uint32_t s = pr.idx % kStages;
    if (pr.lane == 0) {
        Piece& pc = pr.t->piece[s];
        pc.kind = kind;
        pc.layer = layer;
        pc.count = rows;
        pc.flags = flags;
        mbar_arrive_expect_tx(smem_u32(&pr.t->full_bar[s]), 0);
    }
    cp_async_arrive_noinc(smem_u32(&pr.t->full_bar[s]));
    ++pr.idx;
    return true;
}

// GATEUP piece: neurons [n0, n0+count) of one descriptor.
__device__ bool producer_gateup(Producer& pr, const KernelParams& P, const LayerPlan& L, const DescView& d,
                                uint32_t layer, uint32_t n0, uint32_t count) {
    if (!producer_acquire_stage(pr, P)) return false;
    const uint32_t s = pr.idx % kStages;
    uint8_t* st = pr.stages + size_t(s) * kStageBytes;
    const uint32_t bar = smem_u32(&pr.t->full_bar[s]);
    const uint32_t H = P.H;
    const uint64_t rec = uint64_t(3) * H / 2;  // bytes per neuron record
    if (pr.lane == 0) {
        Piece& pc = pr.t->piece[s];
        pc.kind = kPieceGateUp;
        pc.layer = layer;
        pc.row = d.row;
        pc.dest = d.dest;
        pc.n0 = n0;
        pc.count = count;
        mbar_arrive_expect_tx(bar, count * H);
        for (uint32_t k = 0; k < count; ++k)
            bulk_g2s(smem_u32(st + size_t(k) * H), d.src + (n0 + k) * rec, H, bar);
    }
    // gate+up scales: H/128 words per neuron, at the start of its scale row.
    const uint32_t wpn = H / 128;
    const uint32_t words = count * wpn;
    const uint32_t sdst = smem_u32(st + kStageData);
    for (uint32_t i = pr.lane; i < words; i += 32) {
        const uint32_t k = i / wpn, w = i % wpn;
        const uint16_t* src = L.scales + (size_t(d.phys) * P.G + n0 + k) * (3 * H / 128) + 2 * w;
        cp_async4(sdst + 4 * i, src);
    }
    cp_async_arrive_noinc(bar);
    ++pr.idx;
    return true;
}

// DOWN piece: rows [r0, r0+rows) x chunks [k0, k0+m) of one descriptor.
__device__ bool producer_down(Producer& pr, const KernelParams& P, const LayerPlan& L, const DescView& d,
                              uint32_t layer, uint32_t r0, uint32_t rows, uint32_t k0, uint32_t m, uint32_t flags) {
    if (!producer_acquire_stage(pr, P)) return false;
    const uint32_t s = pr.idx % kStages;
    uint8_t* st = pr.stages + size_t(s) * kStageBytes;
    const uint32_t bar = smem_u32(&pr.t->full_bar[s]);
    const uint32_t H = P.H;
    const uint64_t rec = uint64_t(3) * H / 2;
    const uint32_t pitch = 16 * m;
    const uint32_t sb0 = (k0 / 4) & ~1u;
    const uint32_t sb1 = ((k0 + m - 1) / 4 + 2) & ~1u;
    const uint32_t nsb = sb1 - sb0;
    if (pr.lane == 0) {
        Piece& pc = pr.t->piece[s];
        pc.kind = kPieceDown;
        pc.layer = layer;
        pc.row = d.row;
        pc.dest = d.dest;
        pc.n0 = r0;
        pc.count = rows;
        pc.k0 = k0;
        pc.chunks = m;
        pc.sb0 = sb0;
        pc.nsb = nsb;
        pc.flags = flags;
        mbar_arrive_expect_tx(bar, rows * pitch);
        for (uint32_t r = 0; r < rows; ++r)
            bulk_g2s(smem_u32(st + size_t(r) * pitch), d.src + (r0 + r) * rec + H + 16 * k0, pitch, bar);
    }
    const uint32_t wpr = nsb / 2;  // words per row
    const uint32_t words = rows * wpr;
    const uint32_t sdst = smem_u32(st + kStageData);
    for (uint32_t i = pr.lane; i < words; i += 32) {
        const uint32_t r = i / wpr, w = i % wpr;
        const uint16_t* src =
            L.scales + (size_t(d.phys) * P.G + r0 + r) * (3 * H / 128) + 2 * (H / 128) + sb0 + 2 * w;
        cp_async4(sdst + 4 * i, src);
    }
    cp_async_arrive_noinc(bar);
    ++pr.idx;
    return true;
}

// Rows per DOWN piece and 16-byte chunks per DOWN piece (<= 64 so that one
// consumer thread owns one 8-column task).
__device__ __forceinline__ uint32_t down_rows(const KernelParams& P) { return P.G < 32u ? P.G : 32u; }
__device__ __forceinline__ uint32_t down_chunks(const KernelParams& P) {
    const uint32_t hc = P.H / 32;
    uint32_t m = (kStageData / down_rows(P)) / 16;
    if (m > 64u) m = 64u;
    return m < hc ? m : hc;
}
__device__ __forceinline__ uint32_t gateup_neurons(const KernelParams& P) {
    const uint32_t n = kStageData / P.H;
    return n < 32u ? n : 32u;
}

// DOWN pieces of chunks [k0, k0+m) of one descriptor, all row groups.
__device__ bool producer_down_range(Producer& pr, const KernelParams& P, const LayerPlan& L, const DescView& d,
                                    uint32_t layer, uint32_t k0, uint32_t m) {
    const uint32_t G = P.G, hc = P.H / 32, rr = down_rows(P);
    for (uint32_t r = 0; r < G; r += rr) {
        const uint32_t rows = (G - r) < rr ? (G - r) : rr;
        uint32_t f = 0;
        if (r == 0) f |= kFirstRows;
        if (r + rows == G) f |= kLastRows;
        if (r + rows == G && k0 + m == hc) f |= kCompletes;
        if (!producer_down(pr, P, L, d, layer, r, rows, k0, m, f) || pr.t->abort) return false;
    }
    return true;
}

// All pieces of one descriptor (progressive path).
__device__ bool producer_descriptor(Producer& pr, const KernelParams& P, const LayerPlan& L, const DescView& d,
                                    uint32_t layer) {
    const uint32_t G = P.G, hc = P.H / 32;
    const uint32_t np = gateup_neurons(P);
    for (uint32_t n = 0; n < G; n += np) {
        const uint32_t c = (G - n) < np ? (G - n) : np;
        if (!producer_gateup(pr, P, L, d, layer, n, c) || pr.t->abort) return false;
    }
    const uint32_t mm = down_chunks(P);
    for (uint32_t k = 0; k < hc; k += mm) {
        const uint32_t m = (hc - k) < mm ? (hc - k) : mm;
        if (!producer_down_range(pr, P, L, d, layer, k, m)) return false;
    }
    return true;
}

// Loads the descriptor window [base, base+32) into shared memory, one
// descriptor per lane (two dependent reads per lane).
__device__ bool producer_window(Producer& pr, const KernelParams& P, const LayerPlan& L, uint32_t layer,
                                uint32_t base, uint32_t D) {
    const uint32_t d = base + pr.lane;
    uint32_t bad = 0;
    if (d < D) {
        const DescView v = load_desc(P, L, d);
        pr.t->dtab[pr.lane] = v;
        bad = v.ok ? 0u : 1u;
    }
    __syncwarp();
    const uint32_t mask = __ballot_sync(0xffffffffu, bad);
    pr.wbase = base;
    pr.wlayer = layer;
    if (mask) {
        if (pr.lane == 0) raise_error(P, pr.t, LS_B200_DEV_BAD_DESCRIPTOR, base + __ffs(mask) - 1);
        return false;
    }
    return true;
}

// Per-CTA path decision for one layer (streaming_mlp.cu:49-56,
// persistent.py:46-55). BatchCompat / Auto wait for the batch epoch and take
// the fast path; Progressive proposes a path and agrees with the other CTAs
// through a device-memory CAS (QueueControl.consumer_path stays untouched:
// a discrete GPU has no host-native atomics).
__device__ uint32_t decide(const KernelParams& P, const LayerPlan& L, uint32_t l, SmemTail* t, uint64_t deadline,
                           uint32_t* total_out) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(L.q.control);
    const bool batch = L.mode != LS_MODE_PROGRESSIVE;  // Auto follows BatchCompat (streaming_mlp.cu:90)
    uint32_t code = 0;
    for (;;) {
        const uint4 a = ld_relaxed_sys_v4(w);
        const uint4 b = ld_relaxed_sys_v4(w + 4);
        if (b.y) { code = LS_B200_DEV_QUEUE_ERROR; break; }
        if (a.w == L.epoch && (!batch || b.x == L.epoch)) {
            // Acquire the deciding word (a system-scope acquire load is ~0.2 us;
            // a system-scope fence is ~4 us on this part).
            if (ld_acquire_sys(w + (batch ? 4 : 3)) == L.epoch) break;
        }
        if (gtimer() > deadline) { code = LS_B200_DEV_TIMEOUT_EPOCH; break; }
        __nanosleep(100);
    }
    uint32_t path = kPathAbort, total = 0;
    if (!code) {
        const uint4 a = ld_relaxed_sys_v4(w);  // ordered after the acquire above
        total = a.z;
        const uint32_t ready = batch ? total : a.x;
        if (total > L.q.capacity || L.core_count + total > P.N || ready > total) {
            code = LS_B200_DEV_BAD_PLAN;
        } else {
            const uint32_t proposal = ready == total ? kPathFast : kPathProgressive;
            if (batch) {
                path = proposal;
            } else {
                const uint32_t old = atomicCAS(ws_layer(P, l) + 0, 0u, proposal);
                path = old ? old : proposal;
            }
        }
    }
    if (code) {
        raise_error(P, t, code, l);
        path = kPathAbort;
    }
    *total_out = total;
    return path;
}

__device__ void stamp(const LayerPlan& L, const DescView& d) {
    if (L.stamps) L.stamps[d.dest] = gtimer();
}

// Producer warp main loop over the layers of the launch.
__device__ void run_producer(const KernelParams& P, uint8_t* stages, SmemTail* t, uint64_t deadline) {
    Producer pr{0, threadIdx.x & 31u, stages, t, deadline, 0xffffffffu, 0xffffffffu};
    bool ok = true;
    for (uint32_t l = 0; ok && l < P.nlayers; ++l) {
        const LayerPlan& L = plan_at(P, l);
        uint32_t path = 0, total = 0;
        if (pr.lane == 0) path = decide(P, L, l, t, deadline, &total);
        path = __shfl_sync(0xffffffffu, path, 0);
        total = __shfl_sync(0xffffffffu, total, 0);
        if (pr.lane == 0 && l == 0) trace(P, LS_B200_TRACE_DECIDED);
        if (pr.lane == 0) trace_layer(P, l, LS_B200_LTRACE_DECIDED);
        if (path == kPathAbort) break;
        const uint32_t D = L.core_count + total;
        pr.wbase = pr.wlayer = 0xffffffffu;
        if (path == kPathFast) {
            const uint32_t G = P.G, hc = P.H / 32;
            const uint64_t NT = uint64_t(D) * G, CT = uint64_t(D) * hc;
            const uint32_t b = blockIdx.x, grid = gridDim.x;
            const uint64_t u1 = NT * (b + 1) / grid, v1 = CT * (b + 1) / grid;
            uint64_t u = NT * b / grid, v = CT * b / grid;
            const uint32_t np = gateup_neurons(P), mm = down_chunks(P);
            // GATEUP pieces over this CTA's neuron range.
            while (ok && u < u1) {
                const uint32_t d = uint32_t(u / G), n = uint32_t(u % G);
                if (pr.wlayer != l || d < pr.wbase || d >= pr.wbase + 32) ok = producer_window(pr, P, L, l, d, D);
                if (!ok) break;
                const DescView dv = t->dtab[d - pr.wbase];
                if (n == 0 && pr.lane == 0) stamp(L, dv);
                uint32_t c = G - n;
                if (c > np) c = np;
                if (u + c > u1) c = uint32_t(u1 - u);
                ok = producer_gateup(pr, P, L, dv, l, n, c) && !t->abort;
                u += c;
            }
            // DOWN pieces over this CTA's (descriptor, chunk) range.
            while (ok && v < v1) {
                const uint32_t d = uint32_t(v / hc), k = uint32_t(v % hc);
                if (pr.wlayer != l || d < pr.wbase || d >= pr.wbase + 32) ok = producer_window(pr, P, L, l, d, D);
                if (!ok) break;
                const DescView dv = t->dtab[d - pr.wbase];
                uint32_t m = hc - k;
                if (m > mm) m = mm;
                if (v + m > v1) m = uint32_t(v1 - v);
                ok = producer_down_range(pr, P, L, dv, l, k, m);
                v += m;
            }
        } else {
            const uint32_t* words = reinterpret_cast<const uint32_t*>(L.q.control);
            uint32_t* claim = ws_layer(P, l) + 1;
            while (ok && !t->abort) {
                uint32_t pos = 0, code = 0;
                if (pr.lane == 0) {
                    pos = atomicAdd(claim, 1u);
                    if (pos >= D) {
                        code = 0xffffffffu;  // exhausted
                    } else if (pos >= L.core_count) {
                        // Wait until the claimed queue position is published
                        // (persistent.py:71-90; streaming_mlp.cu:63-75).
                        const uint32_t q = pos - L.core_count;
                        for (;;) {
                            if (ld_acquire_sys(words + 5)) { code = LS_B200_DEV_QUEUE_ERROR; break; }
                            if (ld_acquire_sys(words + 0) > q) break;
                            if (gtimer() > deadline) { code = LS_B200_DEV_TIMEOUT_READY; break; }
                            __nanosleep(128);
                        }
                    }
                    if (code && code != 0xffffffffu) raise_error(P, t, code, pos);
                }
                code = __shfl_sync(0xffffffffu, code, 0);
                pos = __shfl_sync(0xffffffffu, pos, 0);
                if (code) break;
                ok = producer_window(pr, P, L, l, pos, pos + 1);  // one descriptor, lane 0
                if (!ok) break;
                const DescView dv = t->dtab[0];
                if (pr.lane == 0) stamp(L, dv);
                ok = producer_descriptor(pr, P, L, dv, l);
            }
            if (t->abort) ok = false;
        }
        if (pr.lane == 0) trace_layer(P, l, LS_B200_LTRACE_ISSUED);
        if (ok) ok = producer_marker(pr, P, kPieceLayer, l, D, t->abort ? 0u : kLayerGood);
    }
    producer_marker(pr, P, kPieceFinal, 0, 0, 0);
    if (pr.lane == 0) trace(P, LS_B200_TRACE_PRODUCED);
}

// ------------------------------------------------------------ consumer side
template <int MAXC>
struct Activation {
    __half2 x[MAXC][16];  // chunk i of this lane: pairs (c, c+4) per 8-coordinate word
};

// Loads this lane's activation chunks with 16-byte loads and, when flagged,
// applies the HF RMSNorm of predictor_shared_input.cu:16-33 per warp:
// inv = rsqrt(sum(x^2)/H + eps); x' = fp16(weight * fp16(x * inv)).
// The sum is per lane in chunk order, then a fixed butterfly: every warp of
// every CTA computes the same value.
template <int MAXC>
__device__ void load_activation(const KernelParams& P, const LayerPlan& L, const __half* xs, Activation<MAXC>& a,
                                int lane) {
    const uint32_t hc = P.H / 32;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
        const uint32_t j = lane + 32 * i;
        uint4 w[4];
        if (j < hc) {
            const uint4* src = reinterpret_cast<const uint4*>(xs + 32 * j);
#pragma unroll
            for (int v = 0; v < 4; ++v) w[v] = src[v];
        } else {
#pragma unroll
            for (int v = 0; v < 4; ++v) w[v] = make_uint4(0, 0, 0, 0);
        }
        // word v holds coordinates 8v..8v+7 as 4 half2 (2e, 2e+1)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const __half2* h = reinterpret_cast<const __half2*>(&w[v]);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const __half lo = (p & 1) ? __high2half(h[p >> 1]) : __low2half(h[p >> 1]);
                const __half hi = (p & 1) ? __high2half(h[2 + (p >> 1)]) : __low2half(h[2 + (p >> 1)]);
                a.x[i][4 * v + p] = __halves2half2(lo, hi);  // (coord 8v+p, 8v+p+4)
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(h[e]);
                ss += f.x * f.x;
                ss += f.y * f.y;
            }
        }
    }
    if (L.flags & LS_B200_NORM_INPUT) {
        const float inv = rsqrtf(warp_sum(ss) / float(P.H) + P.eps);
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
            const uint32_t j = lane + 32 * i;
            __half2 wv[16];
            if (L.norm_w && j < hc) {
                const uint4* src = reinterpret_cast<const uint4*>(L.norm_w + 32 * j);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const uint4 w = __ldg(src + v);
                    const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const __half lo = (p & 1) ? __high2half(h[p >> 1]) : __low2half(h[p >> 1]);
                        const __half hi = (p & 1) ? __high2half(h[2 + (p >> 1)]) : __low2half(h[2 + (p >> 1)]);
                        wv[4 * v + p] = __halves2half2(lo, hi);
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float2 f = __half22float2(a.x[i][k]);
                __half2 n = __halves2half2(__float2half_rn(f.x * inv), __float2half_rn(f.y * inv));
                if (L.norm_w && j < hc) n = __hmul2(wv[k], n);
                a.x[i][k] = n;
            }
        }
    }
}

template <int MAXC>
__device__ void consume_gateup(const KernelParams& P, const LayerPlan& L, const Piece& pc, const uint8_t* st,
                               const Activation<MAXC>& a, int warp, int lane) {
    const uint32_t H = P.H, hc = H / 32;
    const __half* sc = reinterpret_cast<const __half*>(st + kStageData);
    uint32_t* dh = done_h(P, pc.layer) + pc.row;
    for (uint32_t k = warp; k < pc.count; k += kConsumerWarps) {
        const uint8_t* row = st + size_t(k) * H;
        const __half* scr = sc + size_t(k) * (H / 64);
        float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < MAXC; ++i) {
            const uint32_t j = lane + 32 * i;
            if (j < hc) {
                const uint4 wg = *reinterpret_cast<const uint4*>(row + 16 * j);
                const uint4 wu = *reinterpret_cast<const uint4*>(row + H / 2 + 16 * j);
                const __half2 sg = __half2half2(scr[j >> 2]);
                const __half2 su = __half2half2(scr[(H >> 7) + (j >> 2)]);
                dot_word(wg.x, sg, &a.x[i][0], ag);
                dot_word(wu.x, su, &a.x[i][0], au);
                dot_word(wg.y, sg, &a.x[i][4], ag);
                dot_word(wu.y, su, &a.x[i][4], au);
                dot_word(wg.z, sg, &a.x[i][8], ag);
                dot_word(wu.z, su, &a.x[i][8], au);
                dot_word(wg.w, sg, &a.x[i][12], ag);
                dot_word(wu.w, su, &a.x[i][12], au);
            }
        }
        float g = (ag[0] + ag[1]) + (ag[2] + ag[3]);
        float u = (au[0] + au[1]) + (au[2] + au[3]);
        g = warp_sum(g);
        u = warp_sum(u);
        if (lane == 0) {
            const float g16 = round16(g), u16 = round16(u);
            const float s = round16(g16 / (1.f + expf(-g16)));
            const __half h = __float2half_rn(s * u16);
            const uint32_t n = pc.n0 + k;
            P.hbuf[size_t(pc.row) * P.G + n] = __half_as_ushort(h);
            if (L.act) L.act[size_t(pc.dest) * P.G + n] = __half_as_ushort(h);
            red_release_gpu(dh, 1u);
        }
    }
}

// DOWN piece: thread owns 8 columns (4 packed bytes) of the range.
__device__ void consume_down(const Piece& pc, const uint8_t* st, const __half* hs, float (&acc)[8], int tid) {
    const uint32_t pitch = 16 * pc.chunks;
    const uint32_t ntask = 4 * pc.chunks;
    if (uint32_t(tid) >= ntask) return;
    const __half* sc = reinterpret_cast<const __half*>(st + kStageData);
    const uint32_t col = 32 * pc.k0 + 8 * tid;
    const uint32_t sbi = (col >> 7) - pc.sb0;
    const uint8_t* base = st + 4 * tid;
    uint32_t r = 0;
    for (; r + 4 <= pc.count; r += 4) {
        uint32_t wv[4];
        __half2 s2[4];
        __half hh[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            wv[e] = *reinterpret_cast<const uint32_t*>(base + size_t(r + e) * pitch);
            s2[e] = __half2half2(sc[(r + e) * pc.nsb + sbi]);
            hh[e] = hs[pc.n0 + r + e];
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            __half2 q[4];
            unpack8(wv[e], q);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const __half2 v = __hmul2(q[p], s2[e]);
                acc[p] = mfma(__low2half(v), hh[e], acc[p]);
                acc[p + 4] = mfma(__high2half(v), hh[e], acc[p + 4]);
            }
        }
    }
    for (; r < pc.count; ++r) {
        const uint32_t wv = *reinterpret_cast<const uint32_t*>(base + size_t(r) * pitch);
        const __half2 s2 = __half2half2(sc[r * pc.nsb + sbi]);
        const __half hh = hs[pc.n0 + r];
        __half2 q[4];
        unpack8(wv, q);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const __half2 v = __hmul2(q[p], s2);
            acc[p] = mfma(__low2half(v), hh, acc[p]);
            acc[p + 4] = mfma(__high2half(v), hh, acc[p + 4]);
        }
    }
}

// Bounded warp-level wait until *counter >= target (acquire, gpu scope).
// `stop_on_abort`: give up early when this CTA already failed.
__device__ bool warp_wait_count(const KernelParams& P, SmemTail* t, const uint32_t* counter, uint32_t target,
                                uint64_t limit, uint32_t detail, bool stop_on_abort, int lane) {
    uint32_t ok = 1;
    if (lane == 0) {
        uint32_t spins = 0;
        while (ld_acquire_gpu(counter) < target) {
            if (stop_on_abort && t->abort) { ok = 0; break; }
            if ((++spins & 63u) == 0 && gtimer() > limit) {
                raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, detail);
                ok = 0;
                break;
            }
            __nanosleep(32);
        }
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Per-warp staging of the h values of `row` (layer l): lane 0 waits until
// all G neurons of the row published h, then the warp copies them into its
// private shared-memory slice.
__device__ bool stage_h_warp(const KernelParams& P, SmemTail* t, uint32_t l, uint32_t row, int lane, __half* hs,
                             uint64_t deadline) {
    if (!warp_wait_count(P, t, done_h(P, l) + row, P.G, deadline, 3, true, lane)) return false;
    for (uint32_t n = lane; n < P.G; n += 32) hs[n] = __ushort_as_half(__ldcg(P.hbuf + size_t(row) * P.G + n));
    __syncwarp();
    return true;
}

// Compact reduction of one 32-column block (reduction.py:6-28,
// streaming_mlp.cu:80-84): lane = column, partial rows summed in order;
// then the layer epilogue (fp16 output, residual add, fp32 output).
__device__ void reduce_block(const KernelParams& P, const LayerPlan& L, uint32_t blk, uint32_t rows, bool write,
                             int lane) {
    const uint32_t H = P.H, c = 32 * blk + lane;
    const float* p = P.partial + c;
    float s = 0.f;
    uint32_t r = 0;
    for (; r + 8 <= rows; r += 8) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __ldcg(p + size_t(r + e) * H);
#pragma unroll
        for (int e = 0; e < 8; ++e) s += v[e];
    }
    for (; r < rows; ++r) s += __ldcg(p + size_t(r) * H);
    if (!write) return;
    if (L.y32) L.y32[c] = s;
    const __half y16 = __float2half_rn(s);
    if (L.y && !(L.flags & LS_B200_NO_OUTPUT)) L.y[c] = __half_as_ushort(y16);
    if (L.hidden_out && L.residual)
        L.hidden_out[c] = __half_as_ushort(__float2half_rn(h2f(L.residual[c]) + __half2float(y16)));
}

// Bounded wait until a volatile shared-memory word reaches `target`.
__device__ bool smem_wait(const KernelParams& P, SmemTail* t, volatile uint32_t* word, uint32_t target,
                          uint64_t limit, uint32_t detail, int lane) {
    uint32_t ok = 1;
    if (lane == 0) {
        uint32_t spins = 0;
        while (*word < target) {
            if ((++spins & 255u) == 0 && gtimer() > limit) {
                raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, detail);
                ok = 0;
                break;
            }
            __nanosleep(20);
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __threadfence_block();
    return ok != 0;
}

// Warp 0 stages layer l's activation into shared memory once per CTA
// (16-byte loads, bypassing L1: the previous layer's reducers wrote it).
__device__ void stage_x(const KernelParams& P, const LayerPlan& L, SmemTail* t, uint32_t l, int lane) {
    const uint4* src = reinterpret_cast<const uint4*>(L.x);
    uint4* dst = reinterpret_cast<uint4*>(t->xs);
    for (uint32_t i = lane; i < P.H / 8; i += 32) dst[i] = __ldcg(src + i);
    __syncwarp();
    __threadfence_block();
    if (lane == 0) t->xready = l + 1;
}

template <int MAXC>
__device__ void run_consumers(const KernelParams& P, uint8_t* stages, SmemTail* t, uint64_t deadline) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __half* hs = t->hs + warp * kMaxGroupSize;
    uint32_t l = 0;
    const LayerPlan* L = &plan_at(P, 0);
    Activation<MAXC> a;
    if (warp == 0) stage_x(P, *L, t, 0, lane);
    smem_wait(P, t, &t->xready, 1, deadline + kSyncGraceNs, 7, lane);
    load_activation<MAXC>(P, *L, t->xs, a, lane);
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    const uint32_t nblk = P.H / 32;
    for (uint32_t idx = 0;; ++idx) {
        const uint32_t s = idx % kStages;
        const uint32_t parity = (idx / kStages) & 1u;
        const uint32_t bar = smem_u32(&t->full_bar[s]);
        // Warp-uniform bounded wait on the stage's mbarrier (acquire of the
        // TMA-written data).
        uint32_t spins = 0;
        bool timed_out = false;
        for (;;) {
            const bool ready = mbar_try_wait(bar, parity);
            if (__all_sync(0xffffffffu, ready)) break;
            uint32_t late = 0;
            if (lane == 0 && (++spins & 255u) == 0 && gtimer() > deadline + kConsumerGraceNs) late = 1;
            if (__shfl_sync(0xffffffffu, late, 0)) {
                timed_out = true;
                break;
            }
        }
        if (timed_out) {
            // The producer stopped without a FINAL marker; nothing is in
            // flight for this stage. No barrier follows, so leaving is safe.
            if (lane == 0) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 4);
            break;
        }
        const Piece pc = t->piece[s];
        if (idx == 0 && tid == 0) trace(P, LS_B200_TRACE_FIRST);
        if (tid == 0 && pc.kind == kPieceLayer) trace_layer(P, l, LS_B200_LTRACE_PIECES_DONE);
        if (pc.kind == kPieceFinal) {
            if (tid == 0) trace(P, LS_B200_TRACE_PIECES);
            break;
        }
        const uint8_t* st = stages + size_t(s) * kStageBytes;
        const bool aborted = __shfl_sync(0xffffffffu, t->abort, 0) != 0;  // warp-uniform snapshot
        if (pc.kind == kPieceGateUp) {
            if (!aborted) consume_gateup<MAXC>(P, *L, pc, st, a, warp, lane);
        } else if (pc.kind == kPieceDown) {
            bool have_h = true;
            if (pc.flags & kFirstRows) {
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = 0.f;
                if (uint32_t(warp * 32) < 4 * pc.chunks && !aborted)
                    have_h = stage_h_warp(P, t, l, pc.row, lane, hs, deadline);
            }
            if (!aborted && have_h) {
                consume_down(pc, st, hs, acc, tid);
                if ((pc.flags & kLastRows) && uint32_t(tid) < 4 * pc.chunks) {
                    float* dst = P.partial + size_t(pc.row) * P.H + 32 * pc.k0 + 8 * tid;
                    reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
                    reinterpret_cast<float4*>(dst)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
                }
                if ((pc.flags & kCompletes) && tid == 0 && L->execs) atomicAdd(L->execs + pc.dest, 1u);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&t->empty_bar[s]));
        if (pc.kind != kPieceLayer) continue;

        // ---- end of layer l: partial rows -> reduction -> next activation.
        // One poller per CTA for each grid-wide counter; the other warps
        // wait on shared-memory words, so the L2 sees at most gridDim.x
        // pollers per counter.
        uint32_t* wl = ws_layer(P, l);
        const uint64_t limit = deadline + kSyncGraceNs;
        __threadfence();  // this warp's partial rows are visible at gpu scope
        if (lane == 0) {
            const uint32_t old = atomicAdd(&t->warps_done, 1u);
            if (old == uint32_t(kConsumerWarps) * (l + 1) - 1) red_release_gpu(wl + 2, 1u);
        }
        const bool good = (pc.flags & kLayerGood) != 0;
        const uint32_t first_blk = blockIdx.x * kConsumerWarps;
        if (first_blk < nblk) {  // this CTA owns reduction blocks
            if (warp == 0) {
                if (warp_wait_count(P, t, wl + 2, gridDim.x, limit, 5, false, lane) && lane == 0) t->partials = l + 1;
                if (tid == 0) trace_layer(P, l, LS_B200_LTRACE_PARTIALS_READY);
            }
            for (uint32_t blk = first_blk + warp; blk < nblk; blk += gridDim.x * kConsumerWarps) {
                const bool ready = smem_wait(P, t, &t->partials, l + 1, limit, 5, lane);
                const bool write = ready && good && ld_acquire_gpu(P.ws + kWsErr) == 0;
                if (ready) reduce_block(P, *L, blk, pc.count, write, lane);
                __threadfence();
                if (lane == 0) red_release_gpu(wl + 3, 1u);
            }
        }
        if (tid == 0) trace_layer(P, l, LS_B200_LTRACE_REDUCED);
        if (l + 1 >= P.nlayers) continue;  // the FINAL marker follows
        const LayerPlan* next = &plan_at(P, l + 1);
        if (warp == 0) {
            if (warp_wait_count(P, t, wl + 3, nblk, limit, 6, false, lane)) {
                if (tid == 0) trace_layer(P, l, LS_B200_LTRACE_NEXT_READY);
                stage_x(P, *next, t, l + 1, lane);
            }
        }
        if (!smem_wait(P, t, &t->xready, l + 2, limit, 6, lane)) continue;
        ++l;
        L = next;
        load_activation<MAXC>(P, *L, t->xs, a, lane);
        if (tid == 0) trace_layer(P, l, LS_B200_LTRACE_LOADED);
    }
}

template <int MAXC>
__global__ void __launch_bounds__(kThreads, 1) fused_mlp_kernel(const __grid_constant__ KernelParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    SmemTail* t = reinterpret_cast<SmemTail*>(smem + size_t(kStages) * kStageBytes);
    const int tid = threadIdx.x;
    const uint64_t deadline = gtimer() + P.timeout_ns;
    if (tid == 0) {
        trace(P, LS_B200_TRACE_ENTRY);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&t->full_bar[s]), 33);                // producer lane 0 + 32 cp.async lanes
            mbar_init(smem_u32(&t->empty_bar[s]), kConsumerWarps);  // one arrive per consumer warp
        }
        t->warps_done = 0;
        t->abort = 0;
        t->xready = 0;
        t->partials = 0;
        t->last = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (tid >= kConsumerThreads) {
        run_producer(P, stages, t, deadline);
    } else {
        run_consumers<MAXC>(P, stages, t, deadline);
    }
    __syncthreads();
    if (tid == 0) {
        trace(P, LS_B200_TRACE_REDUCED);
        __threadfence();
        const uint32_t prev = atomicAdd(P.ws + kWsExit, 1u);
        t->last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (t->last) {
        // Every other CTA is done with the workspace: restore it to zero.
        __threadfence();
        const uint32_t nl = P.nlayers;
        for (uint32_t i = tid; i < kWsPerLayer * nl; i += blockDim.x) P.ws[kWsHeader + i] = 0;
        for (uint32_t l = 0; l < nl; ++l)
            for (uint32_t i = tid; i < P.N; i += blockDim.x) done_h(P, l)[i] = 0;
        __syncthreads();
        if (tid == 0) {
            const uint32_t err = P.ws[kWsErr];
            if (err) {
                st_relaxed_sys(P.status + LS_B200_STATUS_ERROR_EPOCH, plan_at(P, 0).epoch);
                st_relaxed_sys(P.status + LS_B200_STATUS_ERROR_DETAIL, P.ws[kWsDetail]);
                st_release_sys(P.status + LS_B200_STATUS_ERROR, err);
            }
            P.ws[kWsErr] = 0;
            P.ws[kWsDetail] = 0;
            P.ws[kWsExit] = 0;
            __threadfence();
            for (uint32_t l = 0; l < nl; ++l) {
                const LayerPlan& L = plan_at(P, l);
                st_release_sys(P.done + L.layer, L.epoch);
            }
            st_relaxed_sys(P.status + LS_B200_STATUS_LAUNCHES, P.seq);
        }
    }
    if (tid == 0) trace(P, LS_B200_TRACE_EXIT);
}

template <int MAXC>
static int launch_t(const KernelParams& p, int grid, cudaStream_t stream) {
    fused_mlp_kernel<MAXC><<<grid, kThreads, kernel_smem_bytes(), stream>>>(p);
    return int(cudaGetLastError());
}

int prepare_kernels() {
    const int bytes = int(kernel_smem_bytes());
    cudaError_t e = cudaFuncSetAttribute(fused_mlp_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fused_mlp_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fused_mlp_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    return int(e);
}

int launch_fused(const KernelParams& p, int grid, cudaStream_t stream) {
    const uint32_t hc = p.H / 32;
    if (hc <= 32) return launch_t<1>(p, grid, stream);
    if (hc <= 64) return launch_t<2>(p, grid, stream);
    return launch_t<4>(p, grid, stream);
}

}  // namespace lsb
