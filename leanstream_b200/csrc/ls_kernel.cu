// Fused sparse INT4 SwiGLU MLP layer for sm_100a.
//
// One persistent launch replaces the reference's three-launch chain
// A core_kernel -> B consumer -> reduction (kernels/streaming_mlp.cu:44-93;
// backends/triton/core.py:20-64, persistent.py:33-92, reduction.py:6-28).
//
// CTA = 8 consumer warps + 1 producer warp. The producer streams packed INT4
// rows and fp16 scales into a 6-stage shared-memory ring with
// cp.async.bulk (TMA bulk copies, no multicast) and cp.async, completing an
// mbarrier per stage. Consumers dequantise and accumulate on CUDA cores.
//
// Work is expressed as "pieces" that the producer describes in shared memory:
//   GATEUP piece: up to 32 neurons' gate+up rows  -> h = fp16(fp16(SiLU(g)) * u)
//   DOWN piece:   rows x column-range of the down matrix of one descriptor
//                 -> fp32 partial row segment (one partial row per descriptor)
// Two schedules produce pieces:
//   fast path (every queue descriptor ready at decision time, or BatchCompat):
//     static, balanced split of all neurons (GATEUP) and all (descriptor,
//     32-column chunk) pairs (DOWN) over the grid; DOWN pieces wait on a
//     per-descriptor counter of published h values.
//   progressive path: CTAs claim descriptor positions in ready order from a
//     device-memory counter (core descriptors first) and run all pieces of the
//     claimed descriptor.
// Both schedules compute every partial row with the same canonical arithmetic:
//   g, u  : per lane, chunks j = lane + 32 i, 4 pair accumulators, then a
//           fixed xor-butterfly over the warp;
//   down  : per column, one fp32 chain over the descriptor's neurons in order;
//   y     : per column, 8 interleaved row subsets summed in order.
// so BatchCompat and Progressive outputs are bit-identical, as the reference
// test requires (tests/persistent_mlp_test.cu:65).
//
// Rounding boundaries follow backends/triton/core.py:17,49-52 and
// reduction.py:15: w = fp16(q*s), g,u -> fp16, SiLU -> fp16, h -> fp16,
// fp32 partials, y -> fp16 once.
#include <cuda_fp16.h>
#include <stdint.h>
#include "ls_internal.h"

namespace lsb {

enum : uint32_t { kPieceEnd = 0, kPieceGateUp = 1, kPieceDown = 2 };
enum : uint32_t { kFirstRows = 1u, kLastRows = 2u, kCompletes = 4u };

struct Piece {
    uint32_t kind;
    uint32_t row;     // partial row = descriptor position (core first, then queue index)
    uint32_t dest;    // descriptor dest_slot (activation / counter index)
    uint32_t n0;      // GATEUP: first neuron; DOWN: first row of the down matrix
    uint32_t count;   // GATEUP: neurons; DOWN: rows
    uint32_t k0;      // DOWN: first 16-byte chunk (32 columns)
    uint32_t chunks;  // DOWN: 16-byte chunks per row
    uint32_t sb0;     // DOWN: first scale index (even) of the column range
    uint32_t nsb;     // DOWN: scale halves per row (even)
    uint32_t flags;
    uint32_t pad[6];
};
static_assert(sizeof(Piece) == 64, "piece record");

// Wait bounds, ordered so that a stalled launch always drains its ring:
// host-publication and h waits end at the deadline, the producer's wait for
// a free stage 1 s later, the consumers' wait for a full stage 2 s later and
// the grid barrier 3 s later.
constexpr uint64_t kProducerGraceNs = 1000000000ull;
constexpr uint64_t kConsumerGraceNs = 2000000000ull;
constexpr uint64_t kBarrierGraceNs = 3000000000ull;

struct SmemTail {
    unsigned long long full_bar[kStages];
    unsigned long long empty_bar[kStages];
    Piece piece[kStages];
    __half hs[kConsumerWarps * kMaxGroupSize];
    uint32_t good;
    float red[kConsumerWarps * 33];
    volatile uint32_t abort;
    uint32_t pad[3];
};

size_t kernel_smem_bytes() { return size_t(kStages) * kStageBytes + sizeof(SmemTail); }

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory");
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

__device__ __forceinline__ void trace(const KernelParams& P, uint32_t word) {
    if (P.trace) P.trace[size_t(blockIdx.x) * LS_B200_TRACE_WORDS + word] = gtimer();
}

// Records the first error of this launch and asks the CTA to stop.
__device__ __forceinline__ void raise_error(const KernelParams& P, SmemTail* t, uint32_t code, uint32_t detail) {
    if (atomicCAS(&P.ws->err, 0u, code) == 0u) P.ws->detail = detail;
    t->abort = 1;
}

// ------------------------------------------------------------ descriptors
struct DescView {
    const uint8_t* src;  // packed group base
    uint32_t phys, dest, row;
    bool ok;
};

// Descriptor at canonical position d: core[d] for d < core_count, else the
// queue descriptor published at ready position d - core_count
// (streaming_mlp.cu:60, persistent.py:80). Partial row: d for core, else
// core_count + descriptor index (custom_triton.md:54).
__device__ DescView load_desc(const KernelParams& P, uint32_t d) {
    ls_exec_desc e;
    uint32_t row;
    if (d < P.core_count) {
        const uint32_t* c = reinterpret_cast<const uint32_t*>(P.core + d);
        e.logical_group = ld_relaxed_sys(c + 0);
        e.physical_group = ld_relaxed_sys(c + 1);
        e.source_slot = ld_relaxed_sys(c + 2);
        e.dest_slot = ld_relaxed_sys(c + 3);
        e.source_kind = ld_relaxed_sys(c + 4);
        row = d;
    } else {
        const uint32_t idx = ld_relaxed_sys(P.q.ready_indices + (d - P.core_count));
        DescView bad{nullptr, 0, 0, 0, false};
        if (idx >= P.q.capacity) return bad;
        const uint32_t* c = reinterpret_cast<const uint32_t*>(P.q.descriptors + idx);
        e.logical_group = ld_relaxed_sys(c + 0);
        e.physical_group = ld_relaxed_sys(c + 1);
        e.source_slot = ld_relaxed_sys(c + 2);
        e.dest_slot = ld_relaxed_sys(c + 3);
        e.source_kind = ld_relaxed_sys(c + 4);
        row = P.core_count + idx;
    }
    DescView v;
    v.ok = e.source_kind <= 1u && e.dest_slot < P.N && row < P.N &&
           (P.phys_groups == 0 || e.physical_group < P.phys_groups) &&
           (e.source_kind == 0 ? (P.cache_slots == 0 || e.source_slot < P.cache_slots)
                               : (P.staging_slots == 0 || e.source_slot < P.staging_slots));
    v.src = (e.source_kind == 0 ? P.cache : P.staging) + size_t(e.source_slot) * P.group_bytes;
    v.phys = e.physical_group;
    v.dest = e.dest_slot;
    v.row = row;
    return v;
}

// ------------------------------------------------------------ producer side
struct Producer {
    uint32_t idx;        // pieces issued so far (stage = idx % kStages)
    uint32_t lane;
    uint8_t* stages;
    SmemTail* t;
    uint64_t deadline;
};

// Waits until stage s is free; lane 0 polls, the warp learns the result.
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

// Publishes the END marker so consumers leave their loop. Always completes.
__device__ void producer_end(Producer& pr, const KernelParams& P) {
    const uint32_t s = pr.idx % kStages;
    if (!producer_acquire_stage(pr, P)) {
        // The ring never drained: consumers already stopped. Nothing to publish.
        return;
    }
    if (pr.lane == 0) {
        pr.t->piece[s].kind = kPieceEnd;
        mbar_arrive_expect_tx(smem_u32(&pr.t->full_bar[s]), 0);
    }
    cp_async_arrive_noinc(smem_u32(&pr.t->full_bar[s]));
    ++pr.idx;
}

// GATEUP piece: neurons [n0, n0+count) of one descriptor.
__device__ bool producer_gateup(Producer& pr, const KernelParams& P, const DescView& d, uint32_t n0, uint32_t count) {
    if (!producer_acquire_stage(pr, P)) return false;
    const uint32_t s = pr.idx % kStages;
    uint8_t* st = pr.stages + size_t(s) * kStageBytes;
    const uint32_t bar = smem_u32(&pr.t->full_bar[s]);
    const uint32_t H = P.H;
    const uint64_t rec = uint64_t(3) * H / 2;  // bytes per neuron record
    if (pr.lane == 0) {
        Piece& pc = pr.t->piece[s];
        pc.kind = kPieceGateUp;
        pc.row = d.row;
        pc.dest = d.dest;
        pc.n0 = n0;
        pc.count = count;
        mbar_arrive_expect_tx(bar, count * H);
        for (uint32_t k = 0; k < count; ++k)
            bulk_g2s(smem_u32(st + size_t(k) * H), d.src + (n0 + k) * rec, H, bar);
    }
    // gate+up scales: H/128 words per neuron, at the start of its scale row.
    const uint32_t wpn = H / 128;  // 4-byte words per neuron
    const uint32_t words = count * wpn;
    const uint32_t sdst = smem_u32(st + kStageData);
    for (uint32_t i = pr.lane; i < words; i += 32) {
        const uint32_t k = i / wpn, w = i % wpn;
        const uint16_t* src = P.scales + (size_t(d.phys) * P.G + n0 + k) * (3 * H / 128) + 2 * w;
        cp_async4(sdst + 4 * i, src);
    }
    cp_async_arrive_noinc(bar);
    ++pr.idx;
    return true;
}

// DOWN piece: rows [r0, r0+rows) x chunks [k0, k0+m) of one descriptor.
__device__ bool producer_down(Producer& pr, const KernelParams& P, const DescView& d, uint32_t r0, uint32_t rows,
                              uint32_t k0, uint32_t m, uint32_t flags) {
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
            P.scales + (size_t(d.phys) * P.G + r0 + r) * (3 * H / 128) + 2 * (H / 128) + sb0 + 2 * w;
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
    uint32_t n = kStageData / P.H;
    return n < 32u ? n : 32u;
}

// All pieces of one descriptor (progressive path).
__device__ bool producer_descriptor(Producer& pr, const KernelParams& P, const DescView& d) {
    const uint32_t G = P.G, hc = P.H / 32;
    const uint32_t np = gateup_neurons(P);
    for (uint32_t n = 0; n < G; n += np) {
        const uint32_t c = (G - n) < np ? (G - n) : np;
        if (!producer_gateup(pr, P, d, n, c)) return false;
    }
    const uint32_t rr = down_rows(P), mm = down_chunks(P);
    for (uint32_t k = 0; k < hc; k += mm) {
        const uint32_t m = (hc - k) < mm ? (hc - k) : mm;
        for (uint32_t r = 0; r < G; r += rr) {
            const uint32_t rows = (G - r) < rr ? (G - r) : rr;
            uint32_t f = 0;
            if (r == 0) f |= kFirstRows;
            if (r + rows == G) f |= kLastRows;
            if (r + rows == G && k + m == hc) f |= kCompletes;
            if (!producer_down(pr, P, d, r, rows, k, m, f)) return false;
        }
    }
    return true;
}

__device__ void stamp(const KernelParams& P, const DescView& d) {
    if (P.stamps) P.stamps[d.dest] = gtimer();
}

// Leader decision: waits for the epoch (and batch epoch), then publishes the
// consumer path to the device workspace (streaming_mlp.cu:49-56,
// persistent.py:46-55; consumer_path lives in device memory here).
__device__ void leader_decide(const KernelParams& P, SmemTail* t, uint64_t deadline) {
    const ls_queue_control* c = P.q.control;
    const uint32_t* words = reinterpret_cast<const uint32_t*>(c);
    uint32_t code = 0;
    for (;;) {
        if (ld_acquire_sys(words + 5)) { code = LS_B200_DEV_QUEUE_ERROR; break; }
        if (ld_acquire_sys(words + 3) == P.epoch) break;
        if (gtimer() > deadline) { code = LS_B200_DEV_TIMEOUT_EPOCH; break; }
        __nanosleep(128);
    }
    const bool batch = P.mode != LS_MODE_PROGRESSIVE;  // Auto follows BatchCompat
    if (!code && batch) {
        for (;;) {
            if (ld_acquire_sys(words + 5)) { code = LS_B200_DEV_QUEUE_ERROR; break; }
            if (ld_acquire_sys(words + 4) == P.epoch) break;
            if (gtimer() > deadline) { code = LS_B200_DEV_TIMEOUT_EPOCH; break; }
            __nanosleep(128);
        }
    }
    uint32_t total = 0, path = kPathAbort;
    if (!code) {
        total = ld_relaxed_sys(words + 2);
        const uint32_t ready = ld_acquire_sys(words + 0);
        if (total > P.q.capacity || P.core_count + total > P.N || ready > total)
            code = LS_B200_DEV_BAD_PLAN;
        else
            path = ready == total ? kPathFast : kPathProgressive;
    }
    if (code) raise_error(P, t, code, 0);
    P.ws->total = total;
    st_release_gpu(&P.ws->path, path);
}

// Producer warp main loop.
__device__ void run_producer(const KernelParams& P, uint8_t* stages, SmemTail* t, uint64_t deadline) {
    Producer pr{0, threadIdx.x & 31u, stages, t, deadline};
    // 1. Path decision (CTA 0 lane 0 decides; everyone else waits for it).
    uint32_t path = 0, total = 0;
    if (pr.lane == 0) {
        if (blockIdx.x == 0) leader_decide(P, t, deadline);
        for (;;) {
            path = ld_acquire_gpu(&P.ws->path);
            if (path) break;
            if (gtimer() > deadline) { raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 2); path = kPathAbort; break; }
            __nanosleep(64);
        }
        total = P.ws->total;
        if (path == kPathAbort) t->abort = 1;
    }
    path = __shfl_sync(0xffffffffu, path, 0);
    total = __shfl_sync(0xffffffffu, total, 0);
    if (pr.lane == 0) trace(P, LS_B200_TRACE_DECIDED);
    const uint32_t D = P.core_count + total;

    if (path == kPathFast) {
        // Order later descriptor reads after the host's publication.
        if (pr.lane == 0 && P.q.control) (void)ld_acquire_sys(reinterpret_cast<const uint32_t*>(P.q.control));
        __syncwarp();
        const uint32_t G = P.G, hc = P.H / 32;
        const uint64_t NT = uint64_t(D) * G, CT = uint64_t(D) * hc;
        const uint32_t b = blockIdx.x, grid = gridDim.x;
        // GATEUP pieces over this CTA's neuron range.
        uint64_t u = NT * b / grid;
        const uint64_t u1 = NT * (b + 1) / grid;
        const uint32_t np = gateup_neurons(P);
        uint32_t cur = 0xffffffffu;
        DescView dv{};
        bool ok = !t->abort;
        while (ok && u < u1) {
            const uint32_t d = uint32_t(u / G), n = uint32_t(u % G);
            if (d != cur) {
                dv = load_desc(P, d);
                cur = d;
                if (!dv.ok) { if (pr.lane == 0) raise_error(P, t, LS_B200_DEV_BAD_DESCRIPTOR, d); ok = false; break; }
                if (n == 0 && pr.lane == 0) stamp(P, dv);
            }
            uint32_t c = G - n;
            if (c > np) c = np;
            if (u + c > u1) c = uint32_t(u1 - u);
            ok = producer_gateup(pr, P, dv, n, c) && !t->abort;
            u += c;
        }
        // DOWN pieces over this CTA's (descriptor, chunk) range.
        uint64_t v = CT * b / grid;
        const uint64_t v1 = CT * (b + 1) / grid;
        const uint32_t rr = down_rows(P), mm = down_chunks(P);
        while (ok && v < v1) {
            const uint32_t d = uint32_t(v / hc), k = uint32_t(v % hc);
            if (d != cur) {
                dv = load_desc(P, d);
                cur = d;
                if (!dv.ok) { if (pr.lane == 0) raise_error(P, t, LS_B200_DEV_BAD_DESCRIPTOR, d); ok = false; break; }
            }
            uint32_t m = hc - k;
            if (m > mm) m = mm;
            if (v + m > v1) m = uint32_t(v1 - v);
            for (uint32_t r = 0; ok && r < G; r += rr) {
                const uint32_t rows = (G - r) < rr ? (G - r) : rr;
                uint32_t f = 0;
                if (r == 0) f |= kFirstRows;
                if (r + rows == G) f |= kLastRows;
                if (r + rows == G && k + m == hc) f |= kCompletes;
                ok = producer_down(pr, P, dv, r, rows, k, m, f) && !t->abort;
            }
            v += m;
        }
    } else if (path == kPathProgressive) {
        const uint32_t* words = reinterpret_cast<const uint32_t*>(P.q.control);
        bool ok = true;
        while (ok && !t->abort) {
            uint32_t pos = 0, code = 0;
            if (pr.lane == 0) {
                pos = atomicAdd(&P.ws->claim, 1u);
                if (pos >= D) {
                    code = 0xffffffffu;  // exhausted
                } else if (pos >= P.core_count) {
                    // Wait until the claimed queue position is published
                    // (persistent.py:71-90; streaming_mlp.cu:63-75).
                    const uint32_t q = pos - P.core_count;
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
            const DescView dv = load_desc(P, pos);
            if (!dv.ok) { if (pr.lane == 0) raise_error(P, t, LS_B200_DEV_BAD_DESCRIPTOR, pos); break; }
            if (pr.lane == 0) stamp(P, dv);
            ok = producer_descriptor(pr, P, dv);
        }
    }
    producer_end(pr, P);
    if (pr.lane == 0) trace(P, LS_B200_TRACE_PRODUCED);
}

// ------------------------------------------------------------ consumer side
template <int MAXC>
struct Activation {
    __half2 x[MAXC][16];  // chunk i of this lane: pairs (c, c+4) per 8-coordinate word
};

// Loads the lane's activation chunks, optionally through the HF RMSNorm of
// examples/ministral/native/predictor_shared_input.cu:16-33:
// inv = rsqrt(sum(x^2)/H + eps); x' = fp16(weight * fp16(x * inv)).
template <int MAXC>
__device__ void load_activation(const KernelParams& P, SmemTail* t, Activation<MAXC>& a, int tid) {
    const uint32_t H = P.H, hc = H / 32;
    const int lane = tid & 31, warp = tid >> 5;
    float inv = 1.f;
    const bool norm = (P.flags & LS_B200_NORM_INPUT) != 0;
    if (norm) {
        float s = 0.f;
        for (uint32_t c = tid; c < H; c += kConsumerThreads) {
            const float v = h2f(P.x[c]);
            s += v * v;
        }
        s = warp_sum(s);
        if (lane == 0) t->red[warp] = s;
        consumer_sync();
        float total = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) total += t->red[w];
        consumer_sync();
        inv = rsqrtf(total / float(H) + P.eps);
    }
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
        const uint32_t j = lane + 32 * i;
        if (j < hc) {
#pragma unroll
            for (int w = 0; w < 4; ++w) {
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const uint32_t c0 = 32 * j + 8 * w + p, c1 = c0 + 4;
                    __half lo = __ushort_as_half(P.x[c0]), hi = __ushort_as_half(P.x[c1]);
                    if (norm) {
                        lo = __float2half_rn(__half2float(lo) * inv);
                        hi = __float2half_rn(__half2float(hi) * inv);
                        if (P.norm_w) {
                            lo = __hmul(__ushort_as_half(P.norm_w[c0]), lo);
                            hi = __hmul(__ushort_as_half(P.norm_w[c1]), hi);
                        }
                    }
                    a.x[i][4 * w + p] = __halves2half2(lo, hi);
                }
            }
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) a.x[i][k] = __float2half2_rn(0.f);
        }
    }
}

__device__ __forceinline__ uint32_t* done_h(const KernelParams& P) {
    return reinterpret_cast<uint32_t*>(P.ws + 1);
}

template <int MAXC>
__device__ void consume_gateup(const KernelParams& P, const Piece& pc, const uint8_t* st, const Activation<MAXC>& a,
                               int warp, int lane) {
    const uint32_t H = P.H, hc = H / 32;
    const __half* sc = reinterpret_cast<const __half*>(st + kStageData);
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
            if (P.act) P.act[size_t(pc.dest) * P.G + n] = __half_as_ushort(h);
            red_release_gpu(done_h(P) + pc.row, 1u);
        }
    }
}

// DOWN piece: thread owns 8 columns (4 packed bytes) of the range.
__device__ void consume_down(const KernelParams& P, const Piece& pc, const uint8_t* st, const __half* hs,
                             float (&acc)[8], int tid) {
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

// Per-warp staging of the h values of `row`: lane 0 waits (bounded) until all
// G neurons of the row have published h (release/acquire at gpu scope), then
// the warp copies them into its private shared-memory slice. No CTA-wide
// barrier is involved, so a warp that leaves early can never strand others.
__device__ void stage_h_warp(const KernelParams& P, SmemTail* t, uint32_t row, int lane, __half* hs,
                             uint64_t deadline) {
    if (lane == 0) {
        const uint32_t* cnt = done_h(P) + row;
        uint32_t spins = 0;
        while (ld_acquire_gpu(cnt) < P.G) {
            if (t->abort) break;
            if ((++spins & 63u) == 0 && gtimer() > deadline) {
                raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 3);
                break;
            }
            __nanosleep(32);
        }
    }
    __syncwarp();
    for (uint32_t n = lane; n < P.G; n += 32) hs[n] = __ushort_as_half(__ldcg(P.hbuf + size_t(row) * P.G + n));
    __syncwarp();
}

template <int MAXC>
__device__ void run_consumers(const KernelParams& P, uint8_t* stages, SmemTail* t, uint64_t deadline) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __half* hs = t->hs + warp * kMaxGroupSize;
    Activation<MAXC> a;
    load_activation<MAXC>(P, t, a, tid);
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (uint32_t idx = 0;; ++idx) {
        const uint32_t s = idx % kStages;
        const uint32_t parity = (idx / kStages) & 1u;
        const uint32_t bar = smem_u32(&t->full_bar[s]);
        // Every lane waits on the mbarrier (acquire of the TMA-written data);
        // the loop condition is warp-uniform so the warp never diverges here.
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
            // The producer stopped without END: nothing is in flight for this
            // stage. Leave the loop; later code has no intra-loop barriers.
            raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 4);
            break;
        }
        const Piece pc = t->piece[s];
        if (idx == 0 && tid == 0) trace(P, LS_B200_TRACE_FIRST);
        if (pc.kind == kPieceEnd) {
            if (tid == 0) trace(P, LS_B200_TRACE_PIECES);
            break;
        }
        const uint8_t* st = stages + size_t(s) * kStageBytes;
        const bool aborted = __shfl_sync(0xffffffffu, t->abort, 0) != 0;  // warp-uniform snapshot
        if (pc.kind == kPieceGateUp) {
            if (!aborted) consume_gateup<MAXC>(P, pc, st, a, warp, lane);
        } else {
            if (pc.flags & kFirstRows) {
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = 0.f;
                if (uint32_t(warp * 32) < 4 * pc.chunks && !aborted) stage_h_warp(P, t, pc.row, lane, hs, deadline);
            }
            if (!aborted) {
                consume_down(P, pc, st, hs, acc, tid);
                if ((pc.flags & kLastRows) && uint32_t(tid) < 4 * pc.chunks) {
                    float* dst = P.partial + size_t(pc.row) * P.H + 32 * pc.k0 + 8 * tid;
                    reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
                    reinterpret_cast<float4*>(dst)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
                }
                if ((pc.flags & kCompletes) && tid == 0 && P.execs) atomicAdd(P.execs + pc.dest, 1u);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&t->empty_bar[s]));
    }
}

// Canonical compact reduction (reduction.py:6-28, streaming_mlp.cu:80-84):
// y[c] = sum over 8 interleaved row subsets, each summed in row order.
__device__ void run_reduction(const KernelParams& P, SmemTail* t, uint32_t rows) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t H = P.H;
    for (uint32_t blk = blockIdx.x; blk < H / 32; blk += gridDim.x) {
        const uint32_t c = 32 * blk + lane;
        float s = 0.f;
        for (uint32_t r = warp; r < rows; r += kConsumerWarps) s += __ldcg(P.partial + size_t(r) * H + c);
        t->red[warp * 33 + lane] = s;
        consumer_sync();
        if (warp == 0) {
            float y = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) y += t->red[w * 33 + lane];
            if (P.y32) P.y32[c] = y;
            const __half y16 = __float2half_rn(y);
            if (P.y && !(P.flags & LS_B200_NO_OUTPUT)) P.y[c] = __half_as_ushort(y16);
            if (P.hidden_out && P.residual)
                P.hidden_out[c] = __half_as_ushort(__float2half_rn(h2f(P.residual[c]) + __half2float(y16)));
        }
        consumer_sync();
    }
}

template <int MAXC>
__global__ void __launch_bounds__(kThreads, 1) fused_layer_kernel(const KernelParams P) {
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
        t->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (tid >= kConsumerThreads) {
        run_producer(P, stages, t, deadline);
    } else {
        run_consumers<MAXC>(P, stages, t, deadline);
    }
    __syncthreads();

    // Grid barrier: every partial row of this launch is written.
    Workspace* ws = P.ws;
    if (tid == 0) {
        __threadfence();
        atomicAdd(&ws->arrive, 1u);
        uint32_t spins = 0;
        while (ld_acquire_gpu(&ws->arrive) < gridDim.x) {
            if ((++spins & 63u) == 0 && gtimer() > deadline + kBarrierGraceNs) {
                raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 5);
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
        // One CTA-uniform decision: reduce only a complete, error-free launch.
        const uint32_t path = ld_acquire_gpu(&ws->path);
        t->good = (path == kPathFast || path == kPathProgressive) && ld_acquire_gpu(&ws->err) == 0 && !t->abort;
        trace(P, LS_B200_TRACE_BARRIER);
    }
    __syncthreads();
    if (t->good && tid < kConsumerThreads) run_reduction(P, t, P.core_count + ws->total);
    __syncthreads();
    if (tid == 0) trace(P, LS_B200_TRACE_REDUCED);

    // Exit: the last CTA restores the workspace and publishes completion.
    if (tid == 0) {
        __threadfence();
        const uint32_t prev = atomicAdd(&ws->exit, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence();
            const uint32_t err = ws->err;
            if (err && P.status[LS_B200_STATUS_ERROR] == 0) {
                P.status[LS_B200_STATUS_ERROR_EPOCH] = P.epoch;
                P.status[LS_B200_STATUS_ERROR_DETAIL] = ws->detail;
                st_release_sys(P.status + LS_B200_STATUS_ERROR, err);
            }
            uint32_t* dh = done_h(P);
            for (uint32_t r = 0; r < P.N; ++r) dh[r] = 0;
            ws->path = 0;
            ws->total = 0;
            ws->claim = 0;
            ws->arrive = 0;
            ws->err = 0;
            ws->detail = 0;
            __threadfence();
            ws->exit = 0;
            __threadfence_system();
            P.status[LS_B200_STATUS_LAUNCHES] += 1;
            st_release_sys(P.done + P.layer, P.epoch);
        }
        trace(P, LS_B200_TRACE_EXIT);
    }
}

template <int MAXC>
static int launch_t(const KernelParams& p, int grid, cudaStream_t stream) {
    fused_layer_kernel<MAXC><<<grid, kThreads, kernel_smem_bytes(), stream>>>(p);
    return int(cudaGetLastError());
}

int prepare_kernels() {
    const int bytes = int(kernel_smem_bytes());
    cudaError_t e = cudaFuncSetAttribute(fused_layer_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fused_layer_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fused_layer_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    return int(e);
}

int launch_fused_layer(const KernelParams& p, int grid, cudaStream_t stream) {
    const uint32_t hc = p.H / 32;
    if (hc <= 32) return launch_t<1>(p, grid, stream);
    if (hc <= 64) return launch_t<2>(p, grid, stream);
    return launch_t<4>(p, grid, stream);
}

}  // namespace lsb
