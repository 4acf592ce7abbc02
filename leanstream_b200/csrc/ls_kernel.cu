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
//   g, u : the hidden dimension is split into 8 fixed slices, one per
//          consumer warp; each warp reduces its slice for 8 neurons at a time
//          (tensor-core mma.sync m16n8k16 with the 8 gate rows and 8 up rows
//          as A and x as column 0 of B, or CUDA-core fp16xfp16->fp32 fmas with
//          the same data mapping), and the 8 slice sums are added in warp
//          order by the last warp to finish the piece;
//   down : per column, one fp32 chain over the descriptor's neurons in order;
//   y    : per column, partial rows summed in row order.
// h travels between CTAs as 64-bit words (launch/layer tag << 32 | fp16 h):
// the tag makes a single relaxed store self-validating, so publishing h
// needs no fence or counter. The producer warp polls those words and copies
// h into the DOWN piece's stage, off the consumers' critical path.
// Rounding boundaries (core.py:17,49-52; reduction.py:15): w = fp16(q*s),
// g,u -> fp16, SiLU -> fp16, h -> fp16, fp32 partials, y -> fp16 once.
//
// Synchronisation uses counters and tagged words with bounded waits only --
// no named barriers inside loops -- so a warp that gives up can never strand
// the others. Every wait ends at a %globaltimer deadline and records an error.
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
    uint32_t gcnt[kStages];  // warps done with a GATEUP piece (per stage)
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
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
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
// Tensor-core step: D(16x8,f32) += A(16x16,f16) * B(16x8,f16).
__device__ __forceinline__ void mma16816(float (&d)[4], __half2 a0, __half2 a1, __half2 a2, __half2 a3, __half2 b0,
                                         __half2 b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(*reinterpret_cast<uint32_t*>(&a0)), "r"(*reinterpret_cast<uint32_t*>(&a1)),
          "r"(*reinterpret_cast<uint32_t*>(&a2)), "r"(*reinterpret_cast<uint32_t*>(&a3)),
          "r"(*reinterpret_cast<uint32_t*>(&b0)), "r"(*reinterpret_cast<uint32_t*>(&b1)));
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
// Tag of h words written by layer l of this launch (never 0: seq >= 1).
__device__ __forceinline__ unsigned long long h_tag(const KernelParams& P, uint32_t l) {
    return (static_cast<unsigned long long>((P.seq << 8) | (l & 0xffu))) << 32;
}
__device__ __forceinline__ void trace(const KernelParams& P, uint32_t word) {
    if (P.trace) P.trace[size_t(blockIdx.x) * LS_B200_TRACE_WORDS + word] = gtimer();
}
// Per-piece stamps of CTAs 0..3 after the per-layer block:
// [4][LS_B200_PIECE_TRACE_PIECES][4] = issued, closed (producer), ready, done (consumer warp 0).
__device__ __forceinline__ void trace_piece(const KernelParams& P, uint32_t piece, uint32_t word) {
    if (P.trace && blockIdx.x < 4 && piece < LS_B200_PIECE_TRACE_PIECES)
        P.trace[size_t(gridDim.x) * LS_B200_TRACE_WORDS + size_t(gridDim.x) * P.nlayers * LS_B200_LAYER_TRACE_WORDS +
                (size_t(blockIdx.x) * LS_B200_PIECE_TRACE_PIECES + piece) * 4 + word] = gtimer();
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
// A DOWN stage whose rows are in flight but whose h values are not yet
// staged: the producer keeps issuing later pieces and closes it once the
// tagged h words of its rows appear.
struct OpenStage {
    uint32_t stage, hrow, rows, layer;  // hrow: first tagged word (partial row * G + r0)
    uint32_t piece;                     // piece index (trace)
};

struct Producer {
    uint32_t idx;   // pieces issued so far (stage = idx % kStages)
    uint32_t lane;
    uint8_t* stages;
    SmemTail* t;
    uint64_t deadline;
    uint32_t wbase;  // first descriptor position held in t->dtab
    uint32_t wlayer;
    OpenStage open[kStages];
    uint32_t open_head, open_count;
};

__device__ bool producer_try_close(Producer& pr, const KernelParams& P, bool blocking);

// Waits until the next stage is free, closing open DOWN stages meanwhile
// (one of them may be the stage being waited for).
__device__ bool producer_acquire_stage(Producer& pr, const KernelParams& P) {
    const uint32_t s = pr.idx % kStages;
    const uint32_t parity = ((pr.idx / kStages) & 1u) ^ 1u;
    const uint32_t bar = smem_u32(&pr.t->empty_bar[s]);
    uint32_t spins = 0;
    for (;;) {
        uint32_t ready = 0;
        if (pr.lane == 0) ready = mbar_try_wait(bar, parity) ? 1u : 0u;
        if (__shfl_sync(0xffffffffu, ready, 0)) return true;
        if (pr.open_count && producer_try_close(pr, P, false)) continue;
        __nanosleep(spins < 64 ? 64 : 256);  // back off: keep L2 free for the consumers
        uint32_t late = 0;
        if (pr.lane == 0 && (++spins & 255u) == 0 && gtimer() > pr.deadline + kProducerGraceNs) late = 1;
        if (__shfl_sync(0xffffffffu, late, 0)) {
            if (pr.lane == 0) raise_error(P, pr.t, LS_B200_DEV_TIMEOUT_SYNC, 1);
            return false;
        }
    }
}

// Completes a stage: 32 cp.async arrivals (one per lane, when its scale /
// h copies land) plus one release arrival by lane 0 after the warp's
// shared-memory writes. The full barrier expects 34 arrivals in total.
__device__ __forceinline__ void producer_close(Producer& pr, uint32_t s) {
    const uint32_t bar = smem_u32(&pr.t->full_bar[s]);
    cp_async_arrive_noinc(bar);
    __syncwarp();
    if (pr.lane == 0) mbar_arrive(bar);
}
__device__ __forceinline__ void producer_stamp(const KernelParams& P, const Producer& pr, uint32_t piece,
                                               uint32_t word) {
    if (pr.lane == 0) trace_piece(P, piece, word);
}

// Tries to close the oldest open DOWN stage: polls the tagged h words of its
// rows once (or until they appear / the deadline passes, when blocking).
__device__ bool producer_try_close(Producer& pr, const KernelParams& P, bool blocking) {
    if (!pr.open_count) return true;
    const OpenStage o = pr.open[pr.open_head];
    const unsigned long long tag = h_tag(P, o.layer);
    uint32_t hv = 0, spins = 0;
    bool ok_all = false;
    for (;;) {
        uint32_t ok = 1;
        if (pr.lane < o.rows) {
            const unsigned long long w = ld_relaxed_gpu_u64(P.hbuf + o.hrow + pr.lane);
            ok = (w & 0xffffffff00000000ull) == tag;
            hv = uint32_t(w) & 0xffffu;
        }
        if (__all_sync(0xffffffffu, ok)) { ok_all = true; break; }
        if (!blocking) return false;
        uint32_t late = 0;
        if (pr.lane == 0 && (++spins & 63u) == 0 && (pr.t->abort || gtimer() > pr.deadline)) late = 1;
        if (__shfl_sync(0xffffffffu, late, 0)) break;
        __nanosleep(32);
    }
    if (!ok_all && pr.lane == 0 && !pr.t->abort) raise_error(P, pr.t, LS_B200_DEV_TIMEOUT_SYNC, 3);
    uint8_t* st = pr.stages + size_t(o.stage) * kStageBytes;
    if (pr.lane < o.rows) reinterpret_cast<uint16_t*>(st + kStageData + kAuxSecond)[pr.lane] = uint16_t(hv);
    producer_close(pr, o.stage);
    producer_stamp(P, pr, o.piece, 1);
    pr.open_head = (pr.open_head + 1) % kStages;
    --pr.open_count;
    return ok_all;
}

__device__ void producer_flush(Producer& pr, const KernelParams& P) {
    while (pr.open_count) producer_try_close(pr, P, true);
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
    producer_stamp(P, pr, pr.idx, 0);
    producer_close(pr, s);
    producer_stamp(P, pr, pr.idx, 1);
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
        // rows at a pitch of H + 16 bytes: the consumers' 4-byte loads of 8
        // rows then hit 32 distinct banks
        for (uint32_t k = 0; k < count; ++k)
            bulk_g2s(smem_u32(st + size_t(k) * (H + 16)), d.src + (n0 + k) * rec, H, bar);
    }
    // gate+up scales: H/128 words per neuron, at the start of its scale row;
    // staged at a pitch of H/128 + 1 words so that 8 neurons' scales sit in
    // 8 different banks.
    const uint32_t wpn = H / 128;
    const uint32_t words = count * wpn;
    const uint32_t sdst = smem_u32(st + kStageData);
    for (uint32_t i = pr.lane; i < words; i += 32) {
        const uint32_t k = i / wpn, w = i % wpn;
        const uint16_t* src = L.scales + (size_t(d.phys) * P.G + n0 + k) * (3 * H / 128) + 2 * w;
        cp_async4(sdst + 4 * (k * (wpn + 1) + w), src);
    }
    producer_stamp(P, pr, pr.idx, 0);
    producer_close(pr, s);
    producer_stamp(P, pr, pr.idx, 1);
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
    // The stage stays open until the h of rows [r0, r0+rows) -- written by
    // the GATEUP pieces of this layer, in any CTA -- is staged next to it.
    const uint32_t slot = (pr.open_head + pr.open_count) % kStages;
    producer_stamp(P, pr, pr.idx, 0);
    pr.open[slot] = OpenStage{s, uint32_t(d.row * P.G + r0), rows, layer, pr.idx};
    ++pr.open_count;
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
    const uint32_t n = kStageData / (P.H + 16);
    return n < uint32_t(kGateupMax) ? n : uint32_t(kGateupMax);
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
    Producer pr;
    pr.idx = 0;
    pr.lane = threadIdx.x & 31u;
    pr.stages = stages;
    pr.t = t;
    pr.deadline = deadline;
    pr.wbase = pr.wlayer = 0xffffffffu;
    pr.open_head = pr.open_count = 0;
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
    producer_flush(pr, P);
    if (pr.lane == 0) trace(P, LS_B200_TRACE_PRODUCED);
}

// ------------------------------------------------------------ consumer side
// Register-resident activation fragments of one warp's share of the hidden
// dimension: slice w % 8 (H/8 coordinates = SB 32-coordinate sub-blocks),
// sub-blocks [half*SBH, half*SBH + SBH) with half = w / 8.
// x[b][p] = (x[c + p], x[c + p + 4]), c = sub-block start + 8 (lane & 3):
// for the tensor-core path these are the B fragments (column 0) of
// m16n8k16 for logical k = (2t, 2t+1) and (2t+8, 2t+9).
template <int SBH>
struct Frag {
    __half2 x[SBH][4];
};

template <int SB>
struct Split {
    static constexpr int SBH = SB > 1 ? SB / 2 : 1;
    __device__ static int first(int warp) { return SB > 1 ? (warp / kSlices) * SBH : 0; }
    __device__ static int count(int warp) { return SB > 1 ? SBH : (warp < kSlices ? 1 : 0); }
};

// Builds this warp's fragments from the CTA's staged activation, applying
// the HF RMSNorm of predictor_shared_input.cu:16-33 when flagged:
// inv = rsqrt(sum(x^2)/H + eps); x' = fp16(weight * fp16(x * inv)).
// The sum runs per lane over 8-coordinate groups lane*8 + 256 i, then a
// fixed butterfly: every warp of every CTA computes the same value.
template <int SB>
__device__ void load_activation(const KernelParams& P, const LayerPlan& L, const __half* xs,
                                Frag<Split<SB>::SBH>& f, int warp, int lane) {
    constexpr int SBH = Split<SB>::SBH;
    const uint32_t H = P.H;
    const bool norm = (L.flags & LS_B200_NORM_INPUT) != 0;
    float inv = 1.f;
    if (norm) {
        float ss = 0.f;
        for (uint32_t c = 8 * lane; c < H; c += 256) {
            const uint4 w = *reinterpret_cast<const uint4*>(xs + c);
            const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 v = __half22float2(h[e]);
                ss += v.x * v.x;
                ss += v.y * v.y;
            }
        }
        inv = rsqrtf(warp_sum(ss) / float(H) + P.eps);
    }
    const uint32_t base = (warp % kSlices) * (H / 8) + 32 * Split<SB>::first(warp) + 8 * (lane & 3);
#pragma unroll
    for (int b = 0; b < SBH; ++b) {
        const uint32_t c = (base + 32 * b) % H;  // in range even for an idle half (SB == 1)
        const uint4 w = *reinterpret_cast<const uint4*>(xs + c);
        const __half* h = reinterpret_cast<const __half*>(&w);
        __half v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            v[e] = h[e];
            if (norm) v[e] = __float2half_rn(__half2float(v[e]) * inv);
        }
        if (norm && L.norm_w) {
            const uint4 nw = __ldg(reinterpret_cast<const uint4*>(L.norm_w + c));
            const __half* wh = reinterpret_cast<const __half*>(&nw);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __hmul(wh[e], v[e]);
        }
#pragma unroll
        for (int p = 0; p < 4; ++p) f.x[b][p] = __halves2half2(v[p], v[p + 4]);
    }
}

// GATEUP piece: this warp's share of its hidden slice for every neuron of the
// piece, in tiles of 8 neurons; the partial sums go to the stage's partial
// area and the last warp to finish adds the 16 of them in warp order, forms h
// and publishes it.
template <int SB, bool MMA>
__device__ void consume_gateup(const KernelParams& P, const LayerPlan& L, const Piece& pc, uint8_t* st, SmemTail* t,
                               uint32_t s, const Frag<Split<SB>::SBH>& f, int warp, int lane) {
    constexpr int SBH = Split<SB>::SBH;
    const uint32_t H = P.H, pitch = H + 16;
    const int g = lane >> 2, tq = lane & 3;
    const int nsub = Split<SB>::count(warp);
    const uint32_t slice = (warp % kSlices) * (H / 8) + 32 * Split<SB>::first(warp);  // first coordinate
    const __half* sc = reinterpret_cast<const __half*>(st + kStageData);
    float2* part = reinterpret_cast<float2*>(st + kStageData + kAuxSecond);  // [warp][count]
    for (uint32_t r0 = 0; r0 < pc.count; r0 += 8) {
        const uint32_t k = r0 + g;  // neuron of the piece handled by this lane quad
        const uint8_t* row = st + size_t(k) * pitch + slice / 2 + 4 * tq;
        const __half* scr = sc + size_t(k) * 2 * (H / 128 + 1);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        float acc2[4] = {0.f, 0.f, 0.f, 0.f};  // second tensor-core chain (odd sub-blocks)
#pragma unroll
        for (int b = 0; b < SBH; ++b) {
            if (b >= nsub) break;
            const uint32_t wg = *reinterpret_cast<const uint32_t*>(row + 16 * b);
            const uint32_t wu = *reinterpret_cast<const uint32_t*>(row + H / 2 + 16 * b);
            const uint32_t blk = (slice + 32 * b) >> 7;
            const __half2 sg = __half2half2(scr[blk]);
            const __half2 su = __half2half2(scr[(H >> 7) + blk]);  // gate: H/128 halves, then up
            __half2 qg[4], qu[4];
            unpack8(wg, qg);
            unpack8(wu, qu);
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                qg[p] = __hmul2(qg[p], sg);  // == fp16(float(q) * float(s)), core.py:17
                qu[p] = __hmul2(qu[p], su);
            }
            if constexpr (MMA) {
                // rows 0-7: gate rows of the 8 neurons, rows 8-15: their up rows
                float(&d)[4] = (b & 1) ? acc2 : acc;
                mma16816(d, qg[0], qu[0], qg[1], qu[1], f.x[b][0], f.x[b][1]);
                mma16816(d, qg[2], qu[2], qg[3], qu[3], f.x[b][2], f.x[b][3]);
            } else {
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    acc[p & 1] = mfma(__low2half(qg[p]), __low2half(f.x[b][p]), acc[p & 1]);
                    acc[p & 1] = mfma(__high2half(qg[p]), __high2half(f.x[b][p]), acc[p & 1]);
                    acc[2 + (p & 1)] = mfma(__low2half(qu[p]), __low2half(f.x[b][p]), acc[2 + (p & 1)]);
                    acc[2 + (p & 1)] = mfma(__high2half(qu[p]), __high2half(f.x[b][p]), acc[2 + (p & 1)]);
                }
            }
        }
        float gs, us;
        if constexpr (MMA) {
            gs = acc[0] + acc2[0];  // D[g][0]: lane (g, 0)
            us = acc[2] + acc2[2];  // D[g+8][0]
        } else {
            gs = acc[0] + acc[1];
            us = acc[2] + acc[3];
            gs += __shfl_xor_sync(0xffffffffu, gs, 1);
            us += __shfl_xor_sync(0xffffffffu, us, 1);
            gs += __shfl_xor_sync(0xffffffffu, gs, 2);
            us += __shfl_xor_sync(0xffffffffu, us, 2);
        }
        if (tq == 0 && k < pc.count) part[warp * pc.count + k] = make_float2(gs, us);
    }
    // Last warp to finish this piece combines the partial sums.
    __syncwarp();
    __threadfence_block();
    uint32_t old = 0;
    if (lane == 0) old = atomicAdd(&t->gcnt[s], 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != uint32_t(kConsumerWarps) - 1) return;
    __threadfence_block();
    if (uint32_t(lane) < pc.count) {
        float gsum = 0.f, usum = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
            const float2 v = part[w * pc.count + lane];
            gsum += v.x;
            usum += v.y;
        }
        const float g16 = round16(gsum), u16 = round16(usum);
        const float sl = round16(g16 / (1.f + expf(-g16)));
        const uint16_t h = __half_as_ushort(__float2half_rn(sl * u16));
        const uint32_t n = pc.n0 + lane;
        st_relaxed_gpu_u64(P.hbuf + size_t(pc.row) * P.G + n, h_tag(P, pc.layer) | h);
        if (L.act) L.act[size_t(pc.dest) * P.G + n] = h;
    }
    __syncwarp();
    if (lane == 0) t->gcnt[s] = 0;
}

// DOWN piece: thread owns 8 columns (4 packed bytes) of the range and one
// half of the piece's rows (threads [0,256): first half, [256,512): second).
__device__ __forceinline__ uint32_t down_half_split(uint32_t rows) { return (rows + 1) / 2; }

__device__ void consume_down(const Piece& pc, const uint8_t* st, const __half* hs, float (&acc)[8], int tid) {
    const uint32_t pitch = 16 * pc.chunks;
    const uint32_t task = uint32_t(tid) & 255u, half = uint32_t(tid) >> 8;
    if (task >= 4 * pc.chunks) return;
    const uint32_t split = down_half_split(pc.count);
    const uint32_t rb = half ? split : 0, re = half ? pc.count : split;
    const __half* sc = reinterpret_cast<const __half*>(st + kStageData);
    const uint32_t col = 32 * pc.k0 + 8 * task;
    const uint32_t sbi = (col >> 7) - pc.sb0;
    const uint8_t* base = st + 4 * task;
    uint32_t r = rb;
    for (; r + 4 <= re; r += 4) {
        uint32_t wv[4];
        __half2 s2[4];
        __half hh[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            wv[e] = *reinterpret_cast<const uint32_t*>(base + size_t(r + e) * pitch);
            s2[e] = __half2half2(sc[(r + e) * pc.nsb + sbi]);
            hh[e] = hs[r + e];
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
    for (; r < re; ++r) {
        const uint32_t wv = *reinterpret_cast<const uint32_t*>(base + size_t(r) * pitch);
        const __half2 s2 = __half2half2(sc[r * pc.nsb + sbi]);
        const __half hh = hs[r];
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

// Compact reduction of one 32-column block (reduction.py:6-28,
// streaming_mlp.cu:80-84): lane = column, the 2 partial rows (row halves) of
// every descriptor summed in row order, loads issued 32 at a time; then the
// layer epilogue (fp16 output, residual add, fp32 output).
__device__ void reduce_block(const KernelParams& P, const LayerPlan& L, uint32_t blk, uint32_t rows, bool write,
                             int lane) {
    const uint32_t H = P.H, c = 32 * blk + lane;
    const float* p = P.partial + c;
    const uint32_t n = 2 * rows;
    float s = 0.f;
    uint32_t r = 0;
    for (; r + 32 <= n; r += 32) {
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __ldcg(p + size_t(r + e) * H);
#pragma unroll
        for (int e = 0; e < 32; ++e) s += v[e];
    }
    for (; r + 8 <= n; r += 8) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __ldcg(p + size_t(r + e) * H);
#pragma unroll
        for (int e = 0; e < 8; ++e) s += v[e];
    }
    for (; r < n; ++r) s += __ldcg(p + size_t(r) * H);
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

template <int SB, bool MMA>
__device__ void run_consumers(const KernelParams& P, uint8_t* stages, SmemTail* t, uint64_t deadline) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t l = 0;
    const LayerPlan* L = &plan_at(P, 0);
    Frag<Split<SB>::SBH> a;
    if (warp == 0) stage_x(P, *L, t, 0, lane);
    smem_wait(P, t, &t->xready, 1, deadline + kSyncGraceNs, 7, lane);
    load_activation<SB>(P, *L, t->xs, a, warp, lane);
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
        if (tid == 0) trace_piece(P, idx, 2);
        if (idx == 0 && tid == 0) trace(P, LS_B200_TRACE_FIRST);
        if (tid == 0 && pc.kind == kPieceLayer) trace_layer(P, l, LS_B200_LTRACE_PIECES_DONE);
        if (pc.kind == kPieceFinal) {
            if (tid == 0) trace(P, LS_B200_TRACE_PIECES);
            break;
        }
        uint8_t* st = stages + size_t(s) * kStageBytes;
        const bool aborted = __shfl_sync(0xffffffffu, t->abort, 0) != 0;  // warp-uniform snapshot
        if (pc.kind == kPieceGateUp) {
            // every warp takes part (the last one resets the piece counter)
            consume_gateup<SB, MMA>(P, *L, pc, st, t, s, a, warp, lane);
        } else if (pc.kind == kPieceDown) {
            if (pc.flags & kFirstRows) {
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = 0.f;
            }
            if (!aborted) {
                consume_down(pc, st, reinterpret_cast<const __half*>(st + kStageData + kAuxSecond), acc, tid);
                if ((pc.flags & kLastRows) && (uint32_t(tid) & 255u) < 4 * pc.chunks) {
                    float* dst = P.partial + (size_t(pc.row) * 2 + (uint32_t(tid) >> 8)) * P.H + 32 * pc.k0 +
                                 8 * (uint32_t(tid) & 255u);
                    reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
                    reinterpret_cast<float4*>(dst)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
                }
                if ((pc.flags & kCompletes) && tid == 0 && L->execs) atomicAdd(L->execs + pc.dest, 1u);
            }
        }
        __syncwarp();
        if (tid == 0) trace_piece(P, idx, 3);
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
        load_activation<SB>(P, *L, t->xs, a, warp, lane);
        if (tid == 0) trace_layer(P, l, LS_B200_LTRACE_LOADED);
    }
}

template <int SB, bool MMA>
__global__ void __launch_bounds__(kThreads, 1) fused_mlp_kernel(const __grid_constant__ KernelParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    SmemTail* t = reinterpret_cast<SmemTail*>(smem + size_t(kStages) * kStageBytes);
    const int tid = threadIdx.x;
    const uint64_t deadline = gtimer() + P.timeout_ns;
    if (tid == 0) {
        trace(P, LS_B200_TRACE_ENTRY);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&t->full_bar[s]), 34);                // lane 0 expect_tx + 32 cp.async + lane 0 close
            mbar_init(smem_u32(&t->empty_bar[s]), kConsumerWarps);  // one arrive per consumer warp
            t->gcnt[s] = 0;
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
        run_consumers<SB, MMA>(P, stages, t, deadline);
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

template <int SB, bool MMA>
static int launch_t(const KernelParams& p, int grid, cudaStream_t stream) {
    fused_mlp_kernel<SB, MMA><<<grid, kThreads, kernel_smem_bytes(), stream>>>(p);
    return int(cudaGetLastError());
}

template <int SB, bool MMA>
static cudaError_t raise_smem(int bytes) {
    return cudaFuncSetAttribute(fused_mlp_kernel<SB, MMA>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

int prepare_kernels() {
    const int bytes = int(kernel_smem_bytes());
    const cudaError_t errs[] = {raise_smem<1, false>(bytes),  raise_smem<2, false>(bytes), raise_smem<4, false>(bytes),
                                raise_smem<8, false>(bytes),  raise_smem<16, false>(bytes), raise_smem<1, true>(bytes),
                                raise_smem<2, true>(bytes),   raise_smem<4, true>(bytes),  raise_smem<8, true>(bytes),
                                raise_smem<16, true>(bytes)};
    for (cudaError_t e : errs)
        if (e != cudaSuccess) return int(e);
    return 0;
}

// H = 256 * SB with SB in {1, 2, 4, 8, 16} (each warp owns H/8 coordinates).
int launch_fused(const KernelParams& p, int grid, cudaStream_t stream) {
    const bool mma = p.variant != 0;
    switch (p.H / 256) {
        case 1: return mma ? launch_t<1, true>(p, grid, stream) : launch_t<1, false>(p, grid, stream);
        case 2: return mma ? launch_t<2, true>(p, grid, stream) : launch_t<2, false>(p, grid, stream);
        case 4: return mma ? launch_t<4, true>(p, grid, stream) : launch_t<4, false>(p, grid, stream);
        case 8: return mma ? launch_t<8, true>(p, grid, stream) : launch_t<8, false>(p, grid, stream);
        case 16: return mma ? launch_t<16, true>(p, grid, stream) : launch_t<16, false>(p, grid, stream);
        default: return int(cudaErrorInvalidValue);
    }
}

}  // namespace lsb
