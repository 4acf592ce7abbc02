// Fused sparse INT4 SwiGLU MLP for sm_100a: one persistent launch runs one
// layer (the ComputeBackend path) or a whole stack of layers.
//
// It replaces the reference's three-launch chain A core_kernel -> B consumer
// -> reduction (kernels/streaming_mlp.cu:44-93; backends/triton/core.py:20-64,
// persistent.py:33-92, reduction.py:6-28), and for stacks also the per-layer
// residual + RMSNorm glue (reduction.py:17-20;
// examples/ministral/native/predictor_shared_input.cu:16-33).
//
// CTA = 16 consumer warps + a producer warp + an epilogue warp, one CTA per SM.
//
// Work unit: a slab = up to 16 consecutive neurons of one descriptor (group).
// The CTA that owns a slab computes its gate/up rows, its h values and its
// down rows, and writes one fp32 partial output row for it, so h never
// crosses CTAs. Slabs are split statically over the grid when the whole
// plan is ready at decision time (fast path, BatchCompat / Auto), or claimed
// in ready order from a device counter (progressive path).
//
// Producer warp: streams each slab into a 6-stage shared-memory ring as
// three pieces -- GATEUP (gate+up records of 8 neurons, one cp.async.bulk
// per neuron), GATEUP (the next 8) and DOWN (the slab's down rows) -- plus
// their fp16 scales (cp.async), completing one mbarrier per stage. A slab's
// DOWN piece follows the next slab's GATEUP pieces. Weights do not depend on
// activations, so the producer runs ahead across layer boundaries while the
// consumers synchronise.
//
// Consumers (tensor cores, mma.sync):
//   GATEUP: 16 rows = the gate and up rows of 8 neurons; the hidden dimension
//           is split over the warps. Variant 1: integer MMAs on q + 8 and the
//           three 8-bit digit planes of x as 22-bit fixed point, the fp16
//           scale applied per 128-block to the exact sums. Variant 0: fp16
//           MMAs on w = fp16(q * s) (backends/triton/core.py:17). The
//           epilogue warp sums the warp partials in warp order and forms
//           h = fp16(fp16(SiLU(fp16 g)) * fp16 u).
//   DOWN:   fp16 MMAs, A = down weights with neurons along K (nibbles of two
//           neurons paired with PRMT, exact fp16 subnormals (q + 8) 2^-24),
//           B = h * s as an fp16 value plus its fp16 residual (variant 1) or
//           h with w = fp16(q * s) (variant 0).
//   Canonical arithmetic (identical for both schedules, so BatchCompat and
//   Progressive outputs are bit-identical, tests/persistent_mlp_test.cu:65):
//   a slab's h and partial row depend only on the slab; y sums the partial
//   rows (row = descriptor row * slabs-per-group + slab) in a fixed tree of
//   16-row chunks.
// End of layer: H/32 CTAs each reduce one 32-column block and apply the
// epilogue (fp16 output, fp32 output, residual add); the next layer's input
// is handed over through tagged words, without a grid-wide barrier.
//
// Every wait is bounded by a %globaltimer deadline and records an error;
// consumer warps synchronise through an mbarrier with bounded waits (never
// bar.sync), so a warp that gives up cannot strand the others.
//
// The file is compiled twice: ls_kernel_traced.cu includes it with
// LS_KERNEL_TRACE 1 for the kernels that write phase stamps, which run only
// for launches that ask for stamps; the other kernels carry no stamp code.
#include <cuda_fp16.h>
#include <stdint.h>
#include "ls_internal.h"

#ifndef LS_KERNEL_TRACE
#define LS_KERNEL_TRACE 0
#endif
#if LS_KERNEL_TRACE
#define LS_KERNEL_NS traced
#else
#define LS_KERNEL_NS plain
#endif

namespace lsb {
namespace LS_KERNEL_NS {

enum : uint32_t { kPieceFinal = 0, kPieceGateUp = 1, kPieceDown = 2, kPieceLayer = 3 };
// Piece flags. kPaired: a GATEUP piece whose slab's second GATEUP piece
// is the next stage (both are consumed in one pass). kHsBuf: the h buffer
// of the piece's slab (slabs alternate, so that the next slab's GATEUP can
// finalise h while this slab's DOWN still reads it). kPart1: the piece
// covers the second K part (GATEUP) or column part (DOWN) of its slab
// (hidden sizes above one piece's extent).
enum : uint32_t { kCompletes = 4u, kLayerGood = 8u, kPaired = 16u, kHsBuf = 32u, kPart1 = 64u };
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
    uint32_t row;    // DOWN: partial row (descriptor row * slabs per group + slab)
    uint32_t dest;   // descriptor dest_slot (activation / counter index)
    uint32_t n0;     // first neuron of the piece within the group
    uint32_t count;  // neurons; LAYER: partial rows of the layer
    uint32_t need;   // DOWN: GATEUP pieces that must be finalised first
    uint32_t flags;
    uint32_t layer;  // launch-local layer index
    uint32_t pad[8];
};
static_assert(sizeof(Piece) == 64, "piece record");

struct DescView {
    const uint8_t* src;  // packed group base
    uint32_t phys, dest, row, ok;
};

// Piece geometry per hidden size. A piece covers at most 4096 hidden
// coordinates: above that (H 8192) a slab's gate/up records are split into
// KS parts along K and its down rows into KS parts along the output columns,
// so that every piece has the stage layout of H 4096; the ring then holds
// five stages (the activation planes take the sixth's space).
template <int H>
struct Geo {
    static constexpr int HP = H > kMaxPieceHidden ? kMaxPieceHidden : H;  // hidden extent of one piece
    static constexpr int KS = H / HP;                                    // parts per slab
    static constexpr int NS = H > kMaxPieceHidden ? 5 : 6;               // ring stages
    static constexpr int XPL = H + 32;  // bytes per digit plane of the fixed-point activation (8 banks apart)
    static constexpr int XBYTES = 3 * XPL + 4 * (H / 32) + 4 * (H / 64);
    static constexpr int UPT = (H / 8 + kConsumerThreads - 1) / kConsumerThreads;  // activation units per thread
    static_assert(NS <= kStages, "ring stages");
};

// Stamps the traced build keeps in shared memory: the first 64 pieces of
// CTAs 0..3 and the first 48 layers of every CTA.
constexpr uint32_t kTracePieces = 64, kTraceLayers = 40;
// per-warp completion stamps of pieces [kTraceWarpBase, +kTraceWarpPieces) of CTA 0
constexpr uint32_t kTraceWarpBase = 8, kTraceWarpPieces = 12;
static_assert(kTraceWarpBase + kTraceWarpPieces <= 64, "per-warp stamps of the first pieces");
static_assert(kTracePieces <= LS_B200_PIECE_TRACE_PIECES && kTraceLayers > 0, "trace stamps");

struct alignas(16) SmemTail {
    unsigned long long full_bar[kStages];
    unsigned long long empty_bar[kStages];
    unsigned long long cbar;  // consumer-warp barrier (16 arrivals per phase)
    Piece piece[kStages];
    DescView dtab[32];        // producer's descriptor window
    unsigned long long pbar[kStages];  // GATEUP warp partials written (16 arrivals per phase)
    alignas(16) uint32_t zero16[4];        // read by lanes whose B operand is zero
    alignas(16) uint32_t nib[8];           // nibble masks and offsets (NibMasks), see and_xor
    float xscale;               // variant 1: x = fixed-point value * xscale
    float red[kConsumerWarps];             // RMSNorm warp sums
    float red2[kConsumerWarps][32];        // reduction warp sums
    __half hs[2][kSlab];                   // h of the last two slabs (kHsBuf)
    volatile uint32_t octets_done;         // GATEUP pieces finalised (monotonic)
    uint32_t tagbase;                      // ws[kWsTag] at launch entry (scratch tags)
    volatile uint32_t abort;
    volatile uint32_t flag;                // CTA-uniform decision broadcast by thread 0
    uint32_t last;
    // Layer plans of the consumers and the epilogue warp: layer l in slot
    // l % 3. Warp 0 of the consumers copies layer l+2's plan (cp.async) when
    // layer l ends, and the copy is waited for before the barrier that ends
    // the staging of layer l+1, so the plan fields read on the layer hand-off
    // come from shared memory instead of a global round trip.
    LayerPlan cplan[3];
#if LS_KERNEL_TRACE
    uint32_t tpiece[kTracePieces][4];                     // piece stamps (CTAs 0..3), see trace_piece
    uint32_t tlayer[kTraceLayers][LS_B200_LAYER_TRACE_WORDS];  // layer stamps, see trace_layer
    uint32_t twarp[kTraceWarpPieces][kConsumerWarps];      // per-warp piece completion (CTA 0)
#endif
};
constexpr uint32_t kPlanChunks = sizeof(LayerPlan) / 16;
static_assert(sizeof(LayerPlan) % 16 == 0, "plan copied in 16-byte chunks");

// Activation of the current layer, after the tail (Geo<H>::XBYTES):
// variant 1: three planes of signed 8-bit digits, 16 bytes per two
//            8-coordinate units u, u+1 (even digits of u, of u+1, odd digits
//            of u, of u+1), planes Geo<H>::XPL bytes apart; then the sums of
//            the fixed-point x over each 32-coordinate sub-block and over
//            each 64-coordinate group;
// variant 0: uint4 of four fp16 pairs per 8 coordinates.
template <int H>
__device__ __forceinline__ uint8_t* xarea(SmemTail* t) { return reinterpret_cast<uint8_t*>(t + 1); }
template <int H>
__device__ __forceinline__ int* xsum32(SmemTail* t) { return reinterpret_cast<int*>(xarea<H>(t) + 3 * Geo<H>::XPL); }
template <int H>
__device__ __forceinline__ int* xsum64(SmemTail* t) { return xsum32<H>(t) + H / 32; }

// The part of the activation one GATEUP piece reduces over (K part kp).
struct XPart {
    const uint8_t* x;  // digit plane 0 at the part's first coordinate
    const int* m32;    // sub-block sums of the part
    const int* m64;    // 64-coordinate group sums of the part
};
template <int H>
__device__ __forceinline__ XPart xpart(SmemTail* t, uint32_t kp) {
    constexpr int HP = Geo<H>::HP;
    return XPart{xarea<H>(t) + kp * HP, xsum32<H>(t) + kp * (HP / 32), xsum64<H>(t) + kp * (HP / 64)};
}

template <int H>
__host__ __device__ constexpr size_t kernel_smem_bytes() {
    return size_t(Geo<H>::NS) * kStageBytes + sizeof(SmemTail) + Geo<H>::XBYTES;
}

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
__device__ __forceinline__ uint4 ld_acquire_sys_v4(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.acquire.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ ulonglong2 ld_volatile_v2u64(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_volatile_v2u64(unsigned long long* p, unsigned long long a, unsigned long long b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1,%2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long a) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_max_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.max.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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
template <int BYTES>
__device__ __forceinline__ void cp_async(uint32_t dst, const void* src) {
    if constexpr (BYTES == 16) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    } else if constexpr (BYTES == 8) {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
    } else {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
    }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Tensor-core step: D(16x8,f32) += A(16x16,f16) * B(16x8,f16).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) {
    __half2 h;
    *reinterpret_cast<uint32_t*>(&h) = v;
    return h;
}

// ---- nibble decoding. A 32-bit word holds two 16-bit halves; mask m selects
// one signed two's-complement nibble per half (low nibble = even coordinate,
// backends/triton/core.py:14-15).
// Subnormal form: (q + 8) * 2^-24 (low nibble) or 16 (q + 8) * 2^-24 (high
// nibble), exact fp16 values built by one LOP3.
// (w & m) ^ x as one three-input logic instruction. The masks live in
// registers loaded from shared memory (NibMasks): written as two 32-bit
// immediates, the expression takes two instructions, one per immediate.
__device__ __forceinline__ uint32_t and_xor(uint32_t w, uint32_t m, uint32_t x) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(r) : "r"(w), "r"(m), "r"(x));
    return r;
}
// Nibble masks: q + 8 of the low (high, times 16) nibble of every byte, and
// of the low byte of every 16-bit half (fp16 subnormal operands).
struct NibMasks {
    uint32_t lo_m, lo_x, hi_m, hi_x;    // 0x0F0F0F0F 0x08080808 0xF0F0F0F0 0x80808080
    uint32_t hlo_m, hlo_x, hhi_m, hhi_x;  // 0x000F000F 0x00080008 0x00F000F0 0x00800080
};
__device__ __forceinline__ NibMasks load_nib(const SmemTail* t) {
    const uint4 a = *reinterpret_cast<const uint4*>(t->nib), b = *reinterpret_cast<const uint4*>(t->nib + 4);
    return NibMasks{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
}
__device__ __forceinline__ uint32_t sub_lo(uint32_t w, const NibMasks& k) { return and_xor(w, k.hlo_m, k.hlo_x); }
__device__ __forceinline__ uint32_t sub_hi(uint32_t w, const NibMasks& k) { return and_xor(w, k.hhi_m, k.hhi_x); }
// Exact-integer form: q as fp16.
__device__ __forceinline__ __half2 int_lo(uint32_t w) {
    return __hsub2(bits_h2((w & 0x000F000Fu) ^ 0x64086408u), __float2half2_rn(1032.f));  // 1024 + (q + 8)
}
__device__ __forceinline__ __half2 int_hi(uint32_t w) {
    return __hfma2(bits_h2((w & 0x00F000F0u) ^ 0x64806480u), __float2half2_rn(0.0625f),
                   __float2half2_rn(-72.f));  // (1024 + 16 (q + 8)) / 16 - 72
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}
__device__ __forceinline__ float h2f(uint16_t v) { return __half2float(__ushort_as_half(v)); }
__device__ __forceinline__ float round16(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ uint32_t* ws_layer(const KernelParams& P, uint32_t l) {
    // [0] path [1] slab claim [2] unused [3] reduced blocks [4] unused
    // [5] mirror of ready_count [6] mirror of the queue state
    return P.ws + kWsHeader + kWsPerLayer * l;
}
// Tag of the scratch words written by launch-local layer l: 1 + the device
// tag counter at launch entry + l (never 0). A 64-bit word (tag << 32 | value)
// is written by one store, so a reader that sees the current tag also sees
// the value: no fence or counter is needed.
__device__ __forceinline__ uint32_t scratch_tag(const SmemTail* t, uint32_t l) { return 1u + t->tagbase + l; }
__device__ __forceinline__ bool grid_failed(const KernelParams& P) { return ld_acquire_gpu(P.ws + kWsErr) != 0; }
__device__ __forceinline__ void trace(const KernelParams& P, uint32_t word) {
    if (!LS_KERNEL_TRACE) return;
    if (P.trace) P.trace[size_t(blockIdx.x) * LS_B200_TRACE_WORDS + word] = gtimer();
}
// Per-piece stamps of CTAs 0..3 after the per-layer block:
// [4][LS_B200_PIECE_TRACE_PIECES][4] = issued, closed (producer), ready, done (consumer warp 0).
// Piece and layer stamps are kept in shared memory as the low 32 bits of
// %globaltimer (a global store right after a burst of partial-row stores
// can wait in the store queue and would shift the stamp) and written out
// at the end of the launch (flush_trace).
__device__ __forceinline__ void trace_piece(const KernelParams& P, SmemTail* t, uint32_t piece, uint32_t word) {
#if LS_KERNEL_TRACE
    if (P.trace && blockIdx.x < 4 && piece < kTracePieces) t->tpiece[piece][word] = uint32_t(gtimer());
#endif
}
// Per-layer stamps after the launch-level block: [grid][nlayers][LS_B200_LAYER_TRACE_WORDS].
__device__ __forceinline__ void trace_layer(const KernelParams& P, SmemTail* t, uint32_t l, uint32_t word) {
#if LS_KERNEL_TRACE
    if (P.trace && l < kTraceLayers) t->tlayer[l][word] = uint32_t(gtimer());
#endif
}
// Completion of piece `piece` by consumer warp `warp` (CTA 0, lane 0).
__device__ __forceinline__ void trace_warp(const KernelParams& P, SmemTail* t, uint32_t piece, int warp) {
#if LS_KERNEL_TRACE
    if (P.trace && blockIdx.x == 0 && piece - kTraceWarpBase < kTraceWarpPieces)
        t->twarp[piece - kTraceWarpBase][warp] = uint32_t(gtimer());
#endif
}
// Writes the shared-memory stamps of this CTA to P.trace as 64-bit
// %globaltimer values (after the final barrier of the launch).
__device__ void flush_trace(const KernelParams& P, SmemTail* t, uint64_t entry) {
#if LS_KERNEL_TRACE
    if (!P.trace) return;
    const auto full = [entry](uint32_t v) -> uint64_t {
        return v ? entry + uint64_t(int64_t(int32_t(v - uint32_t(entry)))) : 0ull;
    };
    const uint32_t nl = P.nlayers < kTraceLayers ? P.nlayers : kTraceLayers;
    for (uint32_t i = threadIdx.x; i < nl * LS_B200_LAYER_TRACE_WORDS; i += blockDim.x)
        P.trace[size_t(gridDim.x) * LS_B200_TRACE_WORDS + size_t(blockIdx.x) * P.nlayers * LS_B200_LAYER_TRACE_WORDS +
                i] = full(t->tlayer[i / LS_B200_LAYER_TRACE_WORDS][i % LS_B200_LAYER_TRACE_WORDS]);
    if (blockIdx.x == 0)  // per-warp stamps: CTA 0's piece records from kTracePieces on
        for (uint32_t i = threadIdx.x; i < kTraceWarpPieces * kConsumerWarps; i += blockDim.x)
            P.trace[size_t(gridDim.x) * LS_B200_TRACE_WORDS + size_t(gridDim.x) * P.nlayers * LS_B200_LAYER_TRACE_WORDS +
                    size_t(kTracePieces) * 4 + i] = full(t->twarp[i / kConsumerWarps][i % kConsumerWarps]);
    if (blockIdx.x < 4)
        for (uint32_t i = threadIdx.x; i < kTracePieces * 4; i += blockDim.x)
            P.trace[size_t(gridDim.x) * LS_B200_TRACE_WORDS + size_t(gridDim.x) * P.nlayers * LS_B200_LAYER_TRACE_WORDS +
                    (size_t(blockIdx.x) * LS_B200_PIECE_TRACE_PIECES + i / 4) * 4 + i % 4] = full(t->tpiece[i / 4][i % 4]);
#endif
}

// Records the first error of this launch and asks the CTA to stop.
// Out of line: an error path, kept out of the instruction-cache footprint of
// the loops that call it.
__device__ __noinline__ void raise_error(const KernelParams& P, SmemTail* t, uint32_t code, uint32_t detail) {
    if (atomicCAS(P.ws + kWsErr, 0u, code) == 0u) P.ws[kWsDetail] = detail;
    t->abort = 1;
}
// Plan of launch-local layer l, read in place (kernel parameter or device array).
__device__ __forceinline__ const LayerPlan& plan_at(const KernelParams& P, uint32_t l) {
    return P.plans ? P.plans[l] : P.first;
}

// Consumers' copy of layer l's plan (slot l % 3; see SmemTail::cplan).
__device__ __forceinline__ const LayerPlan& cplan_at(const SmemTail* t, uint32_t l) { return t->cplan[l % 3]; }
// Warp 0 of the consumers: asynchronous copy of layer l's plan into its slot
// (multi-layer launches; a one-layer launch has its plan copied in the
// prologue).
__device__ __forceinline__ void fetch_plan(const KernelParams& P, SmemTail* t, uint32_t l, int tid) {
    if (P.plans && l < P.nlayers && tid < int(kPlanChunks)) {
        cp_async<16>(smem_u32(&t->cplan[l % 3]) + 16u * uint32_t(tid),
                     reinterpret_cast<const uint8_t*>(P.plans + l) + 16u * uint32_t(tid));
        cp_async_commit();
    }
}

// ------------------------------------------------------------ descriptors
// Descriptor at canonical position d: core[d] for d < core_count, else the
// queue descriptor published at ready position d - core_count
// (streaming_mlp.cu:60, persistent.py:80). Descriptor row: d for core, else
// core_count + descriptor index (custom_triton.md:54).
template <bool LEAN>
__device__ DescView load_desc(const KernelParams& P, const LayerPlan& L, uint32_t l, uint32_t d) {
    const uint32_t* c;
    uint32_t row;
    if (!LEAN && (L.flags & kPlanHostQueue)) {
        // the device copy made under the polling lease (mirror_queue)
        const uint4* e = P.qmirror + (size_t(l) * P.N + d) * 2;
        const uint4 a = e[0];
        const uint32_t kind = e[1].x;
        const uint32_t idx = a.x;
        DescView v;
        row = d < L.core_count ? d : L.core_count + idx;
        v.ok = idx != 0xffffffffu && kind <= 1u && a.w < P.N && row < P.N &&
               (P.phys_groups == 0 || a.y < P.phys_groups) &&
               (kind == 0 ? (P.cache_slots == 0 || a.z < P.cache_slots) : (P.staging_slots == 0 || a.z < P.staging_slots));
        v.src = (kind == 0 ? L.cache : L.staging) + size_t(a.z) * P.group_bytes;
        v.phys = a.y;
        v.dest = a.w;
        v.row = row;
        return v;
    }
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
    uint32_t idx;     // pieces issued so far (stage = idx % Geo<H>::NS)
    uint32_t octets;  // GATEUP pieces issued so far
    uint32_t slabs;   // slabs issued so far (h buffer = slabs & 1)
    uint32_t lane;
    uint8_t* stages;
    SmemTail* t;
    uint64_t deadline;
    uint32_t wbase;  // first descriptor position held in t->dtab
    uint32_t wlayer;
};

// Waits until the next stage is free.
template <int H>
__device__ bool producer_acquire_stage(Producer& pr, const KernelParams& P) {
    constexpr uint32_t NS = Geo<H>::NS;
    const uint32_t s = pr.idx % NS;
    const uint32_t parity = ((pr.idx / NS) & 1u) ^ 1u;
    const uint32_t bar = smem_u32(&pr.t->empty_bar[s]);
    uint32_t spins = 0;
    for (;;) {
        uint32_t ready = 0;
        if (pr.lane == 0) ready = mbar_try_wait(bar, parity) ? 1u : 0u;
        if (__shfl_sync(0xffffffffu, ready, 0)) return true;
        __nanosleep(spins < 64 ? 32 : 256);  // back off: keep issue slots free for the consumers
        uint32_t late = 0;
        if (pr.lane == 0 && (++spins & 255u) == 0 && gtimer() > pr.deadline + kProducerGraceNs) late = 1;
        if (__shfl_sync(0xffffffffu, late, 0)) {
            if (pr.lane == 0) raise_error(P, pr.t, LS_B200_DEV_TIMEOUT_SYNC, 1);
            return false;
        }
    }
}

// Completes a stage: 32 cp.async arrivals (one per lane, when its scale
// copies land) plus one arrival by lane 0 after the piece record is written.
// With lane 0's expect_tx arrival the full barrier expects 34 in total.
__device__ __forceinline__ void producer_close(Producer& pr, const KernelParams& P, uint32_t s) {
    const uint32_t bar = smem_u32(&pr.t->full_bar[s]);
    cp_async_arrive_noinc(bar);
    __syncwarp();
    if (pr.lane == 0) {
        mbar_arrive(bar);
        trace_piece(P, pr.t, pr.idx, 1);
    }
}

// A data-less piece (LAYER or FINAL marker).
template <int H>
__device__ bool producer_marker(Producer& pr, const KernelParams& P, uint32_t kind, uint32_t layer, uint32_t rows,
                                uint32_t flags) {
    if (!producer_acquire_stage<H>(pr, P)) return false;
    const uint32_t s = pr.idx % Geo<H>::NS;
    if (pr.lane == 0) {
        Piece& pc = pr.t->piece[s];
        pc.kind = kind;
        pc.layer = layer;
        pc.count = rows;
        pc.flags = flags;
        trace_piece(P, pr.t, pr.idx, 0);
        mbar_arrive_expect_tx(smem_u32(&pr.t->full_bar[s]), 0);
    }
    producer_close(pr, P, s);
    ++pr.idx;
    return true;
}

// Scale copy granule: 16 bytes when every scale row and segment is 16-byte
// aligned (H >= 1024: row pitch 3H/64 bytes), else the segment size.
// Staged scale rows are padded by 16 bytes so that consecutive neurons' rows
// start 4 banks apart (conflict-free reads by the MMA lane layout). A staged
// row holds the scales of the piece's part: gate then up (GATEUP) or down.
template <int H>
struct ScaleCopy {
    static constexpr int HP = Geo<H>::HP;
    static constexpr int kUnit = H >= 1024 ? 16 : H / 64;
    static constexpr uint32_t kRow = 3 * H / 64;   // bytes of one neuron's scales in HBM
    static constexpr uint32_t kGateUp = HP / 32;   // staged gate + up scale bytes of one neuron
    static constexpr uint32_t kDown = HP / 64;     // staged down scale bytes of one neuron
    static constexpr uint32_t kPart = HP / 64;     // offset of part kp+1's gate (or down) scales
    static constexpr uint32_t kUpSkip = (H - HP) / 64;  // the gate scales of the other parts
    static constexpr uint32_t kGateUpPitch = kGateUp + 16;
    static constexpr uint32_t kDownPitch = kDown + 16;
};

// Row pitch of a staged GATEUP record: variant 1 reads 8 bytes per lane, so
// rows start 8 banks apart (H + 32); variant 0 reads 4 bytes (H + 16).
template <int H, bool F>
__host__ __device__ constexpr int gateup_pitch() { return F ? H + 32 : H + 16; }

// One GATEUP piece (gate+up records of neurons [n0, n0+cnt), cnt <= 8) or
// DOWN piece (down rows of one slab, cnt <= 16) of part kp: lane k issues
// the bulk copy of neuron k (parts of a split slab: lanes 0-7 the gate and
// 8-15 the up part of neuron k & 7), every lane up to two 16-byte scale
// copies. No unrolled loops: the producer's code shares the instruction
// caches with the consumers' piece loops. (Out of line, the call costs more
// than the code it saves.)
template <int H, bool F>
__device__ __forceinline__ bool producer_piece(Producer& pr, const KernelParams& P, const LayerPlan& L,
                                            const DescView& d, uint32_t kind, uint32_t layer, uint32_t n0,
                                            uint32_t cnt, uint32_t row, uint32_t flags, uint32_t need) {
    constexpr int HP = Geo<H>::HP, KS = Geo<H>::KS;
    if (!producer_acquire_stage<H>(pr, P)) return false;
    const bool gu = kind == kPieceGateUp;
    const uint32_t kp = (flags & kPart1) ? 1u : 0u;
    const uint32_t s = pr.idx % Geo<H>::NS;
    uint8_t* st = pr.stages + size_t(s) * kStageBytes;
    const uint32_t bar = smem_u32(&pr.t->full_bar[s]);
    constexpr uint64_t rec = uint64_t(3) * H / 2;  // bytes per neuron record
    const uint32_t bytes = gu ? uint32_t(HP) : uint32_t(HP / 2);
    const uint32_t pitch = gu ? uint32_t(gateup_pitch<HP, F>()) : uint32_t(HP / 2 + 16);
    if (pr.lane == 0) {
        Piece& pc = pr.t->piece[s];
        pc.kind = kind;
        pc.layer = layer;
        pc.row = row;
        pc.dest = d.dest;
        pc.n0 = n0;
        pc.count = cnt;
        pc.need = need;
        pc.flags = flags;
        trace_piece(P, pr.t, pr.idx, 0);
        mbar_arrive_expect_tx(bar, cnt * bytes);
    }
    __syncwarp();
    if constexpr (KS == 1) {
        if (pr.lane < cnt)
            bulk_g2s(smem_u32(st + size_t(pr.lane) * pitch), d.src + (n0 + pr.lane) * rec + (gu ? 0u : uint32_t(H)),
                     bytes, bar);
    } else {
        // gate part kp at kp*HP/2 of the record, up part at H/2 + kp*HP/2,
        // down part at H + kp*HP/2; each HP/2 bytes
        const uint32_t k = gu ? (pr.lane & 7u) : pr.lane, half = gu ? (pr.lane >> 3) : 0u;
        if ((gu ? pr.lane < 16u : true) && k < cnt)
            bulk_g2s(smem_u32(st + size_t(k) * pitch + half * (HP / 2)),
                     d.src + (n0 + k) * rec + (gu ? half * uint32_t(H / 2) : uint32_t(H)) + kp * uint32_t(HP / 2),
                     uint32_t(HP / 2), bar);
    }
    using SC = ScaleCopy<H>;
    const uint32_t unit_bytes = gu ? SC::kGateUp : SC::kDown;  // scale bytes of one neuron in this piece
    const uint32_t upn = unit_bytes / SC::kUnit;
    const uint32_t spitch = gu ? SC::kGateUpPitch : SC::kDownPitch;
    const uint8_t* sbase = reinterpret_cast<const uint8_t*>(L.scales) + (size_t(d.phys) * P.G + n0) * SC::kRow +
                           (gu ? 0u : uint32_t(H / 32)) + kp * SC::kPart;
    const uint32_t sdst = smem_u32(st + kStageData);
#pragma unroll 1
    for (uint32_t i = pr.lane; i < cnt * upn; i += 32) {
        const uint32_t k = i / upn, o = i % upn;
        const uint32_t skip = (KS > 1 && gu && 2 * o >= upn) ? SC::kUpSkip : 0u;  // up scales of part kp
        cp_async<SC::kUnit>(sdst + k * spitch + o * SC::kUnit, sbase + k * SC::kRow + o * SC::kUnit + skip);
    }
    producer_close(pr, P, s);
    ++pr.idx;
    if (gu && (KS == 1 || kp == KS - 1)) ++pr.octets;  // h of the octet is formed after its last part
    return true;
}

template <int H, bool F>
__device__ __forceinline__ bool producer_gateup(Producer& pr, const KernelParams& P, const LayerPlan& L,
                                                const DescView& d, uint32_t layer, uint32_t n0, uint32_t cnt,
                                                uint32_t flags) {
    return producer_piece<H, F>(pr, P, L, d, kPieceGateUp, layer, n0, cnt, 0u, flags, 0u);
}

template <int H, bool F>
__device__ __forceinline__ bool producer_down(Producer& pr, const KernelParams& P, const LayerPlan& L,
                                              const DescView& d, uint32_t layer, uint32_t n0, uint32_t cnt,
                                              uint32_t row, uint32_t flags, uint32_t need) {
    return producer_piece<H, F>(pr, P, L, d, kPieceDown, layer, n0, cnt, row, flags, need);
}

// The GATEUP pieces of slab `slab` of one descriptor (variant 1 pairs the
// two halves of a 16-neuron slab so that they are consumed in one pass),
// for each K part in order.
template <int H, bool F>
__device__ bool producer_slab_gateup(Producer& pr, const KernelParams& P, const LayerPlan& L, const DescView& d,
                                     uint32_t layer, uint32_t slab, uint32_t buf) {
    const uint32_t n0 = slab * kSlab;
    const uint32_t cnt = (P.G - n0) < kSlab ? (P.G - n0) : kSlab;
#pragma unroll 1
    for (uint32_t kp = 0; kp < uint32_t(Geo<H>::KS); ++kp) {
        const uint32_t part = kp ? kPart1 : 0u;
        const uint32_t first = (F && cnt > 8u) ? (buf | part | kPaired) : (buf | part);
        if (!producer_gateup<H, F>(pr, P, L, d, layer, n0, cnt < 8u ? cnt : 8u, first) || pr.t->abort) return false;
        if (cnt > 8u && (!producer_gateup<H, F>(pr, P, L, d, layer, n0 + 8, cnt - 8, buf | part) || pr.t->abort))
            return false;
    }
    return true;
}

// A slab whose GATEUP pieces are issued and whose DOWN piece is not yet.
struct PendingDown {
    DescView d;
    uint32_t slab, need, buf;
    bool valid;
};

// The DOWN piece of a pending slab. It is issued after the next slab's
// GATEUP pieces, so that the consumers compute those while the last warp
// of this slab's GATEUP finalises h.
template <int H, bool F>
__device__ bool producer_slab_down(Producer& pr, const KernelParams& P, const LayerPlan& L, PendingDown& pd,
                                   uint32_t layer) {
    if (!pd.valid) return true;
    pd.valid = false;
    const uint32_t spg = slabs_per_group(P.G);
    const uint32_t n0 = pd.slab * kSlab;
    const uint32_t cnt = (P.G - n0) < kSlab ? (P.G - n0) : kSlab;
#pragma unroll 1
    for (uint32_t kp = 0; kp < uint32_t(Geo<H>::KS); ++kp) {
        const bool last = kp + 1 == uint32_t(Geo<H>::KS);
        const uint32_t flags = (last && pd.slab + 1 == spg ? kCompletes : 0u) | pd.buf | (kp ? kPart1 : 0u);
        if (!producer_down<H, F>(pr, P, L, pd.d, layer, n0, cnt, pd.d.row * spg + pd.slab, flags, pd.need) ||
            pr.t->abort)
            return false;
    }
    return true;
}

// Issues the GATEUP pieces of a slab and the DOWN piece of the previous one.
template <int H, bool F>
__device__ bool producer_slab(Producer& pr, const KernelParams& P, const LayerPlan& L, const DescView& d,
                              uint32_t layer, uint32_t slab, PendingDown& pd) {
    const uint32_t buf = (pr.slabs & 1u) ? kHsBuf : 0u;
    if (!producer_slab_gateup<H, F>(pr, P, L, d, layer, slab, buf)) return false;
    const uint32_t need = pr.octets;
    ++pr.slabs;
    if (!producer_slab_down<H, F>(pr, P, L, pd, layer)) return false;
    pd.d = d;
    pd.slab = slab;
    pd.need = need;
    pd.buf = buf;
    pd.valid = true;
    return true;
}

// Loads the descriptor window [base, base+32) into shared memory, one
// descriptor per lane.
template <bool LEAN>
__device__ bool producer_window(Producer& pr, const KernelParams& P, const LayerPlan& L, uint32_t layer,
                                uint32_t base, uint32_t D) {
    const uint32_t d = base + pr.lane;
    uint32_t bad = 0;
    if (d < D) {
        const DescView v = load_desc<LEAN>(P, L, layer, d);
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

// Sleep between polls of a global word that has not changed yet: short for
// the first few microseconds of a wait (the layer hand-off), then growing to
// 1 us, so that a long wait (weights still streaming in) does not flood L2
// with polling loads while the copy engine writes into it.
__device__ __forceinline__ void poll_backoff(uint32_t spins, uint32_t base_ns) {
    const uint32_t shift = spins >> 6;
    __nanosleep(shift >= 5 ? 1024u : (base_ns << shift < 1024u ? base_ns << shift : 1024u));
}

// The queue's control words may be mapped host memory: a grid whose 148
// producers all polled them over PCIe would starve the copy engine that
// streams the weights. So one thread of the grid at a time polls the host
// (a lease of kHostPollNs on a device clock word) and publishes what it saw
// to device mirrors, which every CTA reads.
constexpr uint32_t kHostPollNs = 1000;
constexpr uint32_t kQueueActive = 1, kQueueFailed = 2;
// Waits on a host-memory queue back off quickly to 2 us between polls of the
// device mirrors: the mirror, state and lease words share one L2 line, and
// 148 CTAs polling it every ~150 ns made that L2 slice a hot spot that
// stalled the copy engine's writes of the streamed weights (copies 6x slower).
__device__ __forceinline__ void mirror_backoff(uint32_t polls) {
    const uint32_t shift = polls >> 3;
    __nanosleep(shift >= 4 ? 2048u : 128u << shift);
}
// The lease is exclusive until released (a read of host memory takes ~10 us
// here, far longer than the polling interval) and is taken at most every
// kHostPollNs.
__device__ __forceinline__ bool take_poll_lease(const KernelParams& P) {
    const uint32_t now = uint32_t(gtimer());
    if (now - ld_relaxed_gpu(P.ws + kWsPollClock) < kHostPollNs) return false;
    if (atomicCAS(P.ws + kWsPollLock, 0u, 1u) != 0u) return false;
    st_relaxed_gpu(P.ws + kWsPollClock, now);
    return true;
}
__device__ __forceinline__ void release_poll_lease(const KernelParams& P) { st_release_gpu(P.ws + kWsPollLock, 0u); }

// Warp-wide: copies descriptors [from, to) of layer l (core descriptors
// first, then queue positions through ready_indices) from host memory into
// the device mirror, one descriptor per lane in flight, then publishes the
// number of mirrored queue positions (lane 0, release). Entries of published
// positions never change, so overlapping copies by successive lease holders
// write the same values.
__device__ __noinline__ void mirror_queue(const KernelParams& P, const LayerPlan& L, uint32_t l, uint32_t from,
                                          uint32_t to, uint32_t lane, bool publish_count) {
    for (uint32_t d = from + lane; d < to; d += 32) {
        uint32_t idx, w[4] = {0u, 0u, 0u, 0xffffffffu};
        const uint32_t* c = nullptr;
        if (d < L.core_count) {
            idx = d;
            c = reinterpret_cast<const uint32_t*>(L.core + d);
        } else {
            idx = ld_relaxed_sys(L.q.ready_indices + (d - L.core_count));
            if (idx < L.q.capacity) c = reinterpret_cast<const uint32_t*>(L.q.descriptors + idx);
            else idx = 0xffffffffu;
        }
        if (c) {
#pragma unroll
            for (int k = 0; k < 4; ++k) w[k] = ld_relaxed_sys(c + 1 + k);
        }
        uint4* e = P.qmirror + (size_t(l) * P.N + d) * 2;
        e[0] = make_uint4(idx, w[0], w[1], w[2]);
        e[1] = make_uint4(w[3], 0u, 0u, 0u);
    }
    __threadfence();
    __syncwarp();
    if (publish_count && lane == 0) red_max_release_gpu(ws_layer(P, l) + 5, to - L.core_count);
}

// Per-CTA path decision for one layer (streaming_mlp.cu:49-56,
// persistent.py:46-55), by the producer warp. BatchCompat / Auto wait for the
// batch epoch and take the fast path; Progressive proposes a path and agrees
// with the other CTAs through a device-memory CAS (QueueControl.consumer_path
// stays untouched: a discrete GPU has no host-native atomics). A queue in
// host memory is read by the lease holder alone, who mirrors the plan into
// device memory before the other CTAs see it activated.
// Out of line: once per layer, and kept out of the instruction-cache
// footprint of the producer's per-piece code.
__device__ __noinline__ uint32_t decide(const KernelParams& P, const LayerPlan& L, uint32_t l, SmemTail* t,
                                        uint64_t deadline, uint32_t lane, uint32_t* total_out) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(L.q.control);
    const bool batch = L.mode != LS_MODE_PROGRESSIVE;  // Auto follows BatchCompat (streaming_mlp.cu:90)
    const bool host_queue = (L.flags & kPlanHostQueue) != 0;
    uint32_t* state = ws_layer(P, l) + 6;
    uint32_t code = 0, polls = 0, total = 0, ready = 0;
    for (;;) {
        // lane 0 polls; 0 wait, 1 activated (seen in the mirror), 2 failed,
        // 3 activated now (read from the queue), 4 deadline
        uint32_t st = 0;
        if (lane == 0) {
            const uint32_t m = host_queue ? ld_acquire_gpu(state) : 0u;
            if (m == kQueueActive) {
                st = 1;
            } else if (m == kQueueFailed) {
                st = 2;
            } else if (!host_queue || take_poll_lease(P)) {  // device-memory queue: every CTA reads it
                // The word that decides is read with acquire semantics (a
                // system-scope acquire load is ~0.2 us; a system-scope fence
                // ~4 us): Progressive reads the epoch word (in a), BatchCompat
                // the batch epoch (in b). The other vector is read first, so
                // both loads are in flight together; BatchCompat re-reads the
                // counts after its acquire.
                uint4 a, b;
                if (batch) {
                    a = ld_relaxed_sys_v4(w);
                    b = ld_acquire_sys_v4(w + 4);
                } else {
                    b = ld_relaxed_sys_v4(w + 4);
                    a = ld_acquire_sys_v4(w);
                }
                if (b.y) {
                    if (host_queue) st_release_gpu(state, kQueueFailed);
                    st = 2;
                } else if (a.w == L.epoch && (!batch || b.x == L.epoch)) {
                    if (batch) a = ld_relaxed_sys_v4(w);  // ordered after the acquire
                    total = a.z;
                    ready = batch ? total : a.x;
                    st = 3;
                }
                if (host_queue && st != 3) release_poll_lease(P);  // st 3: released after the mirror
            }
            if (st == 0 && gtimer() > deadline) st = 4;
        }
        st = __shfl_sync(0xffffffffu, st, 0);
        if (st == 0) {
            if (host_queue)
                mirror_backoff(polls++);
            else
                __nanosleep(100);
            continue;
        }
        if (st == 2) code = LS_B200_DEV_QUEUE_ERROR;
        if (st == 4) code = LS_B200_DEV_TIMEOUT_EPOCH;
        if (st == 1 && lane == 0) {
            total = ld_relaxed_gpu(ws_layer(P, l) + 7);
            ready = batch ? total : ld_acquire_gpu(ws_layer(P, l) + 5);
        }
        total = __shfl_sync(0xffffffffu, total, 0);
        ready = __shfl_sync(0xffffffffu, ready, 0);
        if ((st == 1 || st == 3) && (total > L.q.capacity || L.core_count + total > P.N || ready > total)) {
            code = LS_B200_DEV_BAD_PLAN;
            if (host_queue && lane == 0) st_release_gpu(state, kQueueFailed);
        }
        if (st == 3 && host_queue) {
            // core descriptors and the published prefix into device memory,
            // then the activation for the other CTAs
            if (!code) mirror_queue(P, L, l, 0, L.core_count + ready, lane, true);
            if (lane == 0) {
                if (!code) {
                    st_relaxed_gpu(ws_layer(P, l) + 7, total);
                    st_release_gpu(state, kQueueActive);
                }
                release_poll_lease(P);
            }
        }
        break;
    }
    uint32_t path = kPathAbort;
    if (!code && lane == 0) {
        const uint32_t proposal = ready == total ? kPathFast : kPathProgressive;
        if (batch) {
            path = proposal;
        } else {
            const uint32_t old = atomicCAS(ws_layer(P, l) + 0, 0u, proposal);
            path = old ? old : proposal;
        }
    }
    if (code && lane == 0) raise_error(P, t, code, l);
    *total_out = total;
    return __shfl_sync(0xffffffffu, path, 0);
}

__device__ void stamp(const LayerPlan& L, const DescView& d) {
    if (L.stamps) L.stamps[d.dest] = gtimer();
}

// Producer warp main loop over the layers of the launch. LEAN: every layer
// of the launch takes the fast path (BatchCompat / Auto plans on a
// device-memory queue, one GPU), so the progressive claim loop and the
// host-queue reads are not compiled in.
template <int H, bool F, bool LEAN>
__device__ void run_producer(const KernelParams& P, uint8_t* stages, SmemTail* t, uint64_t deadline) {
    Producer pr;
    pr.idx = 0;
    pr.octets = 0;
    pr.slabs = 0;
    pr.lane = threadIdx.x & 31u;
    pr.stages = stages;
    pr.t = t;
    pr.deadline = deadline;
    pr.wbase = pr.wlayer = 0xffffffffu;
    const uint32_t spg = slabs_per_group(P.G);
    bool ok = true;
    for (uint32_t l = 0; ok && l < P.nlayers; ++l) {
        // Layers 0 and 1 from the prologue's shared-memory copies (a global
        // read of the plan is a round trip on the launch's critical path; the
        // consumers overwrite those slots only after finishing layers 1 and
        // 2, which the producer has passed). Later layers from global memory:
        // the producer runs ahead of the consumers' plan fetches.
        const LayerPlan& L = l < 2 ? cplan_at(t, l) : plan_at(P, l);
        uint32_t total = 0;
        const uint32_t path = decide(P, L, l, t, deadline, pr.lane, &total);
        if (pr.lane == 0 && l == 0) trace(P, LS_B200_TRACE_DECIDED);
        if (pr.lane == 0) trace_layer(P, t, l, LS_B200_LTRACE_DECIDED);
        if (path == kPathAbort) break;
        const uint32_t D = L.core_count + total;
        const uint32_t NS = D * spg;
        pr.wbase = pr.wlayer = 0xffffffffu;
        PendingDown pd;
        pd.valid = false;
        if (LEAN || path == kPathFast) {
            // Static balanced split of the layer's slab positions.
            const uint32_t b = blockIdx.x, grid = gridDim.x;
            const uint32_t u1 = uint32_t(uint64_t(NS) * (b + 1) / grid);
            // only the descriptors of this CTA's slabs: a host-memory queue
            // costs a PCIe round trip per word read
            const uint32_t dend = u1 ? (u1 - 1) / spg + 1 : 0;
            for (uint32_t u = uint32_t(uint64_t(NS) * b / grid); ok && u < u1; ++u) {
                const uint32_t d = u / spg, slab = u % spg;
                if (pr.wlayer != l || d < pr.wbase || d >= pr.wbase + 32)
                    ok = producer_window<LEAN>(pr, P, L, l, d, dend);
                if (!ok) break;
                const DescView dv = t->dtab[d - pr.wbase];
                if (slab == 0 && pr.lane == 0) stamp(L, dv);
                ok = producer_slab<H, F>(pr, P, L, dv, l, slab, pd);
            }
        } else if constexpr (!LEAN) {
            const uint32_t* words = reinterpret_cast<const uint32_t*>(L.q.control);
            uint32_t* claim = ws_layer(P, l) + 1;
            const bool host_queue = (L.flags & kPlanHostQueue) != 0;
            uint32_t* mirror = ws_layer(P, l) + 5;
            uint32_t* state = ws_layer(P, l) + 6;
            while (ok && !t->abort) {
                uint32_t pos = 0, code = 0;
                if (pr.lane == 0) {
                    pos = atomicAdd(claim, 1u);
                    if (pos >= NS) code = 0xffffffffu;  // exhausted
                }
                pos = __shfl_sync(0xffffffffu, pos, 0);
                code = __shfl_sync(0xffffffffu, code, 0);
                if (code) break;
                if (pos / spg >= L.core_count) {
                    // Wait until the descriptor of the claimed slab is published
                    // (persistent.py:71-90; streaming_mlp.cu:63-75). A host
                    // queue is read by the lease holder, whose warp copies the
                    // newly published descriptors into the device mirror.
                    const uint32_t q = pos / spg - L.core_count;
                    uint32_t polls = 0;
                    for (;;) {
                        // lane 0: 0 wait, 1 ready, 2 queue error, 3 mirror [from, to), 4 deadline
                        uint32_t st = 0, from = 0, to = 0;
                        if (pr.lane == 0) {
                            if (!host_queue) {  // device-memory queue: read it directly
                                if (ld_acquire_sys(words + 5)) st = 2;
                                else if (ld_acquire_sys(words + 0) > q) st = 1;
                            } else {
                                const uint32_t seen = ld_acquire_gpu(mirror);
                                if (seen > q) {
                                    st = 1;
                                } else if (ld_relaxed_gpu(state) == kQueueFailed) {
                                    st = 2;
                                } else if (take_poll_lease(P)) {
                                    // error word first (relaxed), then ready_count
                                    // (acquire): both reads in flight together
                                    const uint32_t err = ld_relaxed_sys(words + 5);
                                    uint32_t ready = ld_acquire_sys(words + 0);
                                    if (err) {
                                        st_release_gpu(state, kQueueFailed);
                                        st = 2;
                                    } else {
                                        if (ready > total) ready = total;  // bounded by the plan
                                        if (ready > seen) {
                                            st = 3;
                                            from = seen;
                                            to = ready;
                                        }
                                    }
                                    if (st != 3) release_poll_lease(P);
                                }
                            }
                            if (st == 0 && gtimer() > deadline) st = 4;
                        }
                        st = __shfl_sync(0xffffffffu, st, 0);
                        if (st == 3) {
                            from = __shfl_sync(0xffffffffu, from, 0);
                            to = __shfl_sync(0xffffffffu, to, 0);
                            mirror_queue(P, L, l, L.core_count + from, L.core_count + to, pr.lane, true);
                            if (pr.lane == 0) release_poll_lease(P);
                            if (to > q) break;
                            continue;
                        }
                        if (st == 1) break;
                        if (st == 2 || st == 4) {
                            code = st == 2 ? LS_B200_DEV_QUEUE_ERROR : LS_B200_DEV_TIMEOUT_READY;
                            if (pr.lane == 0) raise_error(P, t, code, pos);
                            break;
                        }
                        if (host_queue)
                            mirror_backoff(polls++);
                        else
                            __nanosleep(128);
                    }
                    if (code) break;
                }
                const uint32_t d = pos / spg, slab = pos % spg;
                ok = producer_window<LEAN>(pr, P, L, l, d, d + 1);  // one descriptor, lane 0
                if (!ok) break;
                const DescView dv = t->dtab[0];
                if (slab == 0 && pr.lane == 0) stamp(L, dv);
                ok = producer_slab<H, F>(pr, P, L, dv, l, slab, pd);
            }
            if (t->abort) ok = false;
        }
        if (ok) ok = producer_slab_down<H, F>(pr, P, L, pd, l);
        if (pr.lane == 0) trace_layer(P, t, l, LS_B200_LTRACE_ISSUED);
        if (ok) ok = producer_marker<H>(pr, P, kPieceLayer, l, NS, t->abort ? 0u : kLayerGood);
    }
    producer_marker<H>(pr, P, kPieceFinal, 0, 0, 0);
    if (pr.lane == 0) trace(P, LS_B200_TRACE_PRODUCED);
}

// ------------------------------------------------------------ consumer side
// Bounded barrier of the 16 consumer warps (an mbarrier, 16 arrivals per
// phase). Every consumer warp passes the same sequence of these barriers;
// `phase` counts them. Returns false when the wait gave up.
__device__ bool csync(const KernelParams& P, SmemTail* t, uint32_t& phase, uint64_t limit, int lane) {
    __syncwarp();
    const uint32_t bar = smem_u32(&t->cbar);
    if (lane == 0) mbar_arrive(bar);
    const uint32_t parity = phase & 1u;
    ++phase;
    uint32_t spins = 0;
    for (;;) {
        const bool ready = mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, ready)) return true;
        uint32_t late = 0;
        if (lane == 0 && (++spins & 255u) == 0 && gtimer() > limit) late = 1;
        if (__shfl_sync(0xffffffffu, late, 0)) {
            if (lane == 0) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 8);
            return false;
        }
    }
}

// Bounded wait of one thread until *counter >= target (acquire, gpu scope).
__device__ bool wait_count(const KernelParams& P, SmemTail* t, const uint32_t* counter, uint32_t target,
                           uint64_t limit, uint32_t detail) {
    uint32_t spins = 0;
    while (ld_acquire_gpu(counter) < target) {
        if ((++spins & 63u) == 0 && gtimer() > limit) {
            raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, detail);
            return false;
        }
        __nanosleep(20);
    }
    return true;
}

// Loads the layer's input, applies the HF RMSNorm of
// predictor_shared_input.cu:16-33 when flagged
// (inv = rsqrt(sum(x^2)/H + eps); x' = fp16(weight * fp16(x * inv))), and
// stores it in the B-fragment order of the gate/up MMAs, thread u handling
// coordinates 8u..8u+7 (sub-block u/4, lane quad position u%4):
//   variant 1: x' as 22-bit fixed point, M = rint(x' * 2^(21-E)) with E the
//     exponent of an upper bound of max|x'| (|M| < 2^22; exact for every x'
//     within 2^11 of the bound, within 2^-22 of it otherwise), split into three
//     balanced signed 8-bit digits M = d0 + 256 d1 + 65536 d2; plane p holds,
//     per unit, the digits of coordinates (0,2,4,6) and (1,3,5,7);
//   variant 0: fp16 pairs (0,4) (1,5) (2,6) (3,7).
// Every CTA computes the same values in the same order.
// `tagged` (chained layers): the input is the previous layer's output, read
// from the tagged scratch copy as soon as its words carry `tag` -- no
// grid-wide barrier between layers.
template <int H, bool F>
__device__ void stage_x(const KernelParams& P, const LayerPlan& L, SmemTail* t, uint32_t& cph, uint64_t limit,
                        int tid, bool tagged, uint32_t tag) {
    constexpr int NU = H / 8, UPT = Geo<H>::UPT;  // units u = tid + j * 512, j < UPT
    const int warp = tid >> 5, lane = tid & 31;
    // The norm weights do not depend on the input: their loads are in flight
    // while the input is polled.
    const bool norm = (L.flags & LS_B200_NORM_INPUT) != 0;
    const bool weighted = norm && L.norm_w;
    uint4 nw[UPT];
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
        const int u = tid + j * kConsumerThreads;
        nw[j] = make_uint4(0u, 0u, 0u, 0u);
        if (weighted && u < NU) nw[j] = __ldg(reinterpret_cast<const uint4*>(L.norm_w) + u);
    }
    uint4 raw[UPT];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
        const int u = tid + j * kConsumerThreads;
        raw[j] = make_uint4(0u, 0u, 0u, 0u);
        if (u >= NU) continue;  // warp-uniform: NU is a multiple of 32
        if (tagged) {
            const unsigned long long* src = P.xbuf + (blockIdx.x % kXbufReplicas) * uint32_t(H / 2) + 4 * u;
            ulonglong2 a = ld_volatile_v2u64(src), b = ld_volatile_v2u64(src + 2);
            uint32_t spins = 0, polls = 0;
            for (;;) {
                const bool ok = uint32_t(a.x >> 32) == tag && uint32_t(a.y >> 32) == tag &&
                                uint32_t(b.x >> 32) == tag && uint32_t(b.y >> 32) == tag;
                if (__all_sync(0xffffffffu, ok)) break;
                uint32_t late = 0;
                if (lane == 0 && (++spins & 15u) == 0 && (t->abort || grid_failed(P) || gtimer() > limit)) late = 1;
                if (__shfl_sync(0xffffffffu, late, 0)) {
                    if (lane == 0 && !t->abort && !grid_failed(P)) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 6);
                    break;
                }
                poll_backoff(polls++, 32);
                if (!ok) {
                    a = ld_volatile_v2u64(src);
                    b = ld_volatile_v2u64(src + 2);
                }
            }
            raw[j] = make_uint4(uint32_t(a.x), uint32_t(a.y), uint32_t(b.x), uint32_t(b.y));
        } else {
            raw[j] = __ldcg(reinterpret_cast<const uint4*>(L.x) + u);
        }
        const __half2* h = reinterpret_cast<const __half2*>(&raw[j]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 v = __half22float2(h[e]);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
        }
    }
    // One reduction round: sum of squares (RMSNorm) and, for variant 1, the
    // maxima of |x| and |w| that bound max|x'| for the fixed-point exponent.
    float mx = 0.f, mw = 0.f;
    if constexpr (F) {
#pragma unroll
        for (int j = 0; j < UPT; ++j) {
            const __half* h = reinterpret_cast<const __half*>(&raw[j]);
            const __half* wh = reinterpret_cast<const __half*>(&nw[j]);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                mx = fmaxf(mx, fabsf(__half2float(h[e])));
                mw = fmaxf(mw, fabsf(__half2float(wh[e])));
            }
        }
    }
    float inv = 1.f, xbound = 0.f;
    if (norm || F) {
        if (norm) ss = warp_sum(ss);
        if constexpr (F) {
#pragma unroll
            for (int off = 16; off; off >>= 1) {
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, off));
            }
        }
        if (lane == 0) {
            t->red[warp] = ss;
            t->red2[0][warp] = mx;
            t->red2[1][warp] = mw;
        }
        csync(P, t, cph, limit, lane);
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
            tot += t->red[w];
            mx = fmaxf(mx, t->red2[0][w]);
            mw = fmaxf(mw, t->red2[1][w]);
        }
        if (norm) inv = rsqrtf(tot / float(H) + P.eps);
        // |fp16(fp16(x inv) w)| <= |x| inv |w| (1 + 2^-11)^2 < max|x| inv max|w| (1 + 2^-9)
        xbound = norm ? mx * inv * (weighted ? mw : 1.f) * (1.f + 0.001953125f) : mx;
    }
    // exponent E of the bound on max|x'|: identical in every CTA
    const int E = xbound > 0.f ? int((__float_as_uint(xbound) >> 23) & 0xffu) - 127 : 0;
    const float up = __uint_as_float(uint32_t(127 + 21 - E) << 23);  // 2^(21-E)
    if (F && tid == 0) t->xscale = __uint_as_float(uint32_t(127 - 21 + E) << 23);  // 2^(E-21)
#pragma unroll
    for (int j = 0; j < UPT; ++j) {
        const int u = tid + j * kConsumerThreads;
        if (u >= NU) continue;
        __half v[8];
        {
            const __half* h = reinterpret_cast<const __half*>(&raw[j]);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = norm ? __float2half_rn(__half2float(h[e]) * inv) : h[e];
            if (weighted) {
                const __half* wh = reinterpret_cast<const __half*>(&nw[j]);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __hmul(wh[e], v[e]);
            }
        }
        if constexpr (F) {
            uint32_t pe[3] = {0u, 0u, 0u}, po[3] = {0u, 0u, 0u};
            int msum = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int m = __float2int_rn(__half2float(v[e]) * up);
                msum += m;
                const int d0 = int(int8_t(m & 0xff));
                const int m1 = (m - d0) >> 8;
                const int d1 = int(int8_t(m1 & 0xff));
                const int d2 = (m1 - d1) >> 8;
                const int sh = 8 * (e >> 1);
                uint32_t* dst = (e & 1) ? po : pe;
                dst[0] |= uint32_t(d0 & 0xff) << sh;
                dst[1] |= uint32_t(d1 & 0xff) << sh;
                dst[2] |= uint32_t(d2 & 0xff) << sh;
            }
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                uint32_t* plane = reinterpret_cast<uint32_t*>(xarea<H>(t) + p * Geo<H>::XPL);
                plane[4 * (u >> 1) + (u & 1)] = pe[p];
                plane[4 * (u >> 1) + 2 + (u & 1)] = po[p];
            }
            msum += __shfl_xor_sync(0xffffffffu, msum, 1);
            msum += __shfl_xor_sync(0xffffffffu, msum, 2);
            if ((u & 3) == 0) xsum32<H>(t)[u >> 2] = msum;
            msum += __shfl_xor_sync(0xffffffffu, msum, 4);
            if ((u & 7) == 0) xsum64<H>(t)[u >> 3] = msum;
        } else {
            uint4 f;
            f.x = h2_bits(__halves2half2(v[0], v[4]));
            f.y = h2_bits(__halves2half2(v[1], v[5]));
            f.z = h2_bits(__halves2half2(v[2], v[6]));
            f.w = h2_bits(__halves2half2(v[3], v[7]));
            reinterpret_cast<uint4*>(xarea<H>(t))[u] = f;
        }
    }
    if (tid < int(kPlanChunks)) cp_async_wait_all();  // the next layer's plan (fetch_plan), visible after the barrier
    csync(P, t, cph, limit, lane);
}

// (even, odd) digits of 8-coordinate unit u in one plane (layout of xarea<H>).
__device__ __forceinline__ uint2 x_unit(const uint8_t* plane, int u) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(plane) + 4 * (u >> 1) + (u & 1);
    return make_uint2(w[0], w[2]);
}

// Tensor-core step on 8-bit integers: D(16x8,s32) += A(16x32,u8) * B(32x8,s8).
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// GATEUP piece: warp w reduces sub-blocks [w*SBW, (w+1)*SBW) (32 hidden
// coordinates each) for the piece's 8 neurons (MMA rows 0-7: gate rows,
// 8-15: up rows); the epilogue warp sums the warp partials in warp order and
// forms h.
//   variant 1: one integer MMA per sub-block. A = q + 8 as unsigned bytes
//     (one LOP3 per four weights: the low nibbles of a word are coordinates
//     0,2,4,6, the high nibbles 1,3,5,7); B column p = digit plane p of the
//     fixed-point x (p < 3), other columns 0. Per scale block the exact
//     integer sums give sum(q M) = D0 + 256 D1 + 65536 D2 - 8 sum(M); the
//     fp16 scale and 2^(E-21) are applied to that once.
//   variant 0: fp16 MMAs on w = fp16(q * s) (backends/triton/core.py:17).
template <int H, bool F>
__device__ void consume_gateup(const KernelParams& P, const LayerPlan& L, const Piece& pc, uint8_t* st, SmemTail* t,
                               uint32_t s, int warp, int lane) {
    constexpr int HP = Geo<H>::HP, NSB = HP / 32, AW = NSB < kConsumerWarps ? NSB : kConsumerWarps, SBW = NSB / AW;
    constexpr int CH = SBW < 4 ? SBW : 4;  // sub-blocks per scale block handled at once
    constexpr int PG = gateup_pitch<HP, F>();
    constexpr int SPN = ScaleCopy<H>::kGateUpPitch / 2;  // staged scale row (gate, up, pad) in halves
    const int g = lane >> 2, tq = lane & 3;
    const NibMasks nk = load_nib(t);
    const XPart xq = xpart<H>(t, (Geo<H>::KS > 1 && (pc.flags & kPart1)) ? 1u : 0u);
    float2* part = reinterpret_cast<float2*>(st + kStageData + kAuxPartials);  // [warp][8]
    __syncwarp();  // mma.sync is .aligned: enter converged whatever the caller's waits did
    if (warp < AW) {
        const uint8_t* rowg = st + g * PG + 4 * tq;
        const __half* sc = reinterpret_cast<const __half*>(st + kStageData) + g * SPN;
        float pg = 0.f, pu = 0.f;
        if constexpr (F) {
            // Chunks of CH sub-blocks (one scale block, or the warp's share
            // of one), their MMA chains interleaved. Low nibbles give
            // A = q + 8, high nibbles (masked in place, no shift) 16 (q + 8):
            // two exact integer accumulators, combined as lo + hi / 16.
            // B columns 3..7 are never read, so lanes g >= 3 load any plane.
            constexpr int NC = SBW / CH;
            int alo[NC][4], ahi[NC][4];
            int ms[NC];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                alo[c][0] = alo[c][1] = alo[c][2] = alo[c][3] = 0;
                ahi[c][0] = ahi[c][1] = ahi[c][2] = ahi[c][3] = 0;
            }
            const uint8_t* xp = xq.x + (g < 3 ? g : 0) * Geo<H>::XPL;
            if constexpr (CH >= 2) {
                // 64-coordinate groups: lane t reads bytes 8t..8t+7 of a row
                // (coordinates 16t..16t+15) with one 8-byte load, and the
                // matching digits (two 8-coordinate units) with one 16-byte load.
                constexpr int DC = CH / 2;
                const uint8_t* row2 = st + g * PG + 8 * tq;
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int d0 = (warp * SBW + c * CH) / 2;
                    ms[c] = xq.m64[d0];
                    if constexpr (DC == 2) ms[c] += xq.m64[d0 + 1];
                }
#pragma unroll
                for (int dj = 0; dj < DC; ++dj) {
#pragma unroll
                    for (int c = 0; c < NC; ++c) {
                        const int dg = (warp * SBW + c * CH) / 2 + dj;
                        const uint2 wg = *reinterpret_cast<const uint2*>(row2 + 32 * dg);
                        const uint2 wu = *reinterpret_cast<const uint2*>(row2 + HP / 2 + 32 * dg);
                        const uint4 xb = reinterpret_cast<const uint4*>(xp)[4 * dg + tq];
                        // even coordinates of both units, then odd ones
                        imma16832(alo[c], and_xor(wg.x, nk.lo_m, nk.lo_x), and_xor(wu.x, nk.lo_m, nk.lo_x),
                                  and_xor(wg.y, nk.lo_m, nk.lo_x), and_xor(wu.y, nk.lo_m, nk.lo_x), xb.x, xb.y);
                        imma16832(ahi[c], and_xor(wg.x, nk.hi_m, nk.hi_x), and_xor(wu.x, nk.hi_m, nk.hi_x),
                                  and_xor(wg.y, nk.hi_m, nk.hi_x), and_xor(wu.y, nk.hi_m, nk.hi_x), xb.z, xb.w);
                    }
                }
            } else {
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int sb = warp * SBW + c;
                    const uint32_t wg = *reinterpret_cast<const uint32_t*>(rowg + 16 * sb);
                    const uint32_t wu = *reinterpret_cast<const uint32_t*>(rowg + HP / 2 + 16 * sb);
                    const uint2 xb = x_unit(xp, sb * 4 + tq);
                    ms[c] = xq.m32[sb];
                    imma16832(alo[c], and_xor(wg, nk.lo_m, nk.lo_x), and_xor(wu, nk.lo_m, nk.lo_x),
                              and_xor(wg >> 4, nk.lo_m, nk.lo_x), and_xor(wu >> 4, nk.lo_m, nk.lo_x), xb.x,
                              xb.y);
                }
            }
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int blk = (warp * SBW + c * CH) / 4;
                // per digit plane p (B column p): lo + hi / 16 (exact in fp32);
                // lane (g, 0) holds planes 0,1, lane (g, 1) plane 2
                float dv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) dv[e] = fmaf(0.0625f, float(ahi[c][e]), float(alo[c][e]));
                const float dg2 = __shfl_down_sync(0xffffffffu, dv[0], 1);
                const float du2 = __shfl_down_sync(0xffffffffu, dv[2], 1);
                const float m8 = 8.f * float(ms[c]);
                const float rg = fmaf(dg2, 65536.f, fmaf(dv[1], 256.f, dv[0])) - m8;
                const float ru = fmaf(du2, 65536.f, fmaf(dv[3], 256.f, dv[2])) - m8;
                pg = fmaf(__half2float(sc[blk]), rg, pg);
                pu = fmaf(__half2float(sc[HP / 128 + blk]), ru, pu);
            }
        }
#pragma unroll
        for (int j0 = 0; j0 < SBW; j0 += CH) {
            const int blk = (warp * SBW + j0) / 4;
            if constexpr (F) {
            } else {
                float al[4] = {0.f, 0.f, 0.f, 0.f};
                const __half2 sg2 = __half2half2(sc[blk]), su2 = __half2half2(sc[HP / 128 + blk]);
#pragma unroll
                for (int j = 0; j < CH; ++j) {
                    const int sb = warp * SBW + j0 + j;
                    const uint32_t wg = *reinterpret_cast<const uint32_t*>(rowg + 16 * sb);
                    const uint32_t wu = *reinterpret_cast<const uint32_t*>(rowg + HP / 2 + 16 * sb);
                    const uint4 xv = reinterpret_cast<const uint4*>(xq.x)[sb * 4 + tq];
                    const uint32_t wg8 = wg >> 8, wu8 = wu >> 8;
                    const uint32_t g0 = h2_bits(__hmul2(int_lo(wg), sg2)), g1 = h2_bits(__hmul2(int_hi(wg), sg2));
                    const uint32_t g2 = h2_bits(__hmul2(int_lo(wg8), sg2)), g3 = h2_bits(__hmul2(int_hi(wg8), sg2));
                    const uint32_t u0 = h2_bits(__hmul2(int_lo(wu), su2)), u1 = h2_bits(__hmul2(int_hi(wu), su2));
                    const uint32_t u2 = h2_bits(__hmul2(int_lo(wu8), su2)), u3 = h2_bits(__hmul2(int_hi(wu8), su2));
                    // pairs (0,4),(2,6) then (1,5),(3,7) of the 8 coordinates 8t..8t+7
                    mma16816(al, g0, u0, g2, u2, xv.x, xv.z);
                    mma16816(al, g1, u1, g3, u3, xv.y, xv.w);
                }
                pg += al[0];
                pu += al[2];
            }
        }
        if constexpr (F) {
            pg *= t->xscale;
            pu *= t->xscale;
        }
        if (tq == 0) part[warp * 8 + g] = make_float2(pg, pu);
    }
    // The epilogue warp forms h once every consumer warp has arrived.
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&t->pbar[s]));
}

// Variant-1 sums of one GATEUP tile's scale block: per digit plane p (B
// column p), lo + hi / 16 is exact in fp32; lane (g, 0) holds planes 0 and 1
// and takes plane 2 from lane (g, 1). Returns the scaled gate and up terms.
__device__ __forceinline__ void gateup_block_terms(const int (&alo)[4], const int (&ahi)[4], int ms, float sg, float su,
                                                   float& pg, float& pu) {
    float dv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) dv[e] = fmaf(0.0625f, float(ahi[e]), float(alo[e]));
    const float dg2 = __shfl_down_sync(0xffffffffu, dv[0], 1);
    const float du2 = __shfl_down_sync(0xffffffffu, dv[2], 1);
    const float m8 = 8.f * float(ms);
    const float rg = fmaf(dg2, 65536.f, fmaf(dv[1], 256.f, dv[0])) - m8;
    const float ru = fmaf(du2, 65536.f, fmaf(dv[3], 256.f, dv[2])) - m8;
    pg = fmaf(sg, rg, pg);
    pu = fmaf(su, ru, pu);
}

// Two scale blocks per warp (H 4096): one 16-row tile's gate and up terms
// over the warp's blocks b0 = 2w and b1 = 2w + 1 with one accumulator pair.
// An MMA of block b0 has a nonzero B only in columns 0-2 (digit planes 0-2,
// supplied by lanes g < 3: x0), one of block b1 only in columns 3-5 (lanes
// 3 <= g < 6: x1); every other lane reads zeros. Each B operand is a pair
// of adjacent registers of one 16-byte load.
template <int H>
__device__ __forceinline__ void gateup_tile2(const uint8_t* row, const uint4 (&x0)[2], const uint4 (&x1)[2], int b0,
                                             int b1, const NibMasks& nk, int (&lo)[4], int (&hi)[4]) {
#pragma unroll
    for (int dj = 0; dj < 2; ++dj) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int dg = 2 * (c ? b1 : b0) + dj;
            const uint4 xb = c ? x1[dj] : x0[dj];
            const uint2 wg = *reinterpret_cast<const uint2*>(row + 32 * dg);
            const uint2 wu = *reinterpret_cast<const uint2*>(row + H / 2 + 32 * dg);
            imma16832(lo, and_xor(wg.x, nk.lo_m, nk.lo_x), and_xor(wu.x, nk.lo_m, nk.lo_x),
                      and_xor(wg.y, nk.lo_m, nk.lo_x), and_xor(wu.y, nk.lo_m, nk.lo_x), xb.x, xb.y);
            imma16832(hi, and_xor(wg.x, nk.hi_m, nk.hi_x), and_xor(wu.x, nk.hi_m, nk.hi_x),
                      and_xor(wg.y, nk.hi_m, nk.hi_x), and_xor(wu.y, nk.hi_m, nk.hi_x), xb.z, xb.w);
        }
    }
}

// Per-lane coefficients of the two-block epilogue: the lane's term for a row
// is s_b0 * (kA f0 + kB f1 - mA) + s_b1 * (kC f0 + kD f1 - mB), f the lane's two
// accumulator columns (each 16 times the digit-plane sum), m = 128 * sum(M)
// of the block (8 sum(M) at the same scale).
struct Tile2Coef {
    float kA, kB, kC, kD, mA, mB;
};
__device__ __forceinline__ Tile2Coef tile2_coef(int tq, int ms0, int ms1) {
    Tile2Coef c{0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (tq == 0) {
        c.kA = 1.f;
        c.kB = 256.f;
        c.mA = 128.f * float(ms0);
    } else if (tq == 1) {
        c.kA = 65536.f;
        c.kD = 1.f;
        c.mB = 128.f * float(ms1);
    } else if (tq == 2) {
        c.kC = 256.f;
        c.kD = 65536.f;
    }
    return c;
}
__device__ __forceinline__ void tile2_terms(const int (&lo)[4], const int (&hi)[4], const Tile2Coef& k, float sg0,
                                            float sg1, float su0, float su1, float& pg, float& pu) {
    float f[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) f[e] = float(16 * lo[e] + hi[e]);  // exact: |16 lo + hi| < 2^23
    float tg = sg0 * (fmaf(k.kB, f[1], k.kA * f[0]) - k.mA) + sg1 * (fmaf(k.kD, f[1], k.kC * f[0]) - k.mB);
    float tu = su0 * (fmaf(k.kB, f[3], k.kA * f[2]) - k.mA) + su1 * (fmaf(k.kD, f[3], k.kC * f[2]) - k.mB);
    tg += __shfl_xor_sync(0xffffffffu, tg, 1);
    tu += __shfl_xor_sync(0xffffffffu, tu, 1);
    tg += __shfl_xor_sync(0xffffffffu, tg, 2);
    tu += __shfl_xor_sync(0xffffffffu, tu, 2);
    pg = tg;
    pu = tu;
}

// Both GATEUP pieces of a 16-neuron slab in one pass (variant 1): stage A
// holds neurons 0-7, stage B neurons 8-15. Each warp reads an activation
// fragment once for the two 16-row tiles; the epilogue warp forms the 16
// values of h. The arithmetic of each tile, and the order of the warp
// partials, are those of consume_gateup.
template <int H>
__device__ void consume_gateup_pair(const KernelParams& P, const LayerPlan& L, const Piece& pa, const Piece& pb,
                                    uint8_t* sa, uint8_t* sb, SmemTail* t, uint32_t s, int warp, int lane) {
    constexpr int HP = Geo<H>::HP, NSB = HP / 32, AW = NSB < kConsumerWarps ? NSB : kConsumerWarps, SBW = NSB / AW;
    constexpr int CH = SBW < 4 ? SBW : 4;
    constexpr int NC = SBW / CH;
    constexpr int PG = gateup_pitch<HP, true>();
    constexpr int SPN = ScaleCopy<H>::kGateUpPitch / 2;
    const int g = lane >> 2, tq = lane & 3;
    const NibMasks nk = load_nib(t);
    const XPart xq = xpart<H>(t, (Geo<H>::KS > 1 && (pa.flags & kPart1)) ? 1u : 0u);
    float2* parta = reinterpret_cast<float2*>(sa + kStageData + kAuxPartials);  // [warp][8]
    float2* partb = reinterpret_cast<float2*>(sb + kStageData + kAuxPartials);
    __syncwarp();  // mma.sync is .aligned: enter converged
    if constexpr (SBW == 8) {
        // two scale blocks per warp: one accumulator pair per tile
        const int b0 = 2 * warp, b1 = b0 + 1;
        // digits of units 8 dg + 2t, 8 dg + 2t + 1 of the lane's plane, or zeros
        const uint8_t* z = reinterpret_cast<const uint8_t*>(t->zero16);
        const uint8_t* p0 = g < 3 ? xq.x + g * Geo<H>::XPL + 64 * (2 * b0) + 16 * tq : z;
        const uint8_t* p1 = (g >= 3 && g < 6) ? xq.x + (g - 3) * Geo<H>::XPL + 64 * (2 * b1) + 16 * tq : z;
        const int step0 = g < 3 ? 64 : 0, step1 = (g >= 3 && g < 6) ? 64 : 0;
        uint4 x0[2], x1[2];
#pragma unroll
        for (int dj = 0; dj < 2; ++dj) {
            x0[dj] = *reinterpret_cast<const uint4*>(p0 + dj * step0);
            x1[dj] = *reinterpret_cast<const uint4*>(p1 + dj * step1);
        }
        const Tile2Coef k = tile2_coef(tq, xq.m64[2 * b0] + xq.m64[2 * b0 + 1], xq.m64[2 * b1] + xq.m64[2 * b1 + 1]);
        int loa[4] = {0, 0, 0, 0}, hia[4] = {0, 0, 0, 0}, lob[4] = {0, 0, 0, 0}, hib[4] = {0, 0, 0, 0};
        gateup_tile2<HP>(sa + g * PG + 8 * tq, x0, x1, b0, b1, nk, loa, hia);
        gateup_tile2<HP>(sb + g * PG + 8 * tq, x0, x1, b0, b1, nk, lob, hib);
        const __half* sca = reinterpret_cast<const __half*>(sa + kStageData) + g * SPN;
        const __half* scb = reinterpret_cast<const __half*>(sb + kStageData) + g * SPN;
        float pga, pua, pgb, pub;
        tile2_terms(loa, hia, k, __half2float(sca[b0]), __half2float(sca[b1]), __half2float(sca[HP / 128 + b0]),
                    __half2float(sca[HP / 128 + b1]), pga, pua);
        tile2_terms(lob, hib, k, __half2float(scb[b0]), __half2float(scb[b1]), __half2float(scb[HP / 128 + b0]),
                    __half2float(scb[HP / 128 + b1]), pgb, pub);
        const float xs = t->xscale * 0.0625f;  // the accumulator columns are 16 times the plane sums
        if (tq == 0) {
            parta[warp * 8 + g] = make_float2(pga * xs, pua * xs);
            partb[warp * 8 + g] = make_float2(pgb * xs, pub * xs);
        }
    } else if (warp < AW) {
        const __half* sca = reinterpret_cast<const __half*>(sa + kStageData) + g * SPN;
        const __half* scb = reinterpret_cast<const __half*>(sb + kStageData) + g * SPN;
        float pga = 0.f, pua = 0.f, pgb = 0.f, pub = 0.f;
        int aloa[NC][4], ahia[NC][4], alob[NC][4], ahib[NC][4];
        int ms[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) aloa[c][e] = ahia[c][e] = alob[c][e] = ahib[c][e] = 0;
        const uint8_t* xp = xq.x + (g < 3 ? g : 0) * Geo<H>::XPL;
        if constexpr (CH >= 2) {
            constexpr int DC = CH / 2;
            const uint8_t* rowa = sa + g * PG + 8 * tq;
            const uint8_t* rowb = sb + g * PG + 8 * tq;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int d0 = (warp * SBW + c * CH) / 2;
                ms[c] = xq.m64[d0];
                if constexpr (DC == 2) ms[c] += xq.m64[d0 + 1];
            }
#pragma unroll
            for (int dj = 0; dj < DC; ++dj) {
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int dg = (warp * SBW + c * CH) / 2 + dj;
                    const uint4 xb = reinterpret_cast<const uint4*>(xp)[4 * dg + tq];
                    const uint2 wga = *reinterpret_cast<const uint2*>(rowa + 32 * dg);
                    const uint2 wua = *reinterpret_cast<const uint2*>(rowa + HP / 2 + 32 * dg);
                    const uint2 wgb = *reinterpret_cast<const uint2*>(rowb + 32 * dg);
                    const uint2 wub = *reinterpret_cast<const uint2*>(rowb + HP / 2 + 32 * dg);
                    imma16832(aloa[c], and_xor(wga.x, nk.lo_m, nk.lo_x), and_xor(wua.x, nk.lo_m, nk.lo_x),
                              and_xor(wga.y, nk.lo_m, nk.lo_x), and_xor(wua.y, nk.lo_m, nk.lo_x), xb.x, xb.y);
                    imma16832(ahia[c], and_xor(wga.x, nk.hi_m, nk.hi_x), and_xor(wua.x, nk.hi_m, nk.hi_x),
                              and_xor(wga.y, nk.hi_m, nk.hi_x), and_xor(wua.y, nk.hi_m, nk.hi_x), xb.z, xb.w);
                    imma16832(alob[c], and_xor(wgb.x, nk.lo_m, nk.lo_x), and_xor(wub.x, nk.lo_m, nk.lo_x),
                              and_xor(wgb.y, nk.lo_m, nk.lo_x), and_xor(wub.y, nk.lo_m, nk.lo_x), xb.x, xb.y);
                    imma16832(ahib[c], and_xor(wgb.x, nk.hi_m, nk.hi_x), and_xor(wub.x, nk.hi_m, nk.hi_x),
                              and_xor(wgb.y, nk.hi_m, nk.hi_x), and_xor(wub.y, nk.hi_m, nk.hi_x), xb.z, xb.w);
                }
            }
        } else {
            const uint8_t* rowa = sa + g * PG + 4 * tq;
            const uint8_t* rowb = sb + g * PG + 4 * tq;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int sbk = warp * SBW + c;
                const uint2 xb = x_unit(xp, sbk * 4 + tq);
                ms[c] = xq.m32[sbk];
                const uint32_t wga = *reinterpret_cast<const uint32_t*>(rowa + 16 * sbk);
                const uint32_t wua = *reinterpret_cast<const uint32_t*>(rowa + HP / 2 + 16 * sbk);
                const uint32_t wgb = *reinterpret_cast<const uint32_t*>(rowb + 16 * sbk);
                const uint32_t wub = *reinterpret_cast<const uint32_t*>(rowb + HP / 2 + 16 * sbk);
                imma16832(aloa[c], and_xor(wga, nk.lo_m, nk.lo_x), and_xor(wua, nk.lo_m, nk.lo_x),
                          and_xor(wga >> 4, nk.lo_m, nk.lo_x), and_xor(wua >> 4, nk.lo_m, nk.lo_x), xb.x,
                          xb.y);
                imma16832(alob[c], and_xor(wgb, nk.lo_m, nk.lo_x), and_xor(wub, nk.lo_m, nk.lo_x),
                          and_xor(wgb >> 4, nk.lo_m, nk.lo_x), and_xor(wub >> 4, nk.lo_m, nk.lo_x), xb.x,
                          xb.y);
            }
        }
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int blk = (warp * SBW + c * CH) / 4;
            gateup_block_terms(aloa[c], ahia[c], ms[c], __half2float(sca[blk]), __half2float(sca[HP / 128 + blk]), pga,
                               pua);
            gateup_block_terms(alob[c], ahib[c], ms[c], __half2float(scb[blk]), __half2float(scb[HP / 128 + blk]), pgb,
                               pub);
        }
        const float xs = t->xscale;
        if (tq == 0) {
            parta[warp * 8 + g] = make_float2(pga * xs, pua * xs);
            partb[warp * 8 + g] = make_float2(pgb * xs, pub * xs);
        }
    }
    // The epilogue warp forms h once every consumer warp has arrived.
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&t->pbar[s]));
}

// DOWN piece: warp w owns 64-column tiles [w*TPW, (w+1)*TPW); in each, lane
// (g, t) reads the 8 columns 8g..8g+7 of neurons 2t, 2t+1, 2t+8, 2t+9 and
// pairs the two neurons of each column with PRMT. MMA j (columns 8g+j and
// 8g+j+4 as rows g and g+8 of A) gets a B that is nonzero only in its own
// columns 2j (the fp16 value of h * s, or h) and 2j+1 (the fp16 residual of
// h * s), so the four MMAs of a tile share one accumulator and lane (g, t)
// ends with columns 8g+t and 8g+t+4 -- every lane stores two tagged words.
template <int H, bool F>
__device__ void consume_down(const KernelParams& P, const Piece& pc, const uint8_t* st, const SmemTail* t, int warp,
                             int lane) {
    constexpr int HP = Geo<H>::HP, NT = HP / 64, DW = NT < kConsumerWarps ? NT : kConsumerWarps, TPW = NT / DW;
    constexpr int PD = HP / 2 + 16;
    constexpr int SPN = ScaleCopy<H>::kDownPitch / 2;  // staged down-scale row in halves
    if (warp >= DW) return;
    __syncwarp();  // mma.sync is .aligned: enter converged
    const int g = lane >> 2, tq = lane & 3;
    const NibMasks nk = load_nib(t);
    const uint32_t cnt = pc.count;
    const int n0 = 2 * tq, n1 = n0 + 1, n2 = n0 + 8, n3 = n0 + 9;
    const __half zero = __float2half_rn(0.f);
    const __half* hb = t->hs[(pc.flags & kHsBuf) ? 1 : 0];
    const __half hv0 = uint32_t(n0) < cnt ? hb[n0] : zero, hv1 = uint32_t(n1) < cnt ? hb[n1] : zero;
    const __half hv2 = uint32_t(n2) < cnt ? hb[n2] : zero, hv3 = uint32_t(n3) < cnt ? hb[n3] : zero;
    const __half2 h01 = __halves2half2(hv0, hv1), h23 = __halves2half2(hv2, hv3);
    const __half* sd = reinterpret_cast<const __half*>(st + kStageData);
    // columns [kp HP, (kp + 1) HP) of the slab's partial row
    unsigned long long* out = P.partial + size_t(pc.row) * H + ((Geo<H>::KS > 1 && (pc.flags & kPart1)) ? HP : 0);
    const unsigned long long tag = static_cast<unsigned long long>(scratch_tag(t, pc.layer)) << 32;
    const int mine = g >> 1;  // the MMA whose B column g this lane supplies
    uint32_t bj0[4] = {0u, 0u, 0u, 0u}, bj1[4] = {0u, 0u, 0u, 0u}, s01 = 0, s23 = 0;
    float hsum8 = 0.f;
#pragma unroll 2  // two tiles in flight; full unrolling costs instruction-cache space
    for (int i = 0; i < TPW; ++i) {
        const int tile = warp * TPW + i;
        const int blk = tile >> 1;  // 128-column scale block
        if (i == 0 || (tile & 1) == 0) {
            const __half c0 = uint32_t(n0) < cnt ? sd[n0 * SPN + blk] : zero;
            const __half c1 = uint32_t(n1) < cnt ? sd[n1 * SPN + blk] : zero;
            const __half c2 = uint32_t(n2) < cnt ? sd[n2 * SPN + blk] : zero;
            const __half c3 = uint32_t(n3) < cnt ? sd[n3 * SPN + blk] : zero;
            uint32_t v0, v1;
            if constexpr (F) {
                // h * s split into an fp16 value (even B columns) and the fp16
                // residual (odd B columns): hi = fp16(h s), lo = fp16(h s - hi),
                // the product and the difference exact before their one
                // rounding (packed fp16 multiply and fused multiply-add). The
                // +8 offset of A is removed with their sum over the slab's 16
                // neurons.
                const __half2 c01 = __halves2half2(c0, c1), c23 = __halves2half2(c2, c3);
                const __half2 hi01 = __hmul2(h01, c01), hi23 = __hmul2(h23, c23);
                const __half2 lo01 = __hfma2(h01, c01, __hneg2(hi01)), lo23 = __hfma2(h23, c23, __hneg2(hi23));
                const float2 fh01 = __half22float2(hi01), fl01 = __half22float2(lo01);
                const float2 fh23 = __half22float2(hi23), fl23 = __half22float2(lo23);
                float hsum = fh01.x + fl01.x;
                hsum += fh01.y + fl01.y;
                hsum += fh23.x + fl23.x;
                hsum += fh23.y + fl23.y;
                v0 = (g & 1) ? h2_bits(lo01) : h2_bits(hi01);
                v1 = (g & 1) ? h2_bits(lo23) : h2_bits(hi23);
                hsum += __shfl_xor_sync(0xffffffffu, hsum, 1);
                hsum += __shfl_xor_sync(0xffffffffu, hsum, 2);
                hsum8 = -8.f * hsum;
            } else {
                v0 = (g & 1) ? 0u : h2_bits(__halves2half2(hv0, hv1));
                v1 = (g & 1) ? 0u : h2_bits(__halves2half2(hv2, hv3));
                s01 = h2_bits(__halves2half2(c0, c1));
                s23 = h2_bits(__halves2half2(c2, c3));
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                bj0[j] = j == mine ? v0 : 0u;
                bj1[j] = j == mine ? v1 : 0u;
            }
        }
        const uint8_t* base = st + 32 * tile + 4 * g;
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(base + n0 * PD);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(base + n1 * PD);
        const uint32_t w2 = *reinterpret_cast<const uint32_t*>(base + n2 * PD);
        const uint32_t w3 = *reinterpret_cast<const uint32_t*>(base + n3 * PD);
        // Interleave: [w0.b0 w0.b1 w1.b0 w1.b1] holds columns 0-3 of both neurons.
        const uint32_t p01[2] = {__byte_perm(w0, w1, 0x5410), __byte_perm(w0, w1, 0x7632)};
        const uint32_t p23[2] = {__byte_perm(w2, w3, 0x5410), __byte_perm(w2, w3, 0x7632)};
        uint32_t a01[8], a23[8];  // column c: (neuron 2t, 2t+1) and (2t+8, 2t+9)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            // bytes 1 and 3 moved down by one byte: (v * 2^24) >> 32 runs on the
            // FMA pipe, leaving the integer pipe to the nibble masks
            const uint32_t x = p01[hh], x8 = __umulhi(x, 1u << 24), y = p23[hh], y8 = __umulhi(y, 1u << 24);
            if constexpr (F) {
                a01[4 * hh + 0] = sub_lo(x, nk);
                a01[4 * hh + 1] = sub_hi(x, nk);
                a01[4 * hh + 2] = sub_lo(x8, nk);
                a01[4 * hh + 3] = sub_hi(x8, nk);
                a23[4 * hh + 0] = sub_lo(y, nk);
                a23[4 * hh + 1] = sub_hi(y, nk);
                a23[4 * hh + 2] = sub_lo(y8, nk);
                a23[4 * hh + 3] = sub_hi(y8, nk);
            } else {
                const __half2 t01 = bits_h2(s01), t23 = bits_h2(s23);
                a01[4 * hh + 0] = h2_bits(__hmul2(int_lo(x), t01));
                a01[4 * hh + 1] = h2_bits(__hmul2(int_hi(x), t01));
                a01[4 * hh + 2] = h2_bits(__hmul2(int_lo(x8), t01));
                a01[4 * hh + 3] = h2_bits(__hmul2(int_hi(x8), t01));
                a23[4 * hh + 0] = h2_bits(__hmul2(int_lo(y), t23));
                a23[4 * hh + 1] = h2_bits(__hmul2(int_hi(y), t23));
                a23[4 * hh + 2] = h2_bits(__hmul2(int_lo(y8), t23));
                a23[4 * hh + 3] = h2_bits(__hmul2(int_hi(y8), t23));
            }
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) mma16816(acc, a01[j], a01[j + 4], a23[j], a23[j + 4], bj0[j], bj1[j]);
        // D[g][2t] + D[g][2t+1]: column 8g + t; D[g+8][2t] + D[g+8][2t+1]: column 8g + t + 4
        float v0 = acc[0] + acc[1], v1 = acc[2] + acc[3];
        if constexpr (F) {
            const float k = (tq & 1) ? 1048576.f : 16777216.f;  // odd column: 16 (q + 8) 2^-24; even: (q + 8) 2^-24
            v0 = fmaf(k, v0, hsum8);
            v1 = fmaf(k, v1, hsum8);
        }
        // One exchange with the neighbour lane gives every lane two adjacent
        // columns: even t keeps 8g+t and takes 8g+t+1, odd t takes 8g+t+3 and
        // keeps 8g+t+4. A warp then writes its tile's 64 tagged words with
        // one 16-byte store per lane, 512 contiguous bytes (full sectors).
        const float send = (tq & 1) ? v0 : v1;
        const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
        const float lo = (tq & 1) ? recv : v0, hi = (tq & 1) ? v1 : recv;
        st_volatile_v2u64(out + 64 * tile + 8 * g + ((tq & 1) ? tq + 3 : tq), tag | __float_as_uint(lo),
                          tag | __float_as_uint(hi));
    }
}

// One reduced column c of a layer (warp 0 of a reducer, lane = c % 32): y16 =
// fp16(y), hidden_out = fp16(residual + y16); with `chain` the pair word of
// hidden_out goes to every copy of the tagged hand-off first (the next
// layer's input is on the critical path, and it is published even after an
// error so that no reader waits for it), then the outputs are written unless
// an error had been reported when the reduction started (best effort: the
// error word decides).
template <int H>
__device__ __forceinline__ void emit_column(const KernelParams& P, const LayerPlan& L, SmemTail* t, uint32_t c,
                                            float y, uint16_t res, uint32_t err, bool good, uint32_t tag, bool chain,
                                            int lane) {
    const __half y16 = __float2half_rn(y);
    __half hout = y16;
    if (L.hidden_out && L.residual) hout = __float2half_rn(h2f(res) + __half2float(y16));
    if (chain) {
        // pair word of columns (c & ~1, c | 1) on both lanes of the pair; the
        // even lane writes the first half of the copies, the odd lane the rest
        const uint32_t mine = __half_as_ushort(hout);
        const uint32_t odd = __shfl_down_sync(0xffffffffu, mine, 1);
        const uint32_t pair = __shfl_sync(0xffffffffu, (odd << 16) | mine, lane & ~1);
        const unsigned long long word = (static_cast<unsigned long long>(tag) << 32) | pair;
        constexpr uint32_t kHalf = kXbufReplicas / 2;
        const uint32_t r0 = (lane & 1) * kHalf;
#pragma unroll
        for (uint32_t r = 0; r < kHalf; ++r) st_volatile_u64(P.xbuf + (r0 + r) * uint32_t(H / 2) + c / 2, word);
    }
    uint32_t write = 0;
    if (lane == 0) write = (good && err == 0u && !t->abort) ? 1u : 0u;
    write = __shfl_sync(0xffffffffu, write, 0);
    if (write) {
        if (L.y32) L.y32[c] = y;
        if (L.y && !(L.flags & LS_B200_NO_OUTPUT)) L.y[c] = __half_as_ushort(y16);
        if (L.hidden_out && L.residual) L.hidden_out[c] = __half_as_ushort(hout);
    }
}

// End of layer l: partial rows -> reduction -> epilogue, on CTAs 0..H/32-1
// (one 32-column block each). Each warp polls its rows until they carry the
// layer's tag, so the reduction starts without a grid-wide barrier.
// Canonical sum per column: rows in chunks of 16 (row order inside a chunk),
// chunk c added to warp c % 16's running sum in chunk order, then the 16 warp
// sums in warp order (reduction.py:6-28, streaming_mlp.cu:80-84 sum rows in
// row order). With `chain`, hidden_out is also published as tagged fp16 pairs
// for the next layer of the launch.
template <int H, bool LEAN>
__device__ void end_layer(const KernelParams& P, const LayerPlan& L, uint32_t l, uint32_t rows, bool good,
                          SmemTail* t, uint32_t& cph, uint64_t limit, int tid, bool chain) {
    constexpr uint32_t NBLK = H / 32;
    const int warp = tid >> 5, lane = tid & 31;
    // CTA b reduces column blocks b, b + grid, ... (one block each with a
    // full grid). A fixed assignment costs no claim round trip at the end of
    // every layer; a reducer that is still computing when the other rows are
    // in reads them in one round trip, as an early reducer would detect its
    // last rows.
    const uint32_t blk0 = blockIdx.x, step = gridDim.x;
    if (blk0 >= NBLK) return;
    const uint32_t tag = scratch_tag(t, l);
    const uint32_t nch = (rows + 15) / 16;
    // Blocks are reduced in rounds: with two or more blocks left (hidden
    // sizes above 32 x grid, e.g. H 8192), warps 0..7 take one block and
    // warps 8..15 the next, so both blocks' row polls overlap and share the
    // round's two barriers; a single block takes all 16 warps. A block's sum
    // order is fixed by the round (chunks c = gw, gw + WG, ... per warp, then
    // the warps of its group in order), so every launch with the same grid
    // gives the same bits.
    // Pairing is compiled only where a full grid leaves CTAs with two
    // blocks (H / 32 > 148); smaller sizes keep the one-block loop as is.
    constexpr bool kPair = NBLK > 148;
    for (uint32_t blk_r = blk0; blk_r < NBLK;) {
        const uint32_t nb = kPair && blk_r + step < NBLK ? 2u : 1u;
        const uint32_t WG = kConsumerWarps / nb, grp = uint32_t(warp) / WG, gw = uint32_t(warp) % WG;
        const uint32_t blk = blk_r + grp * step;
        // the residual and the error word are read now, off the critical
        // path of the last rows
        uint16_t res = 0;
        uint32_t err = 0;
        if (gw == 0 && L.hidden_out && L.residual) res = __ldcg(L.residual + 32 * blk + lane);
        if (gw == 0 && lane == 0) err = ld_relaxed_gpu(P.ws + kWsErr);
        float acc = 0.f;
        for (uint32_t c = gw; c < nch; c += WG) {
            const unsigned long long* p = P.partial + size_t(16 * c) * H + 32 * blk + lane;
            const uint32_t nr = rows - 16 * c < 16u ? rows - 16 * c : 16u;
            unsigned long long w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
                w[e] = uint32_t(e) < nr ? ld_volatile_u64(p + size_t(e) * H) : (static_cast<unsigned long long>(tag) << 32);
            uint32_t spins = 0, polls = 0;
            for (;;) {
                bool ok = true;
#pragma unroll
                for (int e = 0; e < 16; ++e) ok &= uint32_t(w[e] >> 32) == tag;
                if (__all_sync(0xffffffffu, ok)) break;
                uint32_t late = 0;
                if (lane == 0 && (++spins & 15u) == 0 && (t->abort || grid_failed(P) || gtimer() > limit)) late = 1;
                if (__shfl_sync(0xffffffffu, late, 0)) {
                    if (lane == 0 && !t->abort && !grid_failed(P)) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 5);
                    break;
                }
                poll_backoff(polls++, 64);
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    if (uint32_t(w[e] >> 32) != tag) w[e] = ld_volatile_u64(p + size_t(e) * H);
            }
            float cs = __uint_as_float(uint32_t(w[0]));
#pragma unroll
            for (int e = 1; e < 16; ++e) cs += __uint_as_float(uint32_t(w[e]));
            acc += cs;
        }
        t->red2[warp][lane] = acc;
        csync(P, t, cph, limit, lane);
        if (gw == 0) {
            if (blk == blk0 && lane == 0) trace_layer(P, t, l, LS_B200_LTRACE_PARTIALS_READY);
            float y = 0.f;
            for (uint32_t w = 0; w < WG; ++w) y += t->red2[grp * WG + w][lane];
            const uint32_t c = 32 * blk + lane;
            if (!LEAN && P.world > 1) {
                // Tensor parallel: this rank's fp32 partial of the column goes
                // to every rank's exchange buffer over NVLink (peer stores);
                // the ranks' partials are summed in the gather pass below.
                const uint32_t slot = (tag - 1u) & 1u;
                const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(y);
                const size_t at = (size_t(slot) * P.world + P.rank) * H + c;
                for (uint32_t r = 0; r < P.world; ++r) st_volatile_u64(P.xpeer[r] + at, w);
            } else {
                emit_column<H>(P, L, t, c, y, res, err, good, tag, chain, lane);
            }
        }
        csync(P, t, cph, limit, lane);  // red2 is reused by the next round
        blk_r += nb * step;
    }
    if (!LEAN && P.world > 1 && warp == 0) {
        // Gather pass (tensor parallel): every block of this CTA was published
        // above, so no rank waits on another while holding back its own. Each
        // block's columns of every rank are read from the local exchange
        // buffer once they carry the tag and summed in rank order (the
        // allreduce, the same bits on every rank); the block then continues
        // as on one GPU.
        // Slot reuse: slot (tag-1)&1 of rank q still holds layer l-2 until q's
        // reducers of l-2 have read it. A rank publishes layer l only after its
        // CTAs computed layer l, which needs the whole input of layer l, hence
        // every rank's layer l-1 partials; a rank publishes those only after
        // its own CTAs loaded the input of layer l-1, which its reducers of
        // layer l-2 had formed from the slot.
        const uint32_t slot = (tag - 1u) & 1u;
        const uint32_t err = ld_relaxed_gpu(P.ws + kWsErr);
        for (uint32_t blk = blk0; blk < NBLK; blk += step) {
            const uint32_t c = 32 * blk + lane;
            const uint16_t res = (L.hidden_out && L.residual) ? __ldcg(L.residual + c) : uint16_t(0);
            const unsigned long long* mine = P.xpeer[P.rank] + size_t(slot) * P.world * H + c;
            float y = 0.f;
            for (uint32_t r = 0; r < P.world; ++r) {
                unsigned long long v = ld_volatile_u64(mine + size_t(r) * H);
                uint32_t spins = 0, polls = 0;
                while (!__all_sync(0xffffffffu, uint32_t(v >> 32) == tag)) {
                    uint32_t late = 0;
                    if (lane == 0 && (++spins & 15u) == 0 && (t->abort || grid_failed(P) || gtimer() > limit))
                        late = 1;
                    if (__shfl_sync(0xffffffffu, late, 0)) {
                        if (lane == 0 && !t->abort && !grid_failed(P)) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 11);
                        break;
                    }
                    poll_backoff(polls++, 32);
                    if (uint32_t(v >> 32) != tag) v = ld_volatile_u64(mine + size_t(r) * H);
                }
                y += __uint_as_float(uint32_t(v));
            }
            emit_column<H>(P, L, t, c, y, res, __shfl_sync(0xffffffffu, err, 0), good, tag, chain, lane);
        }
    }
    // Importance output (CTA 0, which reduced column block 0 and so saw every
    // partial row of the layer, hence every h and its importance addition):
    // each destination's exact sum of |h| * 2^24, read and reset to zero in
    // one exchange, rounded to fp32 once and scaled by 2^-24; then the epoch
    // is released (leanstream_mapped.cu:36-39, 43-47). After the column
    // block's outputs, off the next layer's input path.
    if (L.importance && blockIdx.x == 0) {
        __threadfence();
        unsigned long long* acc = P.impacc + size_t(l & 1u) * P.N;
        for (uint32_t d = uint32_t(tid); d < P.N; d += kConsumerThreads)
            L.importance[d] = float(atomicExch(acc + d, 0ull)) * 5.9604644775390625e-8f;  // 2^-24
        csync(P, t, cph, limit, lane);
        if (tid == 0 && L.imp_flag) {
            __threadfence_system();
            st_release_sys(L.imp_flag, L.epoch);
        }
    }
    // Reduced blocks: an unchained next layer (or the host's view of the
    // layer outputs) waits on this count. A chained next layer reads the
    // tagged words instead, so the fence stays off its critical path.
    if (warp == 0 && !chain) {
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_gpu(ws_layer(P, l) + 3, 1u);
    }
    if (tid == 0) trace_layer(P, t, l, LS_B200_LTRACE_REDUCED);
}

// Sums of neuron i's gate and up warp partials ([warp][8] float2 in a
// GATEUP stage's aux area), in warp order.
template <int H>
__device__ __forceinline__ float2 sum_partials(const uint8_t* st, uint32_t i) {
    constexpr int NSB = Geo<H>::HP / 32, AW = NSB < kConsumerWarps ? NSB : kConsumerWarps;
    const float2* part = reinterpret_cast<const float2*>(st + kStageData + kAuxPartials);
    float gsum = 0.f, usum = 0.f;
#pragma unroll
    for (int w = 0; w < AW; ++w) {
        const float2 v = part[w * 8 + i];
        gsum += v.x;
        usum += v.y;
    }
    return make_float2(gsum, usum);
}

// h from the gate and up sums, each rounded to fp16, then
// fp16(fp16(silu(g)) * u) (kernels/streaming_mlp.cu:34-37,
// backends/triton/core.py:49-52), for neuron n of the slab.
// With an importance output, |h| * 2^24 -- an integer below 2^40 for every
// fp16 value -- is added to the destination's 64-bit sum of this layer's
// parity, so the per-group sum of |h| is exact and does not depend on which
// CTA formed which neuron (examples/ministral/native/leanstream_mapped.cu:43-47
// sums the group's |h| in fp32).
__device__ __forceinline__ void finish_h(const KernelParams& P, const LayerPlan& L, SmemTail* t, uint32_t buf,
                                         uint32_t dest, uint32_t n, float2 gu, uint32_t layer) {
    const float g16 = round16(gu.x), u16 = round16(gu.y);
    const float sl = round16(g16 / (1.f + expf(-g16)));
    const __half h = __float2half_rn(sl * u16);
    t->hs[buf][n & (kSlab - 1)] = h;
    if (L.act) L.act[size_t(dest) * P.G + n] = __half_as_ushort(h);
    if (L.importance)
        atomicAdd(P.impacc + size_t(layer & 1u) * P.N + dest,
                  static_cast<unsigned long long>(fabsf(__half2float(h)) * 16777216.f));
}

// Bounded wait of a warp on an mbarrier phase; false on abort or deadline.
__device__ bool wait_phase(const KernelParams& P, SmemTail* t, uint32_t bar, uint32_t parity, uint64_t limit,
                           int lane, uint32_t detail) {
    uint32_t spins = 0;
    for (;;) {
        const bool ready = mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, ready)) return true;
        uint32_t late = 0;
        if (lane == 0 && (t->abort || ((++spins & 255u) == 0 && gtimer() > limit))) late = 1;
        if (__shfl_sync(0xffffffffu, late, 0)) {
            if (lane == 0 && !t->abort) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, detail);
            return false;
        }
        __nanosleep(32);  // the epilogue warp shares a scheduler with four consumer warps
    }
}

// Warp-uniform bounded wait until piece `idx`'s stage is full (acquire of
// the TMA-written data). False when the producer stopped without a FINAL
// marker.
template <int H>
__device__ bool wait_full(SmemTail* t, uint32_t idx, uint64_t deadline, int lane, uint32_t backoff_ns = 0) {
    constexpr uint32_t NS = Geo<H>::NS;
    const uint32_t bar = smem_u32(&t->full_bar[idx % NS]);
    const uint32_t parity = (idx / NS) & 1u;
    uint32_t spins = 0;
    for (;;) {
        const bool ready = mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, ready)) return true;
        uint32_t late = 0;
        if (lane == 0 && (++spins & 255u) == 0 && gtimer() > deadline + kConsumerGraceNs) late = 1;
        if (__shfl_sync(0xffffffffu, late, 0)) return false;
        if (backoff_ns) __nanosleep(backoff_ns);
    }
}

template <int H, bool F, bool LEAN>
__device__ void run_consumers(const KernelParams& P, uint8_t* stages, SmemTail* t, uint64_t deadline) {
    constexpr uint32_t NBLK = H / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t limit = deadline + kSyncGraceNs;
    uint32_t cph = 0;  // consumer-barrier phase
    uint32_t l = 0;
    const LayerPlan* L = &cplan_at(t, 0);  // slots 0 and 1 were filled in the prologue
    stage_x<H, F>(P, *L, t, cph, limit, tid, false, 0);
    for (uint32_t idx = 0;; ++idx) {
        const uint32_t s = idx % Geo<H>::NS;
        if (!wait_full<H>(t, idx, deadline, lane)) {
            // The producer stopped without a FINAL marker; nothing is in
            // flight for this stage.
            if (lane == 0) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 4);
            break;
        }
        const Piece pc = t->piece[s];
        if (tid == 0) trace_piece(P, t, idx, 2);
        if (idx == 0 && tid == 0) trace(P, LS_B200_TRACE_FIRST);
        if (tid == 0 && pc.kind == kPieceLayer) trace_layer(P, t, l, LS_B200_LTRACE_PIECES_DONE);
        if (pc.kind == kPieceFinal) {
            if (tid == 0) trace(P, LS_B200_TRACE_PIECES);
            break;
        }
        uint8_t* st = stages + size_t(s) * kStageBytes;
        if (pc.kind == kPieceGateUp) {
            if constexpr (F) {
                if (pc.flags & kPaired) {
                    // the slab's second GATEUP piece is the next stage
                    if (!wait_full<H>(t, idx + 1, deadline, lane)) {
                        if (lane == 0) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 4);
                        break;
                    }
                    const uint32_t s2 = (idx + 1) % Geo<H>::NS;
                    const Piece pc2 = t->piece[s2];
                    if (tid == 0) trace_piece(P, t, idx + 1, 2);
                    consume_gateup_pair<H>(P, *L, pc, pc2, st, stages + size_t(s2) * kStageBytes, t, s, warp, lane);
                    __syncwarp();
                    if (lane == 0) trace_warp(P, t, idx + 1, warp);
                    if (tid == 0) {
                        trace_piece(P, t, idx, 3);
                        trace_piece(P, t, idx + 1, 3);
                    }
                    if (lane == 0) {
                        mbar_arrive(smem_u32(&t->empty_bar[s]));
                        mbar_arrive(smem_u32(&t->empty_bar[s2]));
                    }
                    ++idx;
                    continue;
                }
            }
            // every warp takes part (the last one finalises h)
            consume_gateup<H, F>(P, *L, pc, st, t, s, warp, lane);
        } else if (pc.kind == kPieceDown) {
            // h of the slab: finalised by the last warp of its GATEUP pieces.
            // Every lane polls, so the warp leaves the wait converged (the
            // MMAs that follow are .aligned).
            bool ok = true;
            uint32_t sp = 0;
            for (;;) {
                if (__all_sync(0xffffffffu, t->octets_done >= pc.need)) break;
                uint32_t late = 0;
                if (lane == 0 && (t->abort || ((++sp & 255u) == 0 && gtimer() > limit))) late = 1;
                if (__shfl_sync(0xffffffffu, late, 0)) {
                    if (lane == 0 && !t->abort) raise_error(P, t, LS_B200_DEV_TIMEOUT_SYNC, 9);
                    ok = false;
                    break;
                }
                __nanosleep(32);  // leave issue slots to the warp that finalises h
            }
            __threadfence_block();
            const bool aborted = __shfl_sync(0xffffffffu, t->abort, 0) != 0;
            if (ok && !aborted) {
                consume_down<H, F>(P, pc, st, t, warp, lane);
                if ((pc.flags & kCompletes) && tid == 0 && L->execs) atomicAdd(L->execs + pc.dest, 1u);
            }
        }
        __syncwarp();
        if (tid == 0) trace_piece(P, t, idx, 3);
        if (lane == 0) trace_warp(P, t, idx, warp);
        if (lane == 0) mbar_arrive(smem_u32(&t->empty_bar[s]));
        if (pc.kind != kPieceLayer) continue;

        // ---- end of layer l: partial rows -> reduction -> next activation.
        // Chained layers (the next input is this layer's hidden_out) hand the
        // activation over through tagged words; otherwise every CTA waits
        // until all column blocks are reduced and reads the next input.
        fetch_plan(P, t, l + 2, tid);  // slot (l+2) % 3 held layer l-1, whose hand-off is over
        const LayerPlan* next = l + 1 < P.nlayers ? &cplan_at(t, l + 1) : nullptr;
        const bool chain = next && L->hidden_out && L->residual &&
                           reinterpret_cast<const void*>(next->x) == reinterpret_cast<const void*>(L->hidden_out);
        end_layer<H, LEAN>(P, *L, l, pc.count, (pc.flags & kLayerGood) != 0, t, cph, limit, tid, chain);
        if (!next) continue;  // the FINAL marker follows
        if (!chain) {
            if (tid == 0) wait_count(P, t, ws_layer(P, l) + 3, NBLK, limit, 6);
            csync(P, t, cph, limit, lane);
        }
        if (tid == 0) trace_layer(P, t, l, LS_B200_LTRACE_NEXT_READY);
        const uint32_t tag = scratch_tag(t, l);
        ++l;
        L = next;
        stage_x<H, F>(P, *L, t, cph, limit, tid, chain, tag);
        if (tid == 0) trace_layer(P, t, l, LS_B200_LTRACE_LOADED);
    }
}

// Epilogue warp: follows the pieces in ring order and, for each GATEUP
// piece (or pair), waits until the 16 consumer warps have written their
// partials, forms h and publishes it to the DOWN piece through octets_done.
// It is the stage's 17th release, so a stage is refilled only after its
// partials were read. Keeping this off the consumer warps removes a serial
// step from whichever warp finished a GATEUP piece last.
template <int H, bool F>
__device__ void run_epilogue(const KernelParams& P, uint8_t* stages, SmemTail* t, uint64_t deadline) {
    const int lane = threadIdx.x & 31;
    const uint64_t limit = deadline + kSyncGraceNs;
    uint32_t phases = 0;  // completed-phase parity of each stage's pbar
    float2 carry = make_float2(0.f, 0.f);  // gate/up sums of a slab's first K part
    for (uint32_t idx = 0;; ++idx) {
        const uint32_t s = idx % Geo<H>::NS;
        // back off between polls: this warp shares a scheduler with four
        // consumer warps, whose pieces finish at the pace of the slowest
        if (!wait_full<H>(t, idx, deadline, lane, 64)) break;  // the consumers report it
        const Piece pc = t->piece[s];
        if (pc.kind == kPieceFinal) break;
        if (pc.kind == kPieceGateUp) {
            if (!wait_phase(P, t, smem_u32(&t->pbar[s]), (phases >> s) & 1u, limit, lane, 10)) break;
            phases ^= 1u << s;
            const LayerPlan& L = cplan_at(t, pc.layer);
            const uint32_t buf = (pc.flags & kHsBuf) ? 1u : 0u;
            const bool paired = F && (pc.flags & kPaired);
            uint32_t s2 = s, cnt = pc.count, n0 = pc.n0, i = uint32_t(lane);
            const uint8_t* sq = stages + size_t(s) * kStageBytes;
            if (paired) {
                // the consumers saw the second stage full before writing
                // their partials; this wait returns at once
                if (!wait_full<H>(t, idx + 1, deadline, lane)) break;
                s2 = (idx + 1) % Geo<H>::NS;
                i = uint32_t(lane) & 7u;
                if (lane >= 8) {
                    cnt = lane < 16 ? t->piece[s2].count : 0u;
                    n0 = t->piece[s2].n0;
                    sq = stages + size_t(s2) * kStageBytes;
                }
            }
            const bool mine = i < cnt;
            float2 gu = mine ? sum_partials<H>(sq, i) : make_float2(0.f, 0.f);
            // The partials are in registers: the stages may be refilled while
            // h is formed.
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_u32(&t->empty_bar[s]));
                if (paired) mbar_arrive(smem_u32(&t->empty_bar[s2]));
            }
            if constexpr (Geo<H>::KS > 1) {
                // K parts of a slab follow each other: the first part's sums
                // wait in registers for the second's
                if (!(pc.flags & kPart1)) {
                    carry = gu;
                    if (paired) ++idx;
                    continue;
                }
                gu = make_float2(carry.x + gu.x, carry.y + gu.y);
            }
            if (mine) finish_h(P, L, t, buf, pc.dest, n0 + i, gu, pc.layer);
            __syncwarp();
            // the importance additions are performed before the slab's DOWN
            // piece (and so its partial row) can be computed: the reducer that
            // converts them has seen every partial row of the layer
            if (L.importance) __threadfence();
            __threadfence_block();
            if (lane == 0) t->octets_done = t->octets_done + (paired ? 2u : 1u);
            if (paired) ++idx;
            continue;
        }
        if (lane == 0) mbar_arrive(smem_u32(&t->empty_bar[s]));
    }
}

template <int H, bool F, bool LEAN>
__global__ void __launch_bounds__(kThreads, 1) fused_mlp_kernel(const __grid_constant__ KernelParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stages = smem;
    SmemTail* t = reinterpret_cast<SmemTail*>(smem + size_t(Geo<H>::NS) * kStageBytes);
    const int tid = threadIdx.x;
    const uint64_t entry = gtimer(), deadline = entry + P.timeout_ns;
    if (tid == 0) {
        trace(P, LS_B200_TRACE_ENTRY);
        for (int s = 0; s < Geo<H>::NS; ++s) {
            mbar_init(smem_u32(&t->full_bar[s]), 34);                // lane 0 expect_tx + 32 cp.async + lane 0 close
            mbar_init(smem_u32(&t->empty_bar[s]), kConsumerWarps + 1);  // consumer warps + epilogue warp
            mbar_init(smem_u32(&t->pbar[s]), kConsumerWarps);
        }
        mbar_init(smem_u32(&t->cbar), kConsumerWarps);
        t->octets_done = 0;
        t->abort = 0;
        t->tagbase = ld_relaxed_gpu(P.ws + kWsTag);  // advanced by the previous launch's last CTA
        t->zero16[0] = t->zero16[1] = t->zero16[2] = t->zero16[3] = 0u;
        const uint32_t nib[8] = {0x0F0F0F0Fu, 0x08080808u, 0xF0F0F0F0u, 0x80808080u,
                                 0x000F000Fu, 0x00080008u, 0x00F000F0u, 0x00800080u};
        for (int i = 0; i < 8; ++i) t->nib[i] = nib[i];
        t->flag = 0;
        t->last = 0;
        fence_mbar_init();
    }
#if LS_KERNEL_TRACE
    for (uint32_t i = tid; i < kTracePieces * 4; i += blockDim.x) (&t->tpiece[0][0])[i] = 0u;
    for (uint32_t i = tid; i < kTraceLayers * LS_B200_LAYER_TRACE_WORDS; i += blockDim.x) (&t->tlayer[0][0])[i] = 0u;
    for (uint32_t i = tid; i < kTraceWarpPieces * kConsumerWarps; i += blockDim.x) (&t->twarp[0][0])[i] = 0u;
#endif
    if (tid < int(2 * kPlanChunks) && uint32_t(tid) / kPlanChunks < P.nlayers) {
        const uint32_t l = uint32_t(tid) / kPlanChunks, c = uint32_t(tid) % kPlanChunks;
        reinterpret_cast<uint4*>(&t->cplan[l])[c] = reinterpret_cast<const uint4*>(&plan_at(P, l))[c];
    }
    __syncthreads();

    if (tid >= kConsumerThreads + 32) {
        run_epilogue<H, F>(P, stages, t, deadline);
    } else if (tid >= kConsumerThreads) {
        run_producer<H, F, LEAN>(P, stages, t, deadline);
    } else {
        run_consumers<H, F, LEAN>(P, stages, t, deadline);
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
            P.ws[kWsPollLock] = 0;  // every holder has released it; no CTA is left
            uint32_t next_base = t->tagbase + nl;
            if (next_base >= kTagWrap) next_base -= kTagWrap;
            P.ws[kWsTag] = next_base;
            __threadfence();
        }
        __syncthreads();
        // Per-layer completion epochs: one thread per layer reads its plan and
        // publishes (system-scope fence, then the store), in parallel. One
        // thread doing all layers in turn paid a plan load and a system-scope
        // release per layer in series (tens of us for a 36-layer launch).
        for (uint32_t l = tid; l < nl; l += blockDim.x) {
            const LayerPlan& L = plan_at(P, l);
            const uint32_t layer = L.layer, epoch = L.epoch;
            __threadfence_system();
            st_relaxed_sys(P.done + layer, epoch);
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t next_base = t->tagbase + nl;
            if (next_base >= kTagWrap) next_base -= kTagWrap;
            st_relaxed_sys(P.status + LS_B200_STATUS_LAUNCHES, next_base);
        }
    }
    flush_trace(P, t, entry);
    if (tid == 0) trace(P, LS_B200_TRACE_EXIT);
}

template <int H, bool F>
static int launch_t(const KernelParams& p, int grid, cudaStream_t stream) {
    if (p.lean)
        fused_mlp_kernel<H, F, true><<<grid, kThreads, kernel_smem_bytes<H>(), stream>>>(p);
    else
        fused_mlp_kernel<H, F, false><<<grid, kThreads, kernel_smem_bytes<H>(), stream>>>(p);
    return int(cudaGetLastError());
}

template <int H, bool F>
static cudaError_t raise_smem() {
    static_assert(kernel_smem_bytes<H>() <= 232448, "dynamic shared memory of one CTA");
    cudaError_t e = cudaFuncSetAttribute(fused_mlp_kernel<H, F, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(kernel_smem_bytes<H>()));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fused_mlp_kernel<H, F, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(kernel_smem_bytes<H>()));
    return e;
}

int prepare() {
    const cudaError_t errs[] = {raise_smem<256, false>(),  raise_smem<512, false>(), raise_smem<1024, false>(),
                                raise_smem<2048, false>(), raise_smem<4096, false>(), raise_smem<256, true>(),
                                raise_smem<512, true>(),   raise_smem<1024, true>(),  raise_smem<2048, true>(),
                                raise_smem<4096, true>(),  raise_smem<8192, true>()};
    for (cudaError_t e : errs)
        if (e != cudaSuccess) return int(e);
    return 0;
}

// H in {256, 512, 1024, 2048, 4096, 8192}; variant 0 up to 4096 (the
// backend selects variant 1 above). p.lean selects the instance without the
// progressive, host-queue and tensor-parallel paths.
int launch(const KernelParams& p, int grid, cudaStream_t stream) {
    const bool f = p.variant != 0;
    switch (p.H) {
        case 256: return f ? launch_t<256, true>(p, grid, stream) : launch_t<256, false>(p, grid, stream);
        case 512: return f ? launch_t<512, true>(p, grid, stream) : launch_t<512, false>(p, grid, stream);
        case 1024: return f ? launch_t<1024, true>(p, grid, stream) : launch_t<1024, false>(p, grid, stream);
        case 2048: return f ? launch_t<2048, true>(p, grid, stream) : launch_t<2048, false>(p, grid, stream);
        case 4096: return f ? launch_t<4096, true>(p, grid, stream) : launch_t<4096, false>(p, grid, stream);
        case 8192: return f ? launch_t<8192, true>(p, grid, stream) : int(cudaErrorInvalidValue);
        default: return int(cudaErrorInvalidValue);
    }
}

}  // namespace LS_KERNEL_NS

#if LS_KERNEL_TRACE
int prepare_kernels_traced() { return traced::prepare(); }
int launch_fused_traced(const KernelParams& p, int grid, cudaStream_t stream) {
    return traced::launch(p, grid, stream);
}
#else
int prepare_kernels() {
    const int rc = plain::prepare();
    return rc ? rc : prepare_kernels_traced();
}
int launch_fused(const KernelParams& p, int grid, cudaStream_t stream) {
    return p.trace ? launch_fused_traced(p, grid, stream) : plain::launch(p, grid, stream);
}
#endif

}  // namespace lsb
