// Internal types shared by the host backend (ls_backend.cu) and the fused
// layer kernel (ls_kernel.cu). Not part of the public ABI.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>
#include "../../include/leanstream_b200.h"

namespace lsb {

// CTA shape: sixteen consumer warps plus one TMA producer warp, one CTA per SM.
constexpr int kConsumerWarps = 16;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 64;  // + producer warp + epilogue warp

// Work unit: a slab of up to 16 consecutive neurons of one descriptor. One
// CTA computes a slab's gate/up rows, its h values and its down rows, and
// writes the slab's fp32 partial output row; h never leaves the CTA.
constexpr uint32_t kSlab = 16;

// Shared-memory ring: a stage holds either the gate+up records of 8 neurons
// (pitch H + 16 bytes) or the down rows of one slab (pitch H/2 + 16 bytes),
// plus an auxiliary area with the stage's fp16 scales (one row per neuron,
// padded by 16 bytes so that the rows start in different banks; <= 1280 B)
// and the GATEUP warp partials (1 KB). Six stages = two slabs of H = 4096.
constexpr int kStages = 6;
constexpr int kStageData = 33024;  // 16 x (2048 + 16) = 8 x (4096 + 16) + 128
constexpr int kStageAux = 2304;
constexpr int kAuxPartials = 1280;  // aux offset of the GATEUP warp partials
constexpr int kStageBytes = kStageData + kStageAux;
constexpr int kMaxGroupSize = 256;
constexpr int kMaxHidden = 8192;
constexpr int kMaxPieceHidden = 4096;  // hidden extent of one staged piece
constexpr int kMaxRanks = 8;       // tensor-parallel ranks of one in-kernel exchange

// One MLP layer of a launch (POD, copied into kernel parameters or read from
// a device array for multi-layer launches).
struct alignas(16) LayerPlan {
    const uint16_t* x;        // fp16 [H] input (normalised in-kernel when flagged)
    uint16_t* y;              // fp16 [H] output (optional)
    const uint8_t* cache;
    const uint8_t* staging;
    const uint16_t* scales;
    const ls_exec_desc* core;
    ls_device_exec_queue q;
    uint16_t* act;
    uint32_t* execs;
    uint64_t* stamps;
    const uint16_t* residual;
    uint16_t* hidden_out;
    float* y32;
    const uint16_t* norm_w;
    float* importance;        // optional fp32 [N] per-destination sum of |h|
    uint32_t* imp_flag;       // optional: epoch released once `importance` is written
    uint32_t epoch, mode, flags, layer, core_count;
    uint32_t pad[3];
};

// Workspace words (device memory, zero at rest; the last CTA of every
// launch restores the words it used).
// kWsPollClock: %globaltimer (low 32 bits) of the last host-queue poll;
// kWsPollLock: 1 while one thread of the grid reads a host-memory queue.
constexpr uint32_t kWsExit = 0, kWsErr = 1, kWsDetail = 2, kWsTag = 3, kWsPollClock = 4, kWsPollLock = 5,
                   kWsHeader = 8;
// path, slab claim, (unused), reduced column blocks, (unused),
// and for a host-memory queue:
// queue positions mirrored into device memory, queue state (1 activated,
// 2 failed), total_count at activation
constexpr uint32_t kWsPerLayer = 8;
// LayerPlan::flags bit set by the host when the queue's control words are in
// host memory (polled under the grid-wide lease); the public flags use the
// low bits.
constexpr uint32_t kPlanHostQueue = 1u << 31;
// Copies of the tagged layer hand-off (xbuf): CTA b polls copy b % 4, so 148
// CTAs spread their polling over four sets of L2 lines.
constexpr uint32_t kXbufReplicas = 4;
// Scratch tags: tag = 1 + base + l for launch-local layer l, where base is a
// device counter (ws[kWsTag]) advanced by the layers of every launch at its
// end, so CUDA-graph replays get fresh tags too. It wraps below kTagWrap;
// the host clears the tagged scratch when its own count of issued layers
// crosses a wrap (launches it did not issue, such as graph replays, are not
// counted). Tag 0 never occurs: zeroed scratch holds no current word.
constexpr uint32_t kTagWrap = 0xFFFF0000u;
__host__ __device__ inline uint32_t ws_words(uint32_t max_layers) { return kWsHeader + kWsPerLayer * max_layers; }

// Slabs per group and partial rows of the scratch buffer.
__host__ __device__ inline uint32_t slabs_per_group(uint32_t G) { return (G + kSlab - 1) / kSlab; }

// Everything one launch needs, passed by value.
struct KernelParams {
    uint32_t H, G, N;
    uint32_t cache_slots, staging_slots, phys_groups;  // 0 = unchecked
    uint64_t group_bytes;
    uint64_t timeout_ns;
    float eps;
    uint32_t nlayers;     // layers executed by this launch
    uint32_t max_layers;  // workspace capacity
    uint32_t variant;     // 1: scales applied per 128-block after the tensor-core sums; 0: fp16(q*s) weights
    unsigned long long* partial;  // [N * slabs_per_group(G)][H] tagged fp32 slab partial rows
    unsigned long long* xbuf;     // [kXbufReplicas][H/2] tagged fp16 pairs: a layer's hidden_out for the next layer
    uint32_t* ws;         // workspace words
    uint32_t* status;     // mapped host words (LS_B200_STATUS_*)
    uint32_t* done;       // mapped host per-layer completion epochs
    uint64_t* trace;      // optional phase stamps
    uint4* qmirror;       // [max_layers][N][2]: device copy of a host queue's core + published descriptors
    unsigned long long* impacc;  // [2][N]: exact sums of |h| * 2^24 per destination, by layer parity (zero at rest)
    const LayerPlan* plans;  // device array for nlayers > 1, else nullptr
    LayerPlan first;         // layer 0 when plans == nullptr
    // Tensor parallel inside one launch (world > 1): rank r's exchange buffer
    // [2 slots][world][H] tagged fp32 words, mapped on every rank (xpeer[r]).
    uint32_t world, rank;
    unsigned long long* xpeer[kMaxRanks];
    // 1 when every layer of the launch is BatchCompat / Auto on a
    // device-memory queue and world == 1 (lean_plans): the kernel instance
    // without the progressive, host-queue and tensor-parallel paths runs.
    uint32_t lean;
};

// Whether a launch's plans allow the lean kernel instance.
inline bool lean_plans(const LayerPlan* plans, uint32_t count, uint32_t world) {
    if (world != 1) return false;
    for (uint32_t i = 0; i < count; ++i)
        if (plans[i].mode == LS_MODE_PROGRESSIVE || (plans[i].flags & kPlanHostQueue)) return false;
    return true;
}

// Host-side launchers implemented in ls_kernel.cu.
int launch_fused(const KernelParams& p, int grid, cudaStream_t stream);
int launch_fused_traced(const KernelParams& p, int grid, cudaStream_t stream);  // p.trace set
int prepare_kernels_traced();
int prepare_kernels();  // raise the dynamic shared-memory limit once

}  // namespace lsb
