// Internal types shared by the host backend (ls_backend.cu) and the fused
// layer kernel (ls_kernel.cu). Not part of the public ABI.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>
#include "../../include/leanstream_b200.h"

namespace lsb {

// CTA shape: sixteen consumer warps plus one TMA producer warp. Warps w and
// w + 8 share hidden slice w % 8 (gate/up) and split the rows of a DOWN piece.
constexpr int kConsumerWarps = 16;
constexpr int kSlices = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;

// Shared-memory ring: each stage holds up to 33 KB of packed INT4 rows and a
// 3 KB auxiliary area (fp16 scales, staged h values, cross-warp partials).
// Six stages keep ~200 KB of HBM reads in flight per SM -- more than one
// layer's per-SM share at config 2/3 -- so the producer can run a full
// layer ahead of the consumers.
constexpr int kStages = 6;
constexpr int kStageData = 33024;  // 8 rows of H = 4096 at a pitch of H + 16, plus slack
constexpr int kStageAux = 36864 - kStageData;
constexpr int kStageBytes = kStageData + kStageAux;
constexpr int kAuxSecond = 1280;   // aux offset of DOWN h values / GATEUP partials
constexpr int kGateupMax = 16;     // neurons per GATEUP piece
constexpr int kMaxGroupSize = 256;
constexpr int kMaxHidden = 4096;  // register-resident activation limit (4 chunks per lane)

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
    uint32_t epoch, mode, flags, layer, core_count;
    uint32_t pad[3];
};

// Workspace words (device memory, zero at rest; the last CTA of every
// launch restores the words it used).
constexpr uint32_t kWsExit = 0, kWsErr = 1, kWsDetail = 2, kWsHeader = 8;
constexpr uint32_t kWsPerLayer = 4;  // path, claim, partials-done CTAs, reduced column blocks
__host__ __device__ inline uint32_t ws_words(uint32_t max_layers, uint32_t) {
    return kWsHeader + kWsPerLayer * max_layers;
}

// Everything one launch needs, passed by value.
struct KernelParams {
    uint32_t H, G, N;
    uint32_t cache_slots, staging_slots, phys_groups;  // 0 = unchecked
    uint64_t group_bytes;
    uint64_t timeout_ns;
    float eps;
    uint32_t nlayers;     // layers executed by this launch
    uint32_t max_layers;  // workspace capacity
    uint32_t seq;         // launch sequence number (status word, h tags)
    uint32_t variant;     // 0: CUDA-core FMA gate/up, 1: tensor-core (mma.sync) gate/up
    float* partial;       // [2N][H] fp32, two rows (row halves) per descriptor position
    unsigned long long* hbuf;  // [N][G] tagged h words: (tag << 32) | fp16 h
    uint32_t* ws;         // workspace words
    uint32_t* status;     // mapped host words (LS_B200_STATUS_*)
    uint32_t* done;       // mapped host per-layer completion epochs
    uint64_t* trace;      // optional [grid][LS_B200_TRACE_WORDS]
    const LayerPlan* plans;  // device array for nlayers > 1, else nullptr
    LayerPlan first;         // layer 0 when plans == nullptr
};

// Host-side launchers implemented in ls_kernel.cu.
int launch_fused(const KernelParams& p, int grid, cudaStream_t stream);
int prepare_kernels();  // raise the dynamic shared-memory limit once
size_t kernel_smem_bytes();

}  // namespace lsb
