// Internal types shared by the host backend (ls_backend.cu) and the fused
// layer kernel (ls_kernel.cu). Not part of the public ABI.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>
#include "../../include/leanstream_b200.h"

namespace lsb {

// CTA shape: eight consumer warps plus one TMA producer warp.
constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;

// Shared-memory ring: each stage holds up to 32 KB of packed INT4 rows and
// up to 4 KB of fp16 scales. Six stages keep ~190 KB of HBM reads in flight
// per SM, enough to cover DRAM latency at the per-SM share of HBM bandwidth.
constexpr int kStages = 6;
constexpr int kStageData = 32 * 1024;
constexpr int kStageScale = 4 * 1024;
constexpr int kStageBytes = kStageData + kStageScale;
constexpr int kMaxGroupSize = 256;
constexpr int kMaxHidden = 4096;  // register-resident activation limit (MAXC <= 4)

// Device workspace. Zero at rest: the last CTA of every launch restores it.
struct Workspace {
    uint32_t path;    // 0 undecided, 1 all-ready fast path, 2 progressive claims, 3 abort
    uint32_t total;   // QueueControl.total_count of this launch
    uint32_t claim;   // next claim position (core descriptors first)
    uint32_t arrive;  // grid barrier before the reduction
    uint32_t exit;    // CTAs that finished
    uint32_t err;     // first LS_B200_DEV_* error of this launch
    uint32_t detail;  // index involved in that error
    uint32_t pad[25];
    // followed by done_h[group_count]: neurons of each partial row whose h is published
};
constexpr uint32_t kPathFast = 1, kPathProgressive = 2, kPathAbort = 3;

// Everything one launch needs, passed by value.
struct KernelParams {
    uint32_t H, G, N;
    uint32_t cache_slots, staging_slots, phys_groups;  // 0 = unchecked
    uint64_t group_bytes;
    uint64_t timeout_ns;
    float eps;
    uint32_t epoch, mode, flags, layer, core_count;
    const uint16_t* x;
    uint16_t* y;
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
    uint64_t* trace;    // optional [grid][LS_B200_TRACE_WORDS]
    // backend scratch
    float* partial;     // [N][H] fp32, one row per descriptor position
    uint16_t* hbuf;     // [N][G] fp16 h, indexed like partial rows
    Workspace* ws;      // device workspace (+ done_h)
    uint32_t* status;   // mapped host words (LS_B200_STATUS_*)
    uint32_t* done;     // mapped host per-layer completion epochs
};

// Host-side launcher implemented in ls_kernel.cu.
int launch_fused_layer(const KernelParams& p, int grid, cudaStream_t stream);
int prepare_kernels();  // raise the dynamic shared-memory limit once
size_t kernel_smem_bytes();

}  // namespace lsb
