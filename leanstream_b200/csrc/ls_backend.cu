// Host side of the B200 compute backend: backend object, kernel selector,
// ExecutionQueue producer and the extern "C" ABI of include/leanstream_b200.h.
//
// Replaces backends/triton/enqueue.cpp (TritonBackend, ls_triton_*) and the
// launch wrapper of kernels/streaming_mlp.cu:85-93 /
// streaming_mlp_candidates.cu:3-11. The runtime above the boundary
// (Runtime / LayerStep / WeightManager) is not touched: it reaches this
// backend through ls_b200_view, which fills a ComputeBackend
// (include/leanstream/runtime.h:10-22).
#include <atomic>
#include <cerrno>
#include <cstddef>
#include <cstring>
#include <limits>
#include <mutex>
#include <new>
#include <cuda_runtime.h>
#include "ls_internal.h"

// ---------------------------------------------------------------- layout checks
static_assert(sizeof(ls_exec_desc) == 20, "ExecDesc is five uint32 (types.h:16-20)");
static_assert(sizeof(ls_queue_control) == 128, "QueueControl is 128 bytes (execution_queue.h:12)");
static_assert(offsetof(ls_queue_control, epoch) == 12, "execution_queue.h:10");
static_assert(offsetof(ls_queue_control, error) == 20, "QueueControl.error at word 5");
static_assert(offsetof(ls_queue_control, claim_count) == 64, "execution_queue.h:11");
static_assert(sizeof(ls_device_exec_queue) == 32, "DeviceExecQueue: three pointers + capacity");
static_assert(sizeof(ls_exec_span) == 16, "Span<T>: pointer + size_t");
static_assert(offsetof(ls_compute_backend, cancel) == 5 * sizeof(void*), "ComputeBackend layout");

namespace lsb {
namespace {

// ---------------------------------------------------------------- catalog
// Candidate ids 0..3 keep the production Triton geometry of
// include/leanstream/triton_backend.h:5-8 (4/8/16/32 persistent CTAs), so an
// offline LUT written for it keeps its meaning. Id 4 is the B200 entry: one
// persistent CTA per SM (resolved at configure), the fallback. entry_point
// selects the arithmetic variant: 1 = fp16 scales applied per 128-block
// around the tensor-core sums, 0 = weights rounded to fp16(q * s) first as
// backends/triton/core.py:17 does (id 5, same grid as id 4).
constexpr ls_kernel_candidate kCatalog[] = {
    {0, 4, "b200_ctas_4", 4, 0, 0, 0, 1, true},
    {1, 8, "b200_ctas_8", 8, 0, 0, 0, 1, true},
    {2, 16, "b200_ctas_16", 16, 0, 0, 0, 1, true},
    {3, 32, "b200_ctas_32", 32, 0, 0, 0, 1, true},
    {4, 0, "b200_ctas_per_sm", 0, 0, 0, 0, 1, true},
    {5, 0, "b200_ctas_per_sm_exact", 0, 0, 0, 0, 0, true},
};
constexpr uint32_t kCatalogSize = sizeof(kCatalog) / sizeof(kCatalog[0]);
constexpr uint32_t kDefaultCandidate = 4;

uint32_t quantize_io_load(uint32_t remaining, uint32_t total, uint32_t buckets) {
    // kernel_selector.cpp:4-8: floor(min(remaining,total)*buckets/total), clamped.
    if (!total || !buckets) return 0;
    if (remaining >= total) return buckets - 1;
    return uint32_t(uint64_t(remaining) * buckets / total);
}

struct Backend {
    // selector state (kernel_selector.h:27-41)
    const uint8_t* lut = nullptr;
    uint32_t lut_layers = 0, lut_buckets = 0;
    uint32_t state_layer = 0, state_bucket = 0;
    // configuration
    bool configured = false;
    int device = -1, sms = 0;
    ls_b200_geometry geo{};
    ls_b200_layer_args bound{};
    bool bound_set = false;
    // scratch (device) and mapped words (host)
    unsigned long long* partial = nullptr;  // tagged slab partial rows
    unsigned long long* xbuf = nullptr;     // tagged layer output handed to the next layer
    uint4* qmirror = nullptr;               // device copy of host-memory queues' descriptors
    unsigned long long* impacc = nullptr;   // importance sums [2][N] (zero at rest)
    size_t partial_bytes = 0, xbuf_bytes = 0;
    uint32_t* ws = nullptr;
    uint64_t layers_issued = 0;  // layers of the launches issued through this backend
    mutable const void* last_control = nullptr;  // host_memory() cache
    mutable bool last_control_host = false;
    bool clear_tags = false;     // the tag counter wrapped: clear the tagged scratch first
    uint32_t* status_host = nullptr;
    uint32_t* status_dev = nullptr;
    uint32_t* done_host = nullptr;
    uint32_t* done_dev = nullptr;
    uint32_t* last_epoch = nullptr;  // host: epoch of the last enqueue per layer
    uint64_t scratch_bytes = 0;
    // tensor parallel inside one launch (ls_b200_tp_setup / ls_b200_tp_connect)
    uint32_t tp_world = 1, tp_rank = 0;
    bool tp_connected = false;
    unsigned long long* exch = nullptr;  // this rank's exchange buffer [2][world][H]
    size_t exch_bytes = 0;
    unsigned long long* peers[kMaxRanks] = {};
    bool opened[kMaxRanks] = {};

    ls_kernel_candidate candidate(uint32_t id) const {
        // kernel_selector.cpp:9-16: invalid/unavailable ids fall back.
        ls_kernel_candidate c = id < kCatalogSize ? kCatalog[id] : kCatalog[kDefaultCandidate];
        if (c.id != id || !c.available) c = kCatalog[kDefaultCandidate];
        if (c.cta_count == 0) {
            c.cta_count = uint32_t(sms > 0 ? sms : 148);
            c.workers = c.cta_count;
        }
        return c;
    }
    uint32_t select(uint32_t layer, uint32_t bucket) const {
        // kernel_selector.cpp:17-22: direct row-major indexing, O(1), no allocation.
        if (!lut || layer >= lut_layers || bucket >= lut_buckets ||
            (lut_buckets && size_t(lut_layers) > std::numeric_limits<size_t>::max() / lut_buckets))
            return kDefaultCandidate;
        const uint32_t id = lut[size_t(layer) * lut_buckets + bucket];
        return candidate(id).id;
    }
    void release_tp() {
        for (uint32_t r = 0; r < uint32_t(kMaxRanks); ++r) {
            if (opened[r]) cudaIpcCloseMemHandle(peers[r]);
            opened[r] = false;
            peers[r] = nullptr;
        }
        if (exch) cudaFree(exch);
        exch = nullptr;
        exch_bytes = 0;
        tp_world = 1;
        tp_rank = 0;
        tp_connected = false;
    }
    void release() {
        release_tp();
        if (partial) cudaFree(partial);
        if (xbuf) cudaFree(xbuf);
        if (qmirror) cudaFree(qmirror);
        qmirror = nullptr;
        if (impacc) cudaFree(impacc);
        impacc = nullptr;
        if (ws) cudaFree(ws);
        if (status_host) cudaFreeHost(status_host);
        if (done_host) cudaFreeHost(done_host);
        delete[] last_epoch;
        partial = nullptr;
        xbuf = nullptr;
        ws = nullptr;
        status_host = status_dev = nullptr;
        done_host = done_dev = nullptr;
        last_epoch = nullptr;
        configured = false;
    }
    ~Backend() { release(); }
};

int cuda_rc(cudaError_t e) { return e == cudaSuccess ? 0 : (int(e) > 0 ? int(e) : EIO); }

int configure(Backend& b, const ls_b200_geometry& g) {
    if (b.configured) return EBUSY;
    const uint32_t H = g.hidden, G = g.group_size, N = g.group_count;
    // H = 256 * {1, 2, 4, 8, 16, 32}: the kernel is instantiated per hidden size
    const uint32_t sb = H / 256;
    if (!H || H % 256 || (sb & (sb - 1)) || H > uint32_t(kMaxHidden) || !G || G > uint32_t(kMaxGroupSize) || !N)
        return EINVAL;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ENODEV;
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return ENODEV;
    if (prop.major != 10) return ENOTSUP;  // sm_100a image only
    int rc = prepare_kernels();
    if (rc) return cuda_rc(cudaError_t(rc));
    b.device = dev;
    b.sms = prop.multiProcessorCount;
    b.geo = g;
    if (!b.geo.max_layers) b.geo.max_layers = 256;
    if (!b.geo.timeout_us) b.geo.timeout_us = 5000000;
    // one tagged fp32 partial output row per slab of every descriptor row,
    // and one tagged fp16 pair per two hidden coordinates; tag 0 never occurs
    const size_t partial_bytes = size_t(N) * slabs_per_group(G) * H * sizeof(unsigned long long);
    const size_t xbuf_bytes = size_t(kXbufReplicas) * (H / 2) * sizeof(unsigned long long);
    const size_t ws_bytes = size_t(ws_words(b.geo.max_layers)) * sizeof(uint32_t);
    // device copy of a host-memory queue's descriptors, per layer (32 B each)
    const size_t qmirror_bytes = size_t(b.geo.max_layers) * N * 2 * sizeof(uint4);
    cudaError_t e = cudaMalloc(&b.partial, partial_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&b.xbuf, xbuf_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&b.qmirror, qmirror_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&b.ws, ws_bytes);
    if (e == cudaSuccess) e = cudaMemset(b.ws, 0, ws_bytes);
    const size_t impacc_bytes = size_t(2) * N * sizeof(unsigned long long);
    if (e == cudaSuccess) e = cudaMalloc(&b.impacc, impacc_bytes);
    if (e == cudaSuccess) e = cudaMemset(b.impacc, 0, impacc_bytes);
    if (e == cudaSuccess) e = cudaMemset(b.partial, 0, partial_bytes);
    if (e == cudaSuccess) e = cudaMemset(b.xbuf, 0, xbuf_bytes);
    b.partial_bytes = partial_bytes;
    b.xbuf_bytes = xbuf_bytes;
    if (e == cudaSuccess) e = cudaHostAlloc(&b.status_host, 64, cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&b.status_dev), b.status_host, 0);
    if (e == cudaSuccess)
        e = cudaHostAlloc(&b.done_host, size_t(b.geo.max_layers) * sizeof(uint32_t), cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&b.done_dev), b.done_host, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        b.release();
        return cuda_rc(e);
    }
    std::memset(b.status_host, 0, 64);
    std::memset(b.done_host, 0, size_t(b.geo.max_layers) * sizeof(uint32_t));
    b.last_epoch = new (std::nothrow) uint32_t[b.geo.max_layers]();
    if (!b.last_epoch) {
        b.release();
        return ENOMEM;
    }
    b.scratch_bytes = partial_bytes + xbuf_bytes + ws_bytes + qmirror_bytes + impacc_bytes;
    b.configured = true;
    return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether the queue's control words are host memory (mapped pinned or
// registered): the kernel then polls them under a grid-wide lease. One
// pointer query per new control address (cached).
bool host_memory(const Backend& b, const void* control) {
    if (control != b.last_control) {
        cudaPointerAttributes at{};
        const cudaError_t e = cudaPointerGetAttributes(&at, control);
        if (e != cudaSuccess) cudaGetLastError();  // not a CUDA pointer: plain host memory
        b.last_control_host = e != cudaSuccess || at.type != cudaMemoryTypeDevice;
        b.last_control = control;
    }
    return b.last_control_host;
}

// Validates one layer's arguments and encodes its plan. Host only, no
// device work (one cached pointer query).
int encode(const Backend& b, const ls_b200_layer_args& a, LayerPlan* out) {
    if (!b.configured) return EINVAL;
    if (!a.epoch || !a.input || !a.scales || !a.queue.control || !a.queue.descriptors || !a.queue.ready_indices)
        return EINVAL;
    if (!a.cache && !a.staging) return EINVAL;
    if (a.core_count && !a.core) return EINVAL;
    if (!a.output && !a.output_f32 && !a.hidden_out) return EINVAL;
    if (a.hidden_out && !a.residual) return EINVAL;
    if (a.mode > LS_MODE_AUTO) return EINVAL;
    if (a.layer >= b.geo.max_layers) return EINVAL;
    if (a.core_count > b.geo.group_count) return ENOSPC;
    // cp.async.bulk sources and the 16-byte activation loads need alignment
    if ((a.cache && !aligned16(a.cache)) || (a.staging && !aligned16(a.staging)) || !aligned16(a.scales) ||
        !aligned16(a.input) || (a.norm_weight && !aligned16(a.norm_weight)) ||
        (a.output_f32 && !aligned16(a.output_f32)))
        return EINVAL;
    LayerPlan p{};
    p.x = static_cast<const uint16_t*>(a.input);
    p.y = static_cast<uint16_t*>(a.output);
    p.cache = a.cache ? a.cache : a.staging;
    p.staging = a.staging ? a.staging : a.cache;
    p.scales = static_cast<const uint16_t*>(a.scales);
    p.core = a.core;
    p.q = a.queue;
    p.act = static_cast<uint16_t*>(a.activations);
    p.execs = a.executions;
    p.stamps = a.first_compute;
    p.residual = static_cast<const uint16_t*>(a.residual);
    p.hidden_out = static_cast<uint16_t*>(a.hidden_out);
    p.y32 = a.output_f32;
    p.norm_w = static_cast<const uint16_t*>(a.norm_weight);
    p.importance = a.importance;
    p.imp_flag = a.importance_flag;
    p.epoch = a.epoch;
    p.mode = a.mode;
    p.flags = (a.flags & ~kPlanHostQueue) | (host_memory(b, a.queue.control) ? kPlanHostQueue : 0u);
    p.layer = a.layer;
    p.core_count = a.core_count;
    *out = p;
    return 0;
}

KernelParams base_params(Backend& b, uint32_t nlayers, uint64_t* trace, cudaStream_t stream) {
    KernelParams p{};
    p.H = b.geo.hidden;
    p.G = b.geo.group_size;
    p.N = b.geo.group_count;
    p.cache_slots = b.geo.cache_slots;
    p.staging_slots = b.geo.staging_slots;
    p.phys_groups = b.geo.physical_groups;
    p.group_bytes = uint64_t(p.G) * 3 * p.H / 2;
    p.timeout_ns = uint64_t(b.geo.timeout_us) * 1000ull;
    p.eps = b.geo.rms_eps;
    p.nlayers = nlayers;
    p.max_layers = b.geo.max_layers;
    // The device tag counter advances by nlayers per launch and wraps below
    // kTagWrap. After a launch that crossed a wrap, the scratch is cleared on
    // the stream (no allocation) so that no word of the previous cycle can
    // carry a current tag.
    if (b.clear_tags) {
        cudaMemsetAsync(b.partial, 0, b.partial_bytes, stream);
        cudaMemsetAsync(b.xbuf, 0, b.xbuf_bytes, stream);
        b.clear_tags = false;
    }
    const uint64_t before = b.layers_issued;
    b.layers_issued += nlayers;
    if (before / kTagWrap != b.layers_issued / kTagWrap) b.clear_tags = true;
    p.partial = b.partial;
    p.xbuf = b.xbuf;
    p.qmirror = b.qmirror;
    p.impacc = b.impacc;
    p.ws = b.ws;
    p.status = b.status_dev;
    p.done = b.done_dev;
    p.trace = trace;
    p.world = b.tp_connected ? b.tp_world : 1u;
    p.rank = b.tp_connected ? b.tp_rank : 0u;
    for (uint32_t r = 0; r < p.world; ++r) p.xpeer[r] = b.peers[r];
    return p;
}

// A tensor-parallel launch forms each layer's outputs and the next input from
// the layer input (the residual) and the ranks' partials: consecutive layers
// must chain (next input = hidden_out) and a hidden_out's residual must be
// its layer's input.
bool tp_plans_ok(const LayerPlan* hp, uint32_t count) {
    for (uint32_t i = 0; i < count; ++i) {
        if (hp[i].hidden_out && hp[i].residual != hp[i].x) return false;
        if (i + 1 < count && (!hp[i].hidden_out || hp[i + 1].x != hp[i].hidden_out)) return false;
    }
    return true;
}

int grid_for(const Backend& b, int32_t candidate, uint32_t* variant) {
    const uint32_t id = candidate >= 0 ? uint32_t(candidate) : b.select(b.state_layer, b.state_bucket);
    const ls_kernel_candidate c = b.candidate(id);
    // variant 0 is built up to one piece's hidden extent; above it the
    // candidate's grid runs variant 1
    *variant = b.geo.hidden > uint32_t(kMaxPieceHidden) ? 1u : c.entry_point;
    int grid = int(c.cta_count);
    return grid > b.sms ? b.sms : grid;
}

// Hot path: parameter validation and one kernel launch. No allocation,
// no synchronisation, no device queries (triton_cuda.h:19-20).
int launch(Backend& b, const ls_b200_layer_args& a, cudaStream_t stream) {
    LayerPlan plan;
    int rc = encode(b, a, &plan);
    if (rc) return rc;
    if (b.tp_connected && !tp_plans_ok(&plan, 1)) return EINVAL;
    KernelParams p = base_params(b, 1, a.trace, stream);
    p.plans = nullptr;
    p.first = plan;
    p.lean = lean_plans(&plan, 1, p.world) ? 1u : 0u;
    b.last_epoch[a.layer] = a.epoch;
    const int grid = grid_for(b, a.candidate, &p.variant);
    rc = launch_fused(p, grid, stream);
    return rc ? cuda_rc(cudaError_t(rc)) : 0;
}

// ---------------------------------------------------------------- ComputeBackend
// Tensor parallel inside one launch. Setup allocates and zeroes this rank's
// exchange buffer ([2 slots][world][H] tagged fp32 words) and exports it as
// a CUDA IPC handle; connect maps every peer's buffer (NVLink peer memory),
// resets the tag counter and clears the tagged scratch, so that all ranks
// start from the same tags. From then on every launch through this backend
// is a collective of the `world` ranks: they must issue the same launches
// (same layers, in the same order), as for an allreduce.
int tp_setup(Backend& b, uint32_t rank, uint32_t world, void* handle_out) {
    if (!b.configured || world < 2 || world > uint32_t(kMaxRanks) || rank >= world) return EINVAL;
    b.release_tp();
    const size_t bytes = size_t(2) * world * b.geo.hidden * sizeof(unsigned long long);
    cudaError_t e = cudaMalloc(&b.exch, bytes);
    if (e == cudaSuccess) e = cudaMemset(b.exch, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, b.exch);
    if (e != cudaSuccess) {
        b.release_tp();
        return cuda_rc(e);
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == LS_B200_TP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    b.exch_bytes = bytes;
    b.tp_world = world;
    b.tp_rank = rank;
    return 0;
}

int tp_connect(Backend& b, const void* handles) {
    if (!b.exch || b.tp_connected) return EINVAL;
    const auto* hs = static_cast<const uint8_t*>(handles);
    cudaError_t e = cudaSuccess;
    for (uint32_t r = 0; r < b.tp_world && e == cudaSuccess; ++r) {
        if (r == b.tp_rank) {
            b.peers[r] = b.exch;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + size_t(r) * LS_B200_TP_HANDLE_BYTES, sizeof(h));
        void* ptr = nullptr;
        e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e == cudaSuccess) {
            b.peers[r] = static_cast<unsigned long long*>(ptr);
            b.opened[r] = true;
        }
    }
    // same starting tags on every rank
    if (e == cudaSuccess) e = cudaMemset(b.ws, 0, size_t(ws_words(b.geo.max_layers)) * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(b.partial, 0, b.partial_bytes);
    if (e == cudaSuccess) e = cudaMemset(b.xbuf, 0, b.xbuf_bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        b.release_tp();
        return cuda_rc(e);
    }
    b.layers_issued = 0;
    b.clear_tags = false;
    b.tp_connected = true;
    return 0;
}

int view_enqueue(void* ctx, uint32_t layer, const void* input, void* output, void* stream, ls_exec_span core,
                 ls_device_exec_queue queue, uint32_t epoch, uint8_t mode) {
    // TritonBackend::submit (enqueue.cpp:38-43), all three modes accepted.
    auto* b = static_cast<Backend*>(ctx);
    if (!b || !b->bound_set) return EINVAL;
    if (core.size > std::numeric_limits<uint32_t>::max()) return EINVAL;
    ls_b200_layer_args a = b->bound;
    a.input = input;
    a.output = output;
    a.core = core.data;
    a.core_count = uint32_t(core.size);
    a.queue = queue;
    a.epoch = epoch;
    a.mode = mode;
    a.layer = layer;
    a.candidate = -1;
    b->state_layer = layer;
    return launch(*b, a, static_cast<cudaStream_t>(stream));
}

bool view_complete(void* ctx, uint32_t layer) {
    auto* b = static_cast<Backend*>(ctx);
    if (!b || !b->configured || layer >= b->geo.max_layers) return false;
    const uint32_t want = b->last_epoch[layer];
    if (!want) return true;
    return __atomic_load_n(b->done_host + layer, __ATOMIC_ACQUIRE) == want;
}

int view_commit(void*, uint32_t, ls_group_span ids) {
    // Cache installation is application policy (enqueue.cpp:45); this backend
    // keeps no cache of its own, so committing a resident set is a no-op.
    return (ids.size && !ids.data) ? EINVAL : 0;
}

void view_cancel(void*, uint32_t, uint32_t) {
    // The Runtime publishes QueueControl.error before calling cancel
    // (runtime.cpp:41,49,93); the kernel observes it and exits.
}

}  // namespace

// ------------------------------------------------------------ static-scratch launch
// ls_b200_launch_static is for callers that must not allocate device memory
// on their launch path: an engine that has already given all of HBM to its
// own pool (a cudaMalloc would fail, or take pages that pool counts on), a
// layer driven from inside a region where an allocation would synchronise
// the device and stall the pipeline, or a host that cannot own the lifetime
// of a backend object. Such a caller gets the same kernel with its scratch
// fixed at compile time in the arrays below, whose device addresses are
// looked up once per device.
//
// Limits: the partial rows (group_count * ceil(G/16) * hidden tagged words)
// must fit kStaticPartialWords (32 MiB; H 4096 with G 64 allows 256 groups),
// and args.layer must be below kStaticLayers. One scratch set per device:
// two calls whose launches overlap in time on one device race on it.
constexpr size_t kStaticPartialWords = size_t(1) << 22;
constexpr uint32_t kStaticLayers = 256;
constexpr uint32_t kStaticWsWords = 64;
constexpr int kStaticDevices = 64;
static_assert(kWsHeader + kWsPerLayer <= kStaticWsWords, "workspace of a one-layer launch");

static __device__ __align__(256) unsigned long long g_static_partial[kStaticPartialWords];
static __device__ __align__(256) unsigned long long g_static_xbuf[kXbufReplicas * (kMaxHidden / 2)];
static __device__ __align__(256) uint32_t g_static_ws[kStaticWsWords];
static __device__ __align__(256) uint32_t g_static_status[LS_B200_STATUS_WORDS];
static __device__ __align__(256) uint32_t g_static_done[kStaticLayers];
// device copy of a host-memory queue: N <= kStaticPartialWords / 256 groups
// (H >= 256, one slab per group at least)
constexpr size_t kStaticMirror = kStaticPartialWords / 256;
static __device__ __align__(256) uint4 g_static_qmirror[kStaticMirror * 2];
// importance sums [2][N] (N <= kStaticMirror)
static __device__ __align__(256) unsigned long long g_static_impacc[kStaticMirror * 2];

namespace {

struct StaticScratch {
    std::atomic<bool> ready{false};
    int sms = 0;
    unsigned long long* partial = nullptr;
    unsigned long long* xbuf = nullptr;
    uint32_t* ws = nullptr;
    uint32_t* status = nullptr;
    uint32_t* done = nullptr;
    uint4* qmirror = nullptr;
    unsigned long long* impacc = nullptr;
    // Layers launched on this device by successful calls, and whether the
    // tag counter wrapped (the next call clears the tagged scratch first).
    // Atomic: calls may come from several host threads (their launches must
    // still be ordered on the GPU).
    std::atomic<uint64_t> layers_issued{0};
    std::atomic<bool> clear_tags{false};
};
StaticScratch g_static[kStaticDevices];
std::mutex g_static_setup;

template <typename T>
int symbol_address(T** out, const void* symbol) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, symbol);
    if (e != cudaSuccess) return cuda_rc(e);
    if (!p) return EIO;
    *out = static_cast<T*>(p);
    return 0;
}

// First call on a device (that device current): kernel attributes, symbol
// addresses, and zeroing on `stream` of everything that must start at zero:
// the workspace (exit counter, error word, claims), the tagged scratch (a
// zero word carries no tag any launch issues), status and completion words.
int static_setup(StaticScratch& s, int dev, cudaStream_t stream) {
    std::lock_guard<std::mutex> lock(g_static_setup);
    if (s.ready.load(std::memory_order_acquire)) return 0;
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return ENODEV;
    if (major != 10) return ENOTSUP;
    int rc = prepare_kernels();
    if (rc) return cuda_rc(cudaError_t(rc));
    if ((rc = symbol_address(&s.partial, g_static_partial)) || (rc = symbol_address(&s.xbuf, g_static_xbuf)) ||
        (rc = symbol_address(&s.ws, g_static_ws)) || (rc = symbol_address(&s.status, g_static_status)) ||
        (rc = symbol_address(&s.done, g_static_done)) || (rc = symbol_address(&s.qmirror, g_static_qmirror)) ||
        (rc = symbol_address(&s.impacc, g_static_impacc)))
        return rc;
    cudaError_t e = cudaMemsetAsync(s.partial, 0, sizeof(g_static_partial), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(s.xbuf, 0, sizeof(g_static_xbuf), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(s.ws, 0, sizeof(g_static_ws), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(s.status, 0, sizeof(g_static_status), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(s.done, 0, sizeof(g_static_done), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(s.impacc, 0, sizeof(g_static_impacc), stream);
    if (e != cudaSuccess) return cuda_rc(e);
    s.sms = sms;
    s.ready.store(true, std::memory_order_release);
    return 0;
}

int launch_static(const ls_b200_geometry& g, const ls_b200_layer_args& a, uint32_t* status,
                  cudaStream_t stream) {
    // Host-only checks first: nothing below runs for a rejected call.
    const uint32_t H = g.hidden, G = g.group_size, N = g.group_count;
    const uint32_t sb = H / 256;
    if (!H || H % 256 || (sb & (sb - 1)) || H > uint32_t(kMaxHidden) || !G || G > uint32_t(kMaxGroupSize) || !N)
        return EINVAL;
    if (size_t(N) * slabs_per_group(G) * H > kStaticPartialWords || a.layer >= kStaticLayers) return E2BIG;
    Backend b;  // host view for validation and candidate choice; owns nothing
    b.configured = true;
    b.geo = g;
    b.geo.max_layers = kStaticLayers;
    if (!b.geo.timeout_us) b.geo.timeout_us = 5000000;
    LayerPlan plan;
    int rc = encode(b, a, &plan);
    if (rc) return rc;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kStaticDevices) return ENODEV;
    StaticScratch& s = g_static[dev];
    if (!s.ready.load(std::memory_order_acquire) && (rc = static_setup(s, dev, stream))) return rc;
    b.sms = s.sms;

    KernelParams p{};
    p.H = H;
    p.G = G;
    p.N = N;
    p.cache_slots = g.cache_slots;
    p.staging_slots = g.staging_slots;
    p.phys_groups = g.physical_groups;
    p.group_bytes = uint64_t(G) * 3 * H / 2;
    p.timeout_ns = uint64_t(b.geo.timeout_us) * 1000ull;
    p.eps = g.rms_eps;
    p.nlayers = 1;
    p.max_layers = kStaticLayers;
    p.world = 1;  // one GPU: no exchange
    if (s.clear_tags.exchange(false)) {  // the tag counter wrapped: clear the tagged scratch on the stream
        cudaError_t e = cudaMemsetAsync(s.partial, 0, sizeof(g_static_partial), stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(s.xbuf, 0, sizeof(g_static_xbuf), stream);
        if (e != cudaSuccess) {
            s.clear_tags.store(true);
            return cuda_rc(e);
        }
    }
    p.partial = s.partial;
    p.xbuf = s.xbuf;
    p.qmirror = s.qmirror;
    p.impacc = s.impacc;
    p.ws = s.ws;
    p.status = status ? status : s.status;
    p.done = s.done;
    p.trace = a.trace;
    p.plans = nullptr;
    p.first = plan;
    p.lean = lean_plans(&plan, 1, 1) ? 1u : 0u;
    const int grid = grid_for(b, a.candidate, &p.variant);
    rc = launch_fused(p, grid, stream);
    if (rc) return cuda_rc(cudaError_t(rc));
    // the device tag counter advanced by one layer: count it, and clear the
    // tagged scratch before the next call when the counter wrapped
    if ((s.layers_issued.fetch_add(1) + 1) % kTagWrap == 0) s.clear_tags.store(true);
    return 0;
}

// Set-up only (args == NULL): looks up the arrays on the current device and
// zeroes them on `stream`, without launching anything.
int setup_static(cudaStream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kStaticDevices) return ENODEV;
    StaticScratch& s = g_static[dev];
    return s.ready.load(std::memory_order_acquire) ? 0 : static_setup(s, dev, stream);
}

}  // namespace
}  // namespace lsb

using lsb::Backend;

extern "C" {

void* ls_b200_create(void) { return new (std::nothrow) Backend; }

void* ls_b200_create_table(const uint8_t* lut, uint32_t layers, uint32_t buckets) {
    auto* b = new (std::nothrow) Backend;
    if (!b) return nullptr;
    b->lut = lut;
    b->lut_layers = layers;
    b->lut_buckets = buckets;
    return b;
}

void ls_b200_destroy(void* backend) { delete static_cast<Backend*>(backend); }

int ls_b200_configure(void* backend, const ls_b200_geometry* geometry) {
    if (!backend || !geometry) return EINVAL;
    return lsb::configure(*static_cast<Backend*>(backend), *geometry);
}

int ls_b200_set_buffers(void* backend, const ls_b200_layer_args* buffers) {
    if (!backend || !buffers) return EINVAL;
    auto* b = static_cast<Backend*>(backend);
    b->bound = *buffers;
    b->bound_set = true;
    return 0;
}

void ls_b200_set_state(void* backend, uint32_t layer, uint32_t io_bucket) {
    if (!backend) return;
    auto* b = static_cast<Backend*>(backend);
    b->state_layer = layer;
    b->state_bucket = io_bucket;
}

int ls_b200_launch(void* backend, const ls_b200_layer_args* args, void* stream) {
    if (!backend || !args) return EINVAL;
    return lsb::launch(*static_cast<Backend*>(backend), *args, static_cast<cudaStream_t>(stream));
}

int ls_b200_launch_static(const ls_b200_geometry* geometry, const ls_b200_layer_args* args, uint32_t* status,
                          void* stream) {
    if (!args) return lsb::setup_static(static_cast<cudaStream_t>(stream));  // set-up only
    if (!geometry) return EINVAL;
    return lsb::launch_static(*geometry, *args, status, static_cast<cudaStream_t>(stream));
}

int ls_b200_tp_setup(void* backend, uint32_t rank, uint32_t world, void* handle_out) {
    if (!backend || !handle_out) return EINVAL;
    return lsb::tp_setup(*static_cast<Backend*>(backend), rank, world, handle_out);
}

int ls_b200_tp_connect(void* backend, const void* handles) {
    if (!backend || !handles) return EINVAL;
    return lsb::tp_connect(*static_cast<Backend*>(backend), handles);
}

uint32_t ls_b200_plan_size(void) { return uint32_t(sizeof(lsb::LayerPlan)); }

int ls_b200_encode_plan(void* backend, const ls_b200_layer_args* args, void* plan) {
    if (!backend || !args || !plan) return EINVAL;
    auto* b = static_cast<Backend*>(backend);
    lsb::LayerPlan p;
    const int rc = lsb::encode(*b, *args, &p);
    if (rc) return rc;
    std::memcpy(plan, &p, sizeof(p));
    return 0;
}

int ls_b200_launch_plans(void* backend, const void* device_plans, uint32_t count, const void* host_plans,
                         int32_t candidate, uint64_t* trace, void* stream) {
    if (!backend || !device_plans || !host_plans || !count) return EINVAL;
    auto* b = static_cast<Backend*>(backend);
    if (!b->configured || count > b->geo.max_layers) return EINVAL;
    if ((reinterpret_cast<uintptr_t>(device_plans) & 15u) != 0) return EINVAL;
    const auto* hp = static_cast<const lsb::LayerPlan*>(host_plans);
    for (uint32_t i = 0; i < count; ++i)
        if (hp[i].layer >= b->geo.max_layers || !hp[i].epoch) return EINVAL;
    if (b->tp_connected && !lsb::tp_plans_ok(hp, count)) return EINVAL;
    for (uint32_t i = 0; i < count; ++i) b->last_epoch[hp[i].layer] = hp[i].epoch;
    lsb::KernelParams p = lsb::base_params(*b, count, trace, static_cast<cudaStream_t>(stream));
    p.plans = static_cast<const lsb::LayerPlan*>(device_plans);
    p.first = hp[0];
    p.lean = lsb::lean_plans(hp, count, p.world) ? 1u : 0u;
    const int grid = lsb::grid_for(*b, candidate, &p.variant);
    const int rc = lsb::launch_fused(p, grid, static_cast<cudaStream_t>(stream));
    return rc ? lsb::cuda_rc(cudaError_t(rc)) : 0;
}

int ls_b200_enqueue(void* backend, uint32_t layer, uint32_t bucket, uint32_t epoch, void* stream) {
    if (!backend) return EINVAL;
    auto* b = static_cast<Backend*>(backend);
    if (!b->bound_set) return EINVAL;
    ls_b200_layer_args a = b->bound;
    a.epoch = epoch;
    a.layer = layer;
    a.candidate = int32_t(b->select(layer, bucket));
    return lsb::launch(*b, a, static_cast<cudaStream_t>(stream));
}

int ls_b200_view(void* backend, ls_compute_backend* out) {
    if (!backend || !out) return EINVAL;
    out->context = backend;
    out->enqueue = lsb::view_enqueue;
    out->complete = lsb::view_complete;
    out->commit = lsb::view_commit;
    out->defer_commit = nullptr;
    out->cancel = lsb::view_cancel;
    return 0;
}

int ls_b200_completed_epoch(void* backend, uint32_t layer, uint32_t* epoch) {
    if (!backend || !epoch) return EINVAL;
    auto* b = static_cast<Backend*>(backend);
    if (!b->configured || layer >= b->geo.max_layers) return EINVAL;
    *epoch = __atomic_load_n(b->done_host + layer, __ATOMIC_ACQUIRE);
    return 0;
}

int ls_b200_status(void* backend, uint32_t* words, uint32_t count) {
    if (!backend || !words) return EINVAL;
    auto* b = static_cast<Backend*>(backend);
    if (!b->configured) return EINVAL;
    for (uint32_t i = 0; i < count && i < LS_B200_STATUS_WORDS; ++i)
        words[i] = __atomic_load_n(b->status_host + i, __ATOMIC_ACQUIRE);
    return 0;
}

int ls_b200_clear_status(void* backend) {
    if (!backend) return EINVAL;
    auto* b = static_cast<Backend*>(backend);
    if (!b->configured) return EINVAL;
    for (uint32_t i = 0; i < 3; ++i) __atomic_store_n(b->status_host + i, 0u, __ATOMIC_RELEASE);
    return 0;
}

uint64_t ls_b200_scratch_bytes(void* backend) {
    return backend ? static_cast<Backend*>(backend)->scratch_bytes : 0;
}

uint32_t ls_b200_quantize_io_load(uint32_t remaining, uint32_t total, uint32_t buckets) {
    return lsb::quantize_io_load(remaining, total, buckets);
}

uint32_t ls_b200_select(void* backend, uint32_t layer, uint32_t io_bucket) {
    if (!backend) return lsb::kDefaultCandidate;
    return static_cast<Backend*>(backend)->select(layer, io_bucket);
}

int ls_b200_candidate(void* backend, uint32_t id, ls_kernel_candidate* out) {
    if (!out) return EINVAL;
    if (backend) {
        *out = static_cast<Backend*>(backend)->candidate(id);
    } else {
        Backend tmp;
        *out = tmp.candidate(id);
    }
    return 0;
}

uint32_t ls_b200_catalog_size(void) { return lsb::kCatalogSize; }
uint32_t ls_b200_default_candidate(void) { return lsb::kDefaultCandidate; }

// ---------------------------------------------------------------- ExecutionQueue
// Restatement of src/runtime/execution_queue.cpp:4-46 over the C view: the
// same release-store order (ready_count before epoch; batch_epoch when the
// plan is complete) and the same single-shot error CAS. Errors are returned
// instead of asserted.
void ls_b200_queue_bind(ls_b200_queue* q, ls_device_exec_queue view) {
    if (!q) return;
    q->view = view;
    q->tail = q->epoch = q->total = 0;
}

int ls_b200_queue_reset(ls_b200_queue* q, uint32_t epoch) {
    if (!q || !q->view.control || !q->view.descriptors || !q->view.ready_indices || !epoch) return EINVAL;
    ls_queue_control* c = q->view.control;
    q->tail = q->total = 0;
    q->epoch = epoch;
    __atomic_store_n(&c->epoch, 0u, __ATOMIC_RELEASE);
    c->ready_count = 0;
    c->reserved = 0;
    c->claim_count = 0;
    c->total_count = 0;
    c->batch_epoch = 0;
    c->error = 0;
    c->consumer_path = 0;
    c->init_arrived = 0;
    c->init_epoch = 0;
    return 0;
}

int ls_b200_queue_prepare(ls_b200_queue* q, uint32_t total) {
    if (!q || !q->view.control || total > q->view.capacity) return EINVAL;
    q->total = total;
    q->view.control->total_count = total;
    return 0;
}

int ls_b200_queue_append_unpublished(ls_b200_queue* q, uint32_t index) {
    if (!q || q->tail >= q->total || index >= q->total) return EINVAL;
    for (uint32_t i = 0; i < q->tail; ++i)
        if (q->view.ready_indices[i] == index) return EEXIST;
    q->view.ready_indices[q->tail++] = index;
    return 0;
}

int ls_b200_queue_activate(ls_b200_queue* q) {
    if (!q || !q->view.control) return EINVAL;
    ls_queue_control* c = q->view.control;
    __atomic_store_n(&c->ready_count, q->tail, __ATOMIC_RELEASE);
    __atomic_store_n(&c->epoch, q->epoch, __ATOMIC_RELEASE);
    if (q->tail == q->total) __atomic_store_n(&c->batch_epoch, q->epoch, __ATOMIC_RELEASE);
    return 0;
}

int ls_b200_queue_seal(ls_b200_queue* q, uint32_t total) {
    const int rc = ls_b200_queue_prepare(q, total);
    return rc ? rc : ls_b200_queue_activate(q);
}

int ls_b200_queue_publish_all(ls_b200_queue* q) {
    if (!q || !q->view.control || q->tail != 0) return EINVAL;
    for (uint32_t i = 0; i < q->total; ++i) q->view.ready_indices[i] = i;
    q->tail = q->total;
    __atomic_store_n(&q->view.control->ready_count, q->tail, __ATOMIC_RELEASE);
    __atomic_store_n(&q->view.control->batch_epoch, q->epoch, __ATOMIC_RELEASE);
    return 0;
}

int ls_b200_queue_publish(ls_b200_queue* q, uint32_t index) {
    if (!q || !q->view.control || q->tail >= q->total || index >= q->total) return EINVAL;
    for (uint32_t i = 0; i < q->tail; ++i)
        if (q->view.ready_indices[i] == index) return EEXIST;
    q->view.ready_indices[q->tail++] = index;
    __atomic_store_n(&q->view.control->ready_count, q->tail, __ATOMIC_RELEASE);
    if (q->tail == q->total) __atomic_store_n(&q->view.control->batch_epoch, q->epoch, __ATOMIC_RELEASE);
    return 0;
}

int ls_b200_queue_fail(ls_b200_queue* q, uint32_t error) {
    if (!q || !q->view.control) return EINVAL;
    uint32_t clear = 0;
    __atomic_compare_exchange_n(&q->view.control->error, &clear, error, false, __ATOMIC_RELEASE, __ATOMIC_RELAXED);
    return 0;
}

const char* ls_b200_build_info(void) { return "leanstream_b200 sm_100a fused-mlp v4 (CTA-local slabs, tensor-core gate/up and down)"; }

}  // extern "C"
