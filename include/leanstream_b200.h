/*
 * leanstream_b200.h -- C ABI of the B200 sparse streaming-MLP compute backend.
 *
 * This header is the whole drop-in boundary. It replaces two reference
 * surfaces:
 *   - backends/triton/enqueue.cpp + include/leanstream/triton_cuda.h
 *     (the ls_triton_* ABI and TritonBackend::view);
 *   - kernels/streaming_mlp.cu/.cuh and streaming_mlp_candidates.cu
 *     (the CUDA reference backend: core_kernel -> consumer -> reduction).
 * Only plain integers, pointers and POD structs cross it. No torch types.
 *
 * The structs marked "binary-compatible" have exactly the layout of the
 * reference's C++ types. A C++ caller that owns a leanstream::runtime::Runtime
 * can therefore reinterpret an ls_compute_backend as a ComputeBackend.
 * The static asserts in leanstream_b200/csrc/ls_backend.cu check the layout.
 *
 * Memory model (discrete B200, PCIe host):
 *   - Packed weights (cache, staging), scales, input/output vectors and the
 *     optional activation / counter buffers are DEVICE memory.
 *   - Descriptors, ready indices and ls_queue_control may be either device
 *     memory or mapped pinned host memory (cudaHostAllocMapped). The kernel
 *     reads them with system-scope acquire loads and never writes them; a
 *     queue in host memory is read by one thread of the grid at a time,
 *     which copies what was published into backend-owned device memory
 *     for the other CTAs (reads over PCIe are slow and compete with the
 *     copy engine).
 *   - Claim counters live in a backend-owned device workspace. Discrete GPUs
 *     do not provide host-native atomics, so QueueControl.claim_count and
 *     consumer_path are left untouched.
 * Every device-side wait is bounded by a %globaltimer deadline. On expiry
 * the kernel records an LS_B200_DEV_* code in the status words and exits.
 */
#ifndef LEANSTREAM_B200_H
#define LEANSTREAM_B200_H

#include <stddef.h>
#include <stdint.h>
#ifndef __cplusplus
#include <stdbool.h>
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ */
/* Binary-compatible mirrors of the reference descriptor/queue types.  */
/* ------------------------------------------------------------------ */

/* ExecDesc (include/leanstream/types.h:16-20): five uint32, 20 bytes. */
typedef struct ls_exec_desc {
    uint32_t logical_group;  /* predictor / application ID */
    uint32_t physical_group; /* selects the fp16 scale rows */
    uint32_t source_slot;    /* slot in cache (kind 0) or staging (kind 1) */
    uint32_t dest_slot;      /* deterministic partial / activation destination */
    uint32_t source_kind;    /* LS_SOURCE_CACHE or LS_SOURCE_STAGING */
} ls_exec_desc;

enum { LS_SOURCE_CACHE = 0, LS_SOURCE_STAGING = 1 };

/* ConsumerMode (types.h:13), an enum class : uint8_t. */
enum { LS_MODE_BATCH_COMPAT = 0, LS_MODE_PROGRESSIVE = 1, LS_MODE_AUTO = 2 };

/* QueueControl (include/leanstream/execution_queue.h:5-12): 128 bytes,
 * epoch at byte 12, claim_count on its own cache line at byte 64. */
typedef struct ls_queue_control {
    uint32_t ready_count, reserved, total_count, epoch;
    uint32_t batch_epoch, error, consumer_path, init_arrived, init_epoch;
    uint32_t pad0[7];
    uint32_t claim_count;
    uint32_t pad1[15];
} ls_queue_control;

/* DeviceExecQueue (execution_queue.h:13-18). */
typedef struct ls_device_exec_queue {
    ls_exec_desc* descriptors;
    uint32_t* ready_indices;
    ls_queue_control* control;
    uint32_t capacity;
} ls_device_exec_queue;

/* Span<ExecDesc> and Span<GroupId> (types.h:7-10). */
typedef struct ls_exec_span { const ls_exec_desc* data; size_t size; } ls_exec_span;
typedef struct ls_group_span { const int32_t* data; size_t size; } ls_group_span;

/* ComputeBackend (include/leanstream/runtime.h:10-22). ConsumerMode is
 * passed as its underlying uint8_t. */
typedef struct ls_compute_backend {
    void* context;
    int (*enqueue)(void* context, uint32_t layer, const void* input, void* output, void* stream,
                   ls_exec_span core, ls_device_exec_queue queue, uint32_t epoch, uint8_t mode);
    bool (*complete)(void* context, uint32_t layer);
    int (*commit)(void* context, uint32_t layer, ls_group_span ids);
    int (*defer_commit)(void* context, uint32_t layer, ls_group_span ids, uint32_t epoch,
                        void (*retired)(void*, uint32_t epoch), void* retirement_context);
    void (*cancel)(void* context, uint32_t layer, uint32_t epoch);
} ls_compute_backend;

/* KernelCandidate (include/leanstream/kernel_selector.h:6-12). */
typedef struct ls_kernel_candidate {
    uint32_t id;
    uint32_t workers;     /* persistent CTAs, as in the Triton catalog
                           * entry_point: 1 = tensor-core gate/up, 0 = CUDA-core fma */
    const char* name;
    uint32_t cta_count, tile_size, unroll, group_batch, entry_point;
    bool available;
} ls_kernel_candidate;

/* ------------------------------------------------------------------ */
/* Backend geometry and borrowed buffers.                              */
/* ------------------------------------------------------------------ */

typedef struct ls_b200_geometry {
    uint32_t hidden;        /* H: 256, 512, 1024, 2048, 4096 or 8192 */
    uint32_t group_size;    /* G: neurons per logical group, 1..256 */
    uint32_t group_count;   /* N: logical groups = dest slots = partial rows */
    uint32_t max_layers;    /* number of per-layer completion words (0 -> 256) */
    uint32_t cache_slots;   /* optional bound on cache source_slot (0 = unchecked) */
    uint32_t staging_slots; /* optional bound on staging source_slot (0 = unchecked) */
    uint32_t physical_groups; /* optional bound on physical_group (0 = unchecked) */
    uint32_t timeout_us;    /* bound of every device wait (0 -> 5,000,000) */
    float rms_eps;          /* epsilon of the optional RMSNorm prologue */
} ls_b200_geometry;

/* Flags of ls_b200_layer_args.flags. */
enum {
    LS_B200_NORM_INPUT = 1u << 0, /* apply HF RMSNorm to the input before the MLP */
    LS_B200_NO_OUTPUT = 1u << 1   /* skip the fp16 output store (fp32 partial only) */
};

/* Every buffer of one MLP layer invocation. Borrowed until GPU completion. */
typedef struct ls_b200_layer_args {
    const void* input;        /* fp16 [H] */
    void* output;             /* fp16 [H]: y = fp16(sum of partial rows) */
    const uint8_t* cache;     /* packed INT4 groups (device memory) */
    const uint8_t* staging;   /* packed INT4 groups (device memory; may equal cache) */
    const void* scales;       /* fp16 [physical_group][G][3][H/128] */
    const ls_exec_desc* core; /* core descriptors (GPU-addressable), dest slots first */
    uint32_t core_count;
    uint32_t epoch;           /* QueueControl.epoch this launch consumes (nonzero) */
    ls_device_exec_queue queue;
    uint8_t mode;             /* LS_MODE_* */
    uint8_t pad[3];
    uint32_t flags;           /* LS_B200_* flags */
    int32_t candidate;        /* kernel candidate id, or -1 for the selector's choice */
    uint32_t layer;           /* completion word index */
    void* activations;        /* optional fp16 [N*G]: h at dest_slot*G + neuron */
    uint32_t* executions;     /* optional [N]: +1 per executed descriptor, dest-indexed */
    uint64_t* first_compute;  /* optional [N]: %globaltimer when a descriptor is claimed */
    const void* residual;     /* optional fp16 [H]: hidden_out = fp16(residual + y) */
    void* hidden_out;         /* optional fp16 [H] */
    float* output_f32;        /* optional fp32 [H]: unrounded sum (tensor-parallel partial) */
    const void* norm_weight;  /* optional fp16 [H] RMSNorm weight (NULL = ones) */
    uint64_t* trace;          /* optional %globaltimer phase stamps: [grid][LS_B200_TRACE_WORDS]
                               * per CTA, then [grid][layers][LS_B200_LAYER_TRACE_WORDS]
                               * per CTA and layer, then [4][LS_B200_PIECE_TRACE_PIECES][4]
                               * per piece of CTAs 0..3 (LS_B200_*TRACE_*); the Stamp
                               * buffers of backends/triton/core.py:25, persistent.py:37 */
    float* importance;        /* optional fp32 [N], dest-indexed: sum over the group's G neurons
                               * of |h| (the importance output of
                               * examples/ministral/native/leanstream_mapped.cu:43-47,
                               * summed exactly and rounded to fp32 once); entries of
                               * destinations the layer did not execute are 0 */
    uint32_t* importance_flag; /* optional: receives the epoch (release, system scope) once
                               * every importance entry of the layer is written
                               * (leanstream_mapped.cu:36-39 publish) */
} ls_b200_layer_args;

/* Phase stamps written per CTA when ls_b200_layer_args.trace is set. */
enum {
    LS_B200_TRACE_ENTRY = 0,     /* kernel entry */
    LS_B200_TRACE_DECIDED = 1,   /* producer learned the consumer path */
    LS_B200_TRACE_FIRST = 2,     /* first stage consumed */
    LS_B200_TRACE_PIECES = 3,    /* consumers saw END */
    LS_B200_TRACE_PRODUCED = 4,  /* producer issued END */
    LS_B200_TRACE_BARRIER = 5,   /* grid barrier passed */
    LS_B200_TRACE_REDUCED = 6,   /* reduction done */
    LS_B200_TRACE_EXIT = 7,      /* CTA done (after the exit counter) */
    LS_B200_TRACE_WORDS = 8
};
/* Per-layer phase stamps (after the per-CTA block). */
enum {
    LS_B200_LTRACE_DECIDED = 0,        /* producer decided the layer's path */
    LS_B200_LTRACE_ISSUED = 1,         /* producer issued the layer's last piece */
    LS_B200_LTRACE_PIECES_DONE = 2,    /* consumers reached the end-of-layer marker */
    LS_B200_LTRACE_PARTIALS_READY = 3, /* all partial rows of the layer written (reducer warps) */
    LS_B200_LTRACE_REDUCED = 4,        /* this CTA's reduction blocks done */
    LS_B200_LTRACE_NEXT_READY = 5,     /* every reduction block of the layer done */
    LS_B200_LTRACE_LOADED = 6,         /* next layer's activation loaded (stamped under that layer) */
    LS_B200_LAYER_TRACE_WORDS = 8
};
/* Per-piece stamps of CTAs 0..3 (after the per-layer block):
 * [4][LS_B200_PIECE_TRACE_PIECES][4] = producer issued, producer closed,
 * consumer warp 0 saw the stage full, consumer warp 0 finished it. */
enum { LS_B200_PIECE_TRACE_PIECES = 128 };

/* Device status words (ls_b200_status). */
enum {
    LS_B200_STATUS_ERROR = 0,       /* LS_B200_DEV_* code of the latest failed launch */
    LS_B200_STATUS_ERROR_EPOCH = 1, /* epoch (first layer) of that launch */
    LS_B200_STATUS_ERROR_DETAIL = 2,/* position / slot / wait site involved */
    LS_B200_STATUS_LAUNCHES = 3,    /* layers executed by this backend's launches (mod 0xFFFF0000) */
    LS_B200_STATUS_WORDS = 4
};
enum {
    LS_B200_DEV_OK = 0,
    LS_B200_DEV_QUEUE_ERROR = 1,    /* QueueControl.error observed nonzero */
    LS_B200_DEV_TIMEOUT_EPOCH = 2,  /* epoch / batch_epoch never published */
    LS_B200_DEV_TIMEOUT_READY = 3,  /* a claimed position never became ready */
    LS_B200_DEV_TIMEOUT_SYNC = 4,   /* an intra-kernel wait exceeded the deadline */
    LS_B200_DEV_BAD_DESCRIPTOR = 5, /* slot / group / index out of range */
    LS_B200_DEV_BAD_PLAN = 6        /* total_count exceeds capacity or slots */
};

/* ------------------------------------------------------------------ */
/* Backend lifecycle (mirrors ls_triton_*, triton_cuda.h:49-57).        */
/* ------------------------------------------------------------------ */

/* ls_triton_create (triton_cuda.h:50): backend with the built-in fallback only. */
void* ls_b200_create(void);
/* ls_triton_create_table (triton_cuda.h:51): borrowed row-major LUT
 * [layers * buckets] of candidate ids, immutable for the backend lifetime. */
void* ls_b200_create_table(const uint8_t* lut, uint32_t layers, uint32_t buckets);
/* ls_triton_destroy (triton_cuda.h:52). Caller must have proved GPU completion. */
void ls_b200_destroy(void* backend);
/* Cold setup, replaces ls_triton_bind (triton_cuda.h:54-55): validates the
 * geometry, checks the device is sm_100, allocates the device workspace and
 * the mapped status / completion words. Call once on the device that runs
 * the launches; returns 0 or an errno-style code. */
int ls_b200_configure(void* backend, const ls_b200_geometry* geometry);
/* Borrowed buffers used by ls_b200_enqueue and the ComputeBackend view
 * (MLPBuffers, kernels/streaming_mlp.cuh:6-14). input/output fields are
 * overridden by ComputeBackend.enqueue's arguments. */
int ls_b200_set_buffers(void* backend, const ls_b200_layer_args* buffers);
/* KernelRuntimeState (kernel_selector.h:4) used by the next enqueue;
 * TritonBackend::state (triton_cuda.h:38). */
void ls_b200_set_state(void* backend, uint32_t layer, uint32_t io_bucket);

/* ------------------------------------------------------------------ */
/* Submission.                                                          */
/* ------------------------------------------------------------------ */

/* One fused launch (A core + persistent B consumer + compact reduction)
 * on `stream`: every buffer comes from `args`. No allocation,
 * compilation or synchronisation. Replaces enqueue_streaming_mlp
 * (kernels/streaming_mlp.cu:85-93). */
int ls_b200_launch(void* backend, const ls_b200_layer_args* args, void* stream);

/* No counterpart in the reference. The launch of ls_b200_launch for callers
 * that must not allocate device memory: no backend object, no cudaMalloc,
 * no allocating library routine. The scratch is a fixed set of device
 * arrays in the library, one set per device that loads it, held until exit:
 * 32 MiB of partial rows, 128 KiB of layer hand-off words and 512 KiB for a
 * device copy of a queue kept in host memory.
 * geometry: as for ls_b200_configure (max_layers is ignored). Returns
 * E2BIG when group_count * ceil(group_size / 16) * hidden exceeds 2^22 or
 * args->layer >= 256, EINVAL for the cases ls_b200_launch rejects. status:
 * optional GPU-addressable [LS_B200_STATUS_WORDS] words that receive the
 * launch's device status; NULL sends it to a word set in the library that
 * no call reads. The first call on a device (that device current) does the
 * set-up: symbol lookup, kernel attributes and zeroing on `stream`; make it
 * before any stream capture. Under CUDA's lazy module loading the arrays
 * are committed on the device by that set-up, so a caller whose memory pool
 * will claim the rest of HBM makes it first: args == NULL runs the set-up
 * alone (geometry and status are then ignored) and launches nothing. Calls
 * whose launches overlap in time on one device race on the shared scratch:
 * order them on one stream. */
int ls_b200_launch_static(const ls_b200_geometry* geometry, const ls_b200_layer_args* args, uint32_t* status,
                          void* stream);
/* Multi-layer launch: `count` layers in ONE persistent launch, each layer
 * reading the previous layer's hidden_out as input (a decode stack with the
 * residual / RMSNorm epilogue fused). Plans are encoded on the host with
 * ls_b200_encode_plan (ls_b200_plan_size bytes each); the caller copies
 * them to 16-byte-aligned device memory (stream-ordered before the launch)
 * and passes both copies: the device array is read by the kernel, the host
 * array is validated and records per-layer completion epochs. */
uint32_t ls_b200_plan_size(void);
int ls_b200_encode_plan(void* backend, const ls_b200_layer_args* args, void* plan);
int ls_b200_launch_plans(void* backend, const void* device_plans, uint32_t count, const void* host_plans,
                         int32_t candidate, uint64_t* trace, void* stream);
/* ls_triton_enqueue (triton_cuda.h:56; enqueue.cpp:26-37): LUT-selected
 * candidate, bound buffers and queue from ls_b200_set_buffers. */
int ls_b200_enqueue(void* backend, uint32_t layer, uint32_t bucket, uint32_t epoch, void* stream);
/* TritonBackend::view (enqueue.cpp:46): fills a ComputeBackend whose
 * enqueue accepts BatchCompat, Progressive and Auto (Auto waits for the
 * batch epoch, as streaming_mlp.cu:90 does). complete() polls the
 * per-layer completion word; commit() accepts the next resident set
 * (cache installation belongs to the application; returns 0). */
int ls_b200_view(void* backend, ls_compute_backend* out);
/* Last epoch whose launch for `layer` has fully finished on the GPU
 * (reduction included), read from mapped memory without synchronising.
 * This is the Done epoch of backends/triton/primitives.py:10-14. */
int ls_b200_completed_epoch(void* backend, uint32_t layer, uint32_t* epoch);

/* Tensor parallel inside one launch (no counterpart in the reference, whose
 * multi-GPU step is an allreduce between launches). Each rank computes the
 * fp32 partial output of its own groups; at the end of every layer its
 * reducer CTAs store their columns into every rank's exchange buffer over
 * NVLink peer memory, and every rank forms y = the sum over ranks in rank
 * order, fp16(y) and fp16(residual + fp16(y)) -- the arithmetic of an
 * allreduce followed by ls_b200_tp_epilogue -- inside the same persistent
 * launch, so a whole stack of layers is one launch per rank.
 * ls_b200_tp_setup allocates and zeroes this rank's exchange buffer and
 * writes its CUDA IPC handle (LS_B200_TP_HANDLE_BYTES) to handle_out; the
 * host gathers the handles of all ranks (rank order) and passes them to
 * ls_b200_tp_connect, which maps the peers' buffers and resets the tag
 * counter. Afterwards every launch through the backend is a collective:
 * all ranks issue the same launches in the same order. Consecutive layers
 * of one launch must chain (next input = hidden_out) and a hidden_out's
 * residual must be its layer's input, else EINVAL. world <= 8. */
enum { LS_B200_TP_HANDLE_BYTES = 64 };
int ls_b200_tp_setup(void* backend, uint32_t rank, uint32_t world, void* handle_out);
int ls_b200_tp_connect(void* backend, const void* handles);

/* Tensor-parallel layer epilogue (one rank): after the fp32 partial outputs
 * of all ranks are summed (NCCL allreduce of output_f32), round once to fp16
 * and add the residual -- the single-GPU epilogue of
 * backends/triton/reduction.py:14-20 split across the collective.
 * output (optional): fp16 y; hidden_out (optional): fp16(residual + y). */
int ls_b200_tp_epilogue(const float* y32, const void* residual, void* output, void* hidden_out, uint32_t hidden,
                        void* stream);
/* Bounded device-side delay (<= 100 ms) on `stream`. Benchmarks queue it
 * ahead of event-bracketed launches so the brackets measure kernels only. */
int ls_b200_spin(uint64_t nanoseconds, void* stream);

/* Device status words (LS_B200_STATUS_*), read without synchronising. */
int ls_b200_status(void* backend, uint32_t* words, uint32_t count);
int ls_b200_clear_status(void* backend);
/* Scratch sizes the backend allocated (partials, workspace), in bytes. */
uint64_t ls_b200_scratch_bytes(void* backend);

/* ------------------------------------------------------------------ */
/* Kernel selection (src/runtime/kernel_selector.cpp, triton_backend.h). */
/* ------------------------------------------------------------------ */

/* quantize_io_load (kernel_selector.cpp:4-8). */
uint32_t ls_b200_quantize_io_load(uint32_t remaining, uint32_t total, uint32_t buckets);
/* KernelSelector::select (kernel_selector.cpp:17-22) over the B200 catalog. */
uint32_t ls_b200_select(void* backend, uint32_t layer, uint32_t io_bucket);
/* KernelSelector::candidate (kernel_selector.cpp:9-16). */
int ls_b200_candidate(void* backend, uint32_t id, ls_kernel_candidate* out);
/* Number of catalog entries and the fallback id. */
uint32_t ls_b200_catalog_size(void);
uint32_t ls_b200_default_candidate(void);

/* ------------------------------------------------------------------ */
/* Host producer: ExecutionQueue (src/runtime/execution_queue.cpp:4-46) */
/* restated for callers that do not link the reference runtime.        */
/* ------------------------------------------------------------------ */

typedef struct ls_b200_queue {
    ls_device_exec_queue view;
    uint32_t tail, epoch, total;
} ls_b200_queue;

void ls_b200_queue_bind(ls_b200_queue* queue, ls_device_exec_queue view);
int ls_b200_queue_reset(ls_b200_queue* queue, uint32_t epoch);
int ls_b200_queue_prepare(ls_b200_queue* queue, uint32_t total);
int ls_b200_queue_append_unpublished(ls_b200_queue* queue, uint32_t index);
int ls_b200_queue_activate(ls_b200_queue* queue);
int ls_b200_queue_seal(ls_b200_queue* queue, uint32_t total);
int ls_b200_queue_publish_all(ls_b200_queue* queue);
int ls_b200_queue_publish(ls_b200_queue* queue, uint32_t index);
int ls_b200_queue_fail(ls_b200_queue* queue, uint32_t error);

/* ------------------------------------------------------------------ */
/* Batched decode over the union of the tokens' active groups.          */
/* ------------------------------------------------------------------ */

/* (new; the reference decodes one token at a time) Up to 8 tokens share one
 * pass over the union of their active groups: every weight byte is read once
 * and the tokens are the N dimension of the tensor-core MMAs. mask
 * (optional, [tokens][union_count] bytes): token b uses union group u only
 * where mask is nonzero, so its output equals the one-token MLP over its own
 * groups; NULL gives every token the whole union. Rounding as the one-token
 * path (w = fp16(q*s), fp16 g, u, silu and h, fp32 partial sums, one fp16
 * rounding of y), fixed summation order (deterministic). The descriptors are
 * trusted (device memory; physical_group selects the scales, source_slot the
 * group in cache (kind 0) or staging (kind 1)). scratch: device memory of at
 * least ls_b200_batch_scratch_bytes(), 16-byte aligned; x, cache and staging
 * 16-byte aligned, scales 4-byte aligned. Hidden a multiple of 256 up to
 * 8192. Bad arguments return EINVAL (ENOSPC for short scratch) before any
 * CUDA call; nothing is allocated. The first call on a device sets the
 * kernels' shared-memory attributes: make it before any stream capture. */
typedef struct ls_b200_batch_args {
    uint32_t hidden, group_size, union_count, tokens;  /* tokens 1..8 */
    const void* x;            /* fp16 [tokens][H] */
    void* output;             /* fp16 [tokens][H] */
    float* output_f32;        /* optional fp32 [tokens][H] */
    const void* residual;     /* optional fp16 [tokens][H]: hidden_out = fp16(residual + y) */
    void* hidden_out;         /* optional fp16 [tokens][H] */
    const uint8_t* cache;
    const uint8_t* staging;   /* optional (NULL = cache) */
    const void* scales;       /* fp16 [physical_group][G][3][H/128] */
    const ls_exec_desc* union_descs;  /* device [union_count] */
    const uint8_t* mask;      /* optional device [tokens][union_count] */
    void* scratch;
    uint64_t scratch_bytes;
    uint32_t flags;           /* 0 or LS_B200_NORM_INPUT: HF RMSNorm of each token before the MLP
                               * (predictor_shared_input.cu:16-33), so that with residual and
                               * hidden_out the call is one layer of a decode stack */
    float rms_eps;            /* epsilon of the RMSNorm */
    const void* norm_weight;  /* optional fp16 [H] RMSNorm weight (NULL = ones) */
    uint32_t* error;          /* optional device word: bit 0 set (atomic OR, never cleared) when a
                               * bounded wait of the tensor-core kernels gave up; the call's
                               * outputs are then invalid */
    uint64_t timeout_ns;      /* bound of every wait of the tensor-core kernels (0 = 2 s, at most
                               * 60 s); after it, the kernels still wait up to 1 s more for their
                               * own copies and MMAs in flight before they end */
} ls_b200_batch_args;
/* Flags of ls_b200_batch_args.flags besides LS_B200_NORM_INPUT. */
enum {
    /* The two weight kernels on the legacy warp-level MMA (mma.sync m16n8k16)
     * instead of the 5th-generation tensor cores (tcgen05.mma with the
     * accumulator in tensor memory, the default) -- kept for comparison. */
    LS_B200_BATCH_MMA_SYNC = 1u << 8
};
uint64_t ls_b200_batch_scratch_bytes(uint32_t hidden, uint32_t group_size, uint32_t union_count);
int ls_b200_batch_mlp(const ls_b200_batch_args* args, void* stream);

/* ------------------------------------------------------------------ */
/* Streaming IO: IOBackend (include/leanstream/weight_manager.h:8-24)  */
/* over pinned host memory -> HBM staging copies.                      */
/* ------------------------------------------------------------------ */

/* IOCompletion (weight_manager.h:8-11) and its callback; the reference
 * passes the completion by const reference, i.e. by address. */
typedef struct ls_io_completion {
    uint32_t epoch;
    int32_t logical_group;
    int32_t staging_slot;
    int32_t error;
    uint64_t slot_sequence;
} ls_io_completion;
typedef void (*ls_io_completion_fn)(void* arg, const ls_io_completion* completion);

/* IOBackend (weight_manager.h:14-24): the table a WeightManager borrows
 * through ManagerConfig::io_backend. */
typedef struct ls_io_backend {
    void* context;
    int (*begin)(void* context, ls_io_completion_fn callback, void* arg, uint32_t epoch);
    int (*update)(void* context, ls_group_span priority);
    int (*consume)(void* context, ls_group_span final_reads);
    int (*retire)(void* context);
    int32_t (*ready_slot)(void* context, int32_t group);
    uint64_t (*requests)(void* context);
    int (*wait)(void* context, int timeout_ms);
} ls_io_backend;

/* io_states words, as the reference stream engine publishes them
 * (src/io/stream_io.h:6); io_states[group_count] holds a terminal errno. */
enum { LS_IO_EMPTY = 0, LS_IO_INFLIGHT = 1, LS_IO_READY = 2, LS_IO_ERROR = 3 };

typedef struct ls_b200_stream_config {
    const void* host_base;         /* pinned host memory (cudaHostAlloc / cudaHostRegister) */
    const uint64_t* host_offsets;  /* [group_count]: byte offset of logical group g in host_base */
    void* staging;                 /* device memory: group g lands at staging + g * staging_stride */
    uint64_t staging_stride;
    uint64_t group_bytes;          /* bytes copied per group (<= staging_stride) */
    uint32_t* io_states;           /* [group_count + 1] host words shared with the caller */
    uint32_t group_count;
    uint32_t queue_depth;          /* copies in flight, 1..32 (ManagerConfig::qd) */
    int32_t device;                /* CUDA device of the staging memory */
    float delay_mean_us;           /* emulated IO latency: each landed group becomes READY after an
                                    * extra delay ~ Exp(mean) (seeded); 0 = none */
    uint64_t delay_seed;
    /* Optional SSD leg (src/io/stream_io.cpp:75-148): with file_path set, an
     * admitted group is first read from the file (pread by a pool of reader
     * threads) into its host slot host_base + host_offsets[g], then copied
     * to HBM as above; NULL = host_base already holds every group. */
    const char* file_path;
    const uint64_t* file_offsets;  /* [group_count]: byte offset of group g in the file */
    uint32_t read_workers;         /* reader threads, 1..16 (0 = 4) */
    uint32_t o_direct;             /* 1: open with O_DIRECT (no page cache). Each read is then
                                    * group_bytes rounded up to file_alignment, so every host slot
                                    * must hold that many bytes; when the file system refuses
                                    * O_DIRECT or an offset / slot is not aligned, buffered reads
                                    * are used (ls_b200_stream_counters.direct tells which) */
    uint32_t file_alignment;       /* O_DIRECT alignment in bytes, a power of two (0 = 4096) */
} ls_b200_stream_config;

typedef struct ls_b200_stream_counters {
    uint64_t admissions;    /* copies issued (IOBackend::requests) */
    uint64_t completions;   /* groups published READY */
    uint64_t bytes;         /* bytes copied host -> HBM */
    uint64_t first_issue_ns, last_land_ns;  /* CLOCK_MONOTONIC of the first copy issue / last landing */
    uint64_t copy_ns;       /* sum over copies of issue -> landing as the worker observed it */
    int32_t error;          /* first error (CUDA error code or errno), 0 if none */
    uint32_t outstanding;   /* reads and copies in flight now */
    uint32_t direct;        /* file source: 1 when reads bypass the page cache (O_DIRECT) */
    uint32_t reserved;
    uint64_t read_bytes;    /* file source: bytes read from the file */
    uint64_t read_ns;       /* file source: sum over reads of the pread time */
} ls_b200_stream_counters;

/* (new; the reference transport reads an O_DIRECT file into host memory the
 * GPU maps, src/io/stream_io.cpp:75-148, which a discrete GPU cannot use as
 * staging) Creates the engine: one worker thread, one CUDA stream and
 * `queue_depth` events on `device`. Returns NULL (errno EINVAL / ENOMEM /
 * ENODEV) on failure. The worker admits groups in the priority order of the
 * last update (then, after consume, the committed final reads), one
 * cudaMemcpyAsync per group, never preempting a started copy; a landed
 * group's io_states word turns READY (release) before its completion
 * callback runs on the worker thread. */
void* ls_b200_stream_create(const ls_b200_stream_config* config);
/* Fills the IOBackend table for this engine. */
int ls_b200_stream_view(void* engine, ls_io_backend* out);
int ls_b200_stream_stats(void* engine, ls_b200_stream_counters* out);
/* Admission order of the current session (logical ids), up to `capacity`;
 * returns the number written. Tests and diagnostics. */
uint32_t ls_b200_stream_issue_log(void* engine, int32_t* out, uint32_t capacity);
/* Stops the worker after draining in-flight copies; the caller has retired
 * the session. */
void ls_b200_stream_destroy(void* engine);

/* Library build identity: "sm_100a" plus the kernel revision. */
const char* ls_b200_build_info(void);

#ifdef __cplusplus
}
#endif
#endif /* LEANSTREAM_B200_H */
