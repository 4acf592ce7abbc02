// Timing driver for the reference's own CUDA backend, test infrastructure
// only: kernels/streaming_mlp.cu of the reference is compiled unmodified
// from the reference tree and linked with this file by oracle/Makefile
// (target ref-cuda, output oracle/_ref/ref_streaming_timer). It runs the
// reference's enqueue_streaming_mlp (kernels/streaming_mlp.cu:85-93: core
// kernel -> persistent consumer -> reduction) on seeded synthetic inputs of
// a BASELINE.json configuration and prints one JSON line per worker count.
//
// Set-up (all in device memory, so the consumer's atomics on the queue
// control are device-local): `active` groups, descriptors in caller order
// {logical = physical = slot = group id, dest = position, kind = cache}, a
// sealed all-ready plan (epoch = batch_epoch = 1, ready_count =
// total_count = active), BatchCompat mode: the consumer takes its all-ready
// static-stripe path (streaming_mlp.cu:58-62), no claims, no host atomics.
// Every index the kernels use is inside its buffer: dest < active rows of
// `partial`, slot < groups of `cache`, physical < groups of `scales`.
//
//   ref_streaming_timer <hidden> <group_size> <groups> <active> <reps> <workers...>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <numeric>
#include <random>
#include <vector>

#include "streaming_mlp.cuh"

using namespace leanstream::runtime;

#define CHECK(x)                                                                   \
    do {                                                                           \
        cudaError_t e_ = (x);                                                      \
        if (e_ != cudaSuccess) {                                                   \
            std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));         \
            std::exit(2);                                                          \
        }                                                                          \
    } while (0)

int main(int argc, char** argv) {
    if (argc < 7) {
        std::fprintf(stderr, "usage: %s hidden group_size groups active reps workers...\n", argv[0]);
        return 1;
    }
    const uint32_t H = uint32_t(std::atoi(argv[1])), G = uint32_t(std::atoi(argv[2]));
    const uint32_t groups = uint32_t(std::atoi(argv[3])), active = uint32_t(std::atoi(argv[4]));
    const int reps = std::atoi(argv[5]);
    if (!H || H % 256 || !G || !groups || !active || active > groups || reps < 1) return 1;
    const size_t group_bytes = size_t(G) * 3 * H / 2;
    const size_t scale_count = size_t(groups) * G * 3 * (H / 128);

    std::mt19937_64 rng(1234);
    std::vector<uint8_t> cache(group_bytes * groups);
    for (auto& b : cache) b = uint8_t(rng());
    std::uniform_real_distribution<float> su(0.005f, 0.02f);
    std::vector<__half> scales(scale_count);
    for (auto& s : scales) s = __float2half(su(rng));
    std::normal_distribution<float> nd(0.f, 1.f);
    std::vector<__half> x(H);
    for (auto& v : x) v = __float2half(nd(rng));
    std::vector<uint32_t> ids(groups);
    std::iota(ids.begin(), ids.end(), 0u);
    std::shuffle(ids.begin(), ids.end(), rng);
    ids.resize(active);
    std::sort(ids.begin(), ids.end());
    std::vector<ExecDesc> desc(active);
    std::vector<uint32_t> ready(active);
    for (uint32_t i = 0; i < active; ++i) {
        desc[i].logical_group = ids[i];
        desc[i].physical_group = ids[i];
        desc[i].source_slot = ids[i];
        desc[i].dest_slot = i;
        desc[i].source_kind = SourceKind::Cache;
        ready[i] = i;
    }
    QueueControl ctl{};
    ctl.ready_count = active;
    ctl.total_count = active;
    ctl.epoch = 1;
    ctl.batch_epoch = 1;

    uint8_t* d_cache;
    __half *d_scales, *d_x, *d_y;
    float* d_partial;
    ExecDesc* d_desc;
    uint32_t* d_ready;
    QueueControl* d_ctl;
    CHECK(cudaMalloc(&d_cache, cache.size()));
    CHECK(cudaMalloc(&d_scales, scales.size() * sizeof(__half)));
    CHECK(cudaMalloc(&d_x, H * sizeof(__half)));
    CHECK(cudaMalloc(&d_y, H * sizeof(__half)));
    CHECK(cudaMalloc(&d_partial, size_t(active) * H * sizeof(float)));
    CHECK(cudaMalloc(&d_desc, active * sizeof(ExecDesc)));
    CHECK(cudaMalloc(&d_ready, active * sizeof(uint32_t)));
    CHECK(cudaMalloc(&d_ctl, sizeof(QueueControl)));
    CHECK(cudaMemcpy(d_cache, cache.data(), cache.size(), cudaMemcpyHostToDevice));
    CHECK(cudaMemcpy(d_scales, scales.data(), scales.size() * sizeof(__half), cudaMemcpyHostToDevice));
    CHECK(cudaMemcpy(d_x, x.data(), H * sizeof(__half), cudaMemcpyHostToDevice));
    CHECK(cudaMemcpy(d_desc, desc.data(), active * sizeof(ExecDesc), cudaMemcpyHostToDevice));
    CHECK(cudaMemcpy(d_ready, ready.data(), active * sizeof(uint32_t), cudaMemcpyHostToDevice));
    CHECK(cudaMemcpy(d_ctl, &ctl, sizeof(QueueControl), cudaMemcpyHostToDevice));

    DeviceExecQueue q;
    q.descriptors = d_desc;
    q.ready_indices = d_ready;
    q.control = d_ctl;
    q.capacity = active;
    MLPBuffers b{d_x, d_cache, d_cache, d_scales, d_partial, nullptr, nullptr};
    cudaStream_t s;
    CHECK(cudaStreamCreate(&s));
    cudaEvent_t e0, e1;
    CHECK(cudaEventCreate(&e0));
    CHECK(cudaEventCreate(&e1));
    const double alg_bytes = double(active) * G * (3.0 * H / 2 + 3.0 * (H / 128) * 2);
    for (int a = 6; a < argc; ++a) {
        const uint32_t workers = uint32_t(std::atoi(argv[a]));
        if (!workers) continue;
        CHECK(enqueue_streaming_mlp({nullptr, 0}, q, b, d_y, 1, H, G, workers, ConsumerMode::BatchCompat, s));
        CHECK(cudaStreamSynchronize(s));
        CHECK(cudaEventRecord(e0, s));
        for (int r = 0; r < reps; ++r)
            CHECK(enqueue_streaming_mlp({nullptr, 0}, q, b, d_y, 1, H, G, workers, ConsumerMode::BatchCompat, s));
        CHECK(cudaEventRecord(e1, s));
        CHECK(cudaEventSynchronize(e1));
        float ms = 0.f;
        CHECK(cudaEventElapsedTime(&ms, e0, e1));
        std::vector<__half> y(H);
        CHECK(cudaMemcpy(y.data(), d_y, H * sizeof(__half), cudaMemcpyDeviceToHost));
        double l1 = 0.0;
        bool finite = true;
        for (auto v : y) {
            const float f = __half2float(v);
            finite = finite && std::isfinite(f);
            l1 += std::fabs(f);
        }
        const double us = 1e3 * ms / reps;
        std::printf(
            "{\"hidden\": %u, \"group_size\": %u, \"groups\": %u, \"active\": %u, \"workers\": %u, "
            "\"launches_per_layer\": 2, \"reps\": %d, \"us_per_layer\": %.3f, \"gb_per_s\": %.2f, "
            "\"output_finite\": %s, \"output_l1\": %.4g}\n",
            H, G, groups, active, workers, reps, us, alg_bytes / (us * 1e-6) / 1e9, finite ? "true" : "false", l1);
        std::fflush(stdout);
    }
    return 0;
}
