// Integration driver (test infrastructure): the reference's own C++ runtime
// (leanstream::runtime::Runtime / LayerStep / WeightManager / ExecutionQueue,
// compiled unmodified from its sources into oracle/_ref) drives the B200
// ComputeBackend (ls_b200_view) and the B200 streaming IOBackend
// (ls_b200_stream_view) through their reference interfaces, one layer step
// at a time, as include/leanstream/runtime.h prescribes:
//   begin_layer -> update_prediction(P0) -> enqueue_compute (Progressive
//   launch) -> update_prediction(P1) (reorders unstarted reads) ->
//   finalize(F) -> kernel completes -> commit({}).
// Weights live in pinned host memory; only predicted groups are copied.
//
// usage: runtime_driver DIR H G N QD DELAY_US CANDIDATE STEPS
//   DIR/packed.bin  N * G * 3H/2 bytes     DIR/scales.bin  N * G * 3 * H/128 fp16
//   DIR/x.bin       H fp16                  DIR/plan.txt    three lines: P0, P1, F (group ids)
// writes DIR/y.bin (fp16 y of the last step) and prints one JSON line of timings.
#include <cuda_runtime.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "leanstream/runtime.h"
#include "leanstream_b200.h"

namespace rt = leanstream::runtime;

static_assert(sizeof(rt::IOCompletion) == sizeof(ls_io_completion), "IOCompletion layout");
static_assert(sizeof(rt::IOBackend) == sizeof(ls_io_backend), "IOBackend layout");
static_assert(sizeof(rt::ComputeBackend) == sizeof(ls_compute_backend), "ComputeBackend layout");

static uint64_t now_ns() {
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return uint64_t(t.tv_sec) * 1000000000ull + uint64_t(t.tv_nsec);
}

#define CHECK(x)                                                                            \
    do {                                                                                    \
        const long _r = long(x);                                                            \
        if (_r) {                                                                           \
            std::fprintf(stderr, "%s:%d: %s -> %ld\n", __FILE__, __LINE__, #x, _r);         \
            std::exit(2);                                                                   \
        }                                                                                   \
    } while (0)

static std::vector<char> slurp(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) {
        std::fprintf(stderr, "cannot read %s\n", path.c_str());
        std::exit(2);
    }
    return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

static std::vector<int32_t> ids_line(std::istream& in) {
    std::string line;
    std::getline(in, line);
    std::istringstream s(line);
    std::vector<int32_t> v;
    int32_t x;
    while (s >> x) v.push_back(x);
    return v;
}

int main(int argc, char** argv) {
    if (argc != 9) {
        std::fprintf(stderr, "usage: %s DIR H G N QD DELAY_US CANDIDATE STEPS\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    const uint32_t H = uint32_t(std::atoi(argv[2])), G = uint32_t(std::atoi(argv[3])), N = uint32_t(std::atoi(argv[4]));
    const uint32_t qd = uint32_t(std::atoi(argv[5]));
    const float delay_us = float(std::atof(argv[6]));
    const int candidate = std::atoi(argv[7]), steps = std::atoi(argv[8]);
    const uint64_t group_bytes = uint64_t(G) * 3 * H / 2;
    const char* basic_env = std::getenv("LS_DRIVER_BASIC");
    const bool basic = basic_env && basic_env[0] == '1';

    const std::vector<char> packed = slurp(dir + "/packed.bin"), scales = slurp(dir + "/scales.bin"),
                            x = slurp(dir + "/x.bin");
    std::ifstream pf(dir + "/plan.txt");
    const std::vector<int32_t> p0 = ids_line(pf), p1 = ids_line(pf), fin = ids_line(pf);
    if (packed.size() != N * group_bytes || x.size() != 2 * H || fin.empty()) {
        std::fprintf(stderr, "input sizes\n");
        return 2;
    }

    const char* blocking_env = std::getenv("LS_DRIVER_BLOCKING_SYNC");
    if (blocking_env && blocking_env[0] == '1') CHECK(cudaSetDeviceFlags(cudaDeviceScheduleBlockingSync));
    CHECK(cudaSetDevice(0));
    // weights in pinned host memory; staging, scales, x and y on the device
    void* host = nullptr;
    CHECK(cudaHostAlloc(&host, packed.size(), cudaHostAllocDefault));
    std::memcpy(host, packed.data(), packed.size());
    void *staging = nullptr, *dscales = nullptr, *dx = nullptr, *dy = nullptr;
    CHECK(cudaMalloc(&staging, packed.size()));
    CHECK(cudaMemset(staging, 0, packed.size()));
    CHECK(cudaMalloc(&dscales, scales.size()));
    CHECK(cudaMemcpy(dscales, scales.data(), scales.size(), cudaMemcpyHostToDevice));
    CHECK(cudaMalloc(&dx, x.size()));
    CHECK(cudaMemcpy(dx, x.data(), x.size(), cudaMemcpyHostToDevice));
    CHECK(cudaMalloc(&dy, 2 * H));
    // queue storage the GPU reads with system-scope loads: mapped pinned memory
    rt::ExecDesc* desc = nullptr;
    uint32_t* ready = nullptr;
    rt::QueueControl* control = nullptr;
    CHECK(cudaHostAlloc(&desc, N * sizeof(rt::ExecDesc), cudaHostAllocMapped));
    CHECK(cudaHostAlloc(&ready, N * sizeof(uint32_t), cudaHostAllocMapped));
    CHECK(cudaHostAlloc(&control, sizeof(rt::QueueControl), cudaHostAllocMapped));
    std::memset(static_cast<void*>(control), 0, sizeof(rt::QueueControl));
    std::vector<uint32_t> io_states(N + 1, 0);

    // compute backend: one layer, the LUT pins the candidate (4/8/16/32 CTAs or one per SM)
    const uint8_t lut[1] = {uint8_t(candidate)};
    void* backend = ls_b200_create_table(lut, 1, 1);
    ls_b200_geometry geo{H, G, N, 1, 0, N, N, 2000000, 1e-5f};
    CHECK(ls_b200_configure(backend, &geo));
    ls_b200_layer_args bound{};
    bound.cache = static_cast<const uint8_t*>(staging);
    bound.staging = static_cast<const uint8_t*>(staging);
    bound.scales = dscales;
    bound.candidate = -1;
    // optional phase stamps of the kernel (LS_DRIVER_TRACE=1): per CTA and per layer
    const char* trace_env = std::getenv("LS_DRIVER_TRACE");
    const bool tracing = trace_env && trace_env[0] == '1';
    const size_t trace_words = 148 * LS_B200_TRACE_WORDS + 148 * LS_B200_LAYER_TRACE_WORDS +
                               4 * LS_B200_PIECE_TRACE_PIECES * 4;
    uint64_t* dtrace = nullptr;
    if (tracing) {
        CHECK(cudaMalloc(&dtrace, trace_words * 8));
        CHECK(cudaMemset(dtrace, 0, trace_words * 8));
        bound.trace = dtrace;
    }
    CHECK(ls_b200_set_buffers(backend, &bound));
    ls_b200_set_state(backend, 0, 0);
    ls_compute_backend cview{};
    CHECK(ls_b200_view(backend, &cview));

    // streaming IO backend over the pinned weights
    std::vector<uint64_t> offsets(N);
    for (uint32_t g = 0; g < N; ++g) offsets[g] = g * group_bytes;
    ls_b200_stream_config sc{host, offsets.data(), staging, group_bytes, group_bytes, io_states.data(),
                             N, qd, 0, delay_us, 20240601ull};
    void* engine = ls_b200_stream_create(&sc);
    if (!engine) {
        std::fprintf(stderr, "ls_b200_stream_create: errno %d\n", errno);
        return 2;
    }
    ls_io_backend iview{};
    CHECK(ls_b200_stream_view(engine, &iview));

    // the reference runtime, unmodified
    rt::ManagerConfig mc{};
    mc.group_count = N;
    mc.qd = qd;
    mc.group_bytes = group_bytes;
    mc.staging_stride = group_bytes;
    mc.mode = rt::ConsumerMode::Progressive;
    std::memcpy(&mc.io_backend, &iview, sizeof(iview));
    rt::ComputeBackend cb;
    std::memcpy(&cb, &cview, sizeof(cview));
    rt::Runtime runtime(mc, cb, 1);

    std::vector<rt::GroupLayout> layout(N);
    std::vector<rt::SlotId> cache_slots(N, -1);
    for (uint32_t g = 0; g < N; ++g) layout[g] = {g, g, offsets[g], uint32_t(group_bytes)};
    rt::LayerStorage storage{};
    storage.layout = {layout.data(), layout.size()};
    storage.cache_slots = cache_slots.data();
    storage.staging = staging;
    storage.io_states = io_states.data();
    storage.queue = {desc, ready, control, N};
    storage.layout_generation = 1;

    cudaStream_t stream;
    CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    double sum_step = 0, sum_tail = 0, sum_gbs = 0, sum_io = 0, sum_copy = 0;
    uint64_t bytes = 0, requests = 0;
    int measured = 0;
    for (int s = 0; s < steps; ++s) {
        rt::LayerStep step;
        const uint64_t t0 = now_ns();
        CHECK(runtime.begin_layer(0, storage, &step));
        CHECK(step.update_prediction({p0.data(), p0.size()}));
        if (basic) {
            // the reference's basic mode: finalize, wait for the reads, then launch
            CHECK(step.update_prediction({p1.data(), p1.size()}));
            CHECK(step.finalize({fin.data(), fin.size()}));
            CHECK(runtime.weights(0).wait_io(5000));
            CHECK(step.enqueue_compute(dx, dy, stream));
        } else {
            CHECK(step.enqueue_compute(dx, dy, stream));
            CHECK(step.update_prediction({p1.data(), p1.size()}));
            CHECK(step.finalize({fin.data(), fin.size()}));
        }
        CHECK(cudaStreamSynchronize(stream));
        const uint64_t t1 = now_ns();
        uint32_t status[4] = {0, 0, 0, 0};
        CHECK(ls_b200_status(backend, status, 4));
        if (status[0]) {
            std::fprintf(stderr, "device status %u detail %u\n", status[0], status[2]);
            return 3;
        }
        ls_b200_stream_counters st{};
        CHECK(ls_b200_stream_stats(engine, &st));
        requests = runtime.weights(0).read_requests();
        CHECK(step.commit({nullptr, 0}));
        if (s > 0 || steps == 1) {
            const double io_ns = double(st.last_land_ns - st.first_issue_ns);
            sum_step += double(t1 - t0);
            sum_tail += double(t1 - st.last_land_ns);
            sum_io += io_ns;
            sum_gbs += io_ns > 0 ? double(st.bytes) / io_ns : 0.0;
            sum_copy += st.admissions ? double(st.copy_ns) / double(st.admissions) : 0.0;
            bytes = st.bytes;
            ++measured;
        }
    }
    if (tracing) {
        // stamps of the last step: per CTA, relative to the earliest entry (us)
        std::vector<uint64_t> tr(trace_words);
        CHECK(cudaMemcpy(tr.data(), dtrace, trace_words * 8, cudaMemcpyDeviceToHost));
        const char* names[8] = {"entry", "decided", "first", "pieces", "produced", "barrier", "reduced", "exit"};
        uint64_t t0 = ~0ull;
        for (int c = 0; c < 148; ++c)
            if (tr[c * 8] && tr[c * 8] < t0) t0 = tr[c * 8];
        for (int k = 0; k < 8; ++k) {
            std::vector<double> v;
            for (int c = 0; c < 148; ++c)
                if (tr[c * 8 + k]) v.push_back(double(tr[c * 8 + k] - t0) / 1e3);
            if (v.empty()) continue;
            std::sort(v.begin(), v.end());
            std::fprintf(stderr, "trace %-9s n=%3zu min %8.1f med %8.1f max %8.1f us\n", names[k], v.size(), v.front(),
                         v[v.size() / 2], v.back());
        }
    }
    std::vector<uint16_t> y(H);
    CHECK(cudaMemcpy(y.data(), dy, 2 * H, cudaMemcpyDeviceToHost));
    std::ofstream(dir + "/y.bin", std::ios::binary).write(reinterpret_cast<const char*>(y.data()), 2 * H);
    std::printf(
        "{\"candidate\": %d, \"queue_depth\": %u, \"delay_mean_us\": %.1f, \"steps\": %d, \"step_us\": %.2f, "
        "\"io_span_us\": %.2f, \"h2d_gbs\": %.3f, \"tail_after_last_landing_us\": %.2f, \"h2d_bytes\": %llu, "
        "\"read_requests\": %llu, \"final_groups\": %zu, \"copy_issue_to_land_us\": %.2f, \"mode\": \"%s\", "
        "\"host_cores\": %ld, \"blocking_sync\": %d}\n",
        candidate, qd, delay_us, measured, sum_step / measured / 1e3, sum_io / measured / 1e3, sum_gbs / measured,
        sum_tail / measured / 1e3, (unsigned long long)bytes, (unsigned long long)requests, fin.size(),
        sum_copy / measured / 1e3, basic ? "basic" : "progressive", sysconf(_SC_NPROCESSORS_ONLN),
        blocking_env && blocking_env[0] == '1' ? 1 : 0);
    CHECK(runtime.drain());
    ls_b200_stream_destroy(engine);
    ls_b200_destroy(backend);
    return 0;
}
