// Streaming IO engine: the IOBackend of include/leanstream/weight_manager.h:14-24
// for a discrete GPU. Logical groups live in pinned host memory; the worker
// copies the groups a WeightManager asks for into HBM staging (group g at
// staging + g * stride, the slot the reference engine uses,
// weight_manager.cpp:94) with one cudaMemcpyAsync per group on its own
// stream, in the priority order of the last update and then the committed
// final reads (the admission order of src/io/stream_io.cpp:62-73), at most
// `queue_depth` copies in flight and never preempting a started copy. When a
// copy's event has completed, the group's io_states word becomes READY
// (release) and the completion callback runs on the worker thread; the
// WeightManager then publishes the descriptor to the ExecutionQueue, from
// which the running kernel claims it (system-scope acquire).
//
// With a file source (the SSD leg of src/io/stream_io.cpp:75-148), an
// admitted group is first read from the file into its pinned host slot by a
// pool of reader threads (pread, O_DIRECT when the file system and the
// alignment allow it); the worker issues the group's copy once its read has
// returned. Reads and copies together are bounded by queue_depth.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <mutex>
#include <new>
#include <random>
#include <thread>
#include <vector>

#include "ls_internal.h"

static_assert(sizeof(ls_io_completion) == 24, "IOCompletion: epoch, group, slot, error, sequence");
static_assert(sizeof(ls_io_backend) == 8 * sizeof(void*), "IOBackend: context + seven entry points");
static_assert(sizeof(ls_group_span) == 16, "Span<GroupId>: pointer + size_t");

namespace lsb {
namespace {

uint64_t mono_ns() {
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return uint64_t(t.tv_sec) * 1000000000ull + uint64_t(t.tv_nsec);
}
uint32_t load_state(const uint32_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
void store_state(uint32_t* p, uint32_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

struct Inflight {
    int32_t id;
    uint32_t event;
    uint64_t issued;
};
struct Landed {
    int32_t id;
    uint64_t due;
};
struct ReadDone {
    int32_t id;
    uint32_t event;
    int error;
};

struct Engine {
    ls_b200_stream_config cfg{};
    std::vector<uint64_t> offsets;
    cudaStream_t stream = nullptr;
    std::vector<cudaEvent_t> events;
    std::vector<uint32_t> free_events;
    std::mutex m;
    std::condition_variable work, changed;
    std::thread worker;
    bool stop = false;
    // session state (under m)
    bool active = false, closing = false, consuming = false;
    uint32_t epoch = 0;
    ls_io_completion_fn callback = nullptr;
    void* callback_arg = nullptr;
    std::vector<int32_t> rank, committed, issue_log;
    std::vector<uint8_t> claimed, committed_bit;
    size_t cursor = 0, fallback = 0;
    std::deque<Inflight> inflight;
    std::vector<Landed> landed;
    // file source: reads waiting for a reader, reads in progress, returned reads
    int fd = -1;
    bool direct = false;
    uint64_t read_size = 0;  // bytes per read (group_bytes, rounded up to the alignment with O_DIRECT)
    std::vector<uint64_t> file_offsets;
    std::vector<std::thread> readers;
    std::condition_variable read_work;
    std::deque<std::pair<int32_t, uint32_t>> to_read;
    uint32_t reading = 0;
    std::vector<ReadDone> read_done;
    uint64_t sequence = 0;
    std::mt19937_64 rng;
    ls_b200_stream_counters stats{};

    uint32_t* states() const { return cfg.io_states; }
    bool terminal() const { return load_state(cfg.io_states + cfg.group_count) != 0; }

    int select() {
        while (cursor < rank.size()) {
            const int32_t id = rank[cursor++];
            if (!claimed[id]) return id;
        }
        if (consuming)
            while (fallback < committed.size()) {
                const int32_t id = committed[fallback++];
                if (!claimed[id]) return id;
            }
        return -1;
    }

    // A failed copy: the group and the session turn to ERROR; the callback
    // reports it (the WeightManager fails the ExecutionQueue).
    void fail(std::unique_lock<std::mutex>& l, int32_t id, int error) {
        store_state(states() + id, LS_IO_ERROR);
        uint32_t expected = 0;
        __atomic_compare_exchange_n(states() + cfg.group_count, &expected, uint32_t(error), false, __ATOMIC_RELEASE,
                                    __ATOMIC_RELAXED);
        if (!stats.error) stats.error = error;
        const ls_io_completion c{epoch, id, id, error, ++sequence};
        const ls_io_completion_fn fn = callback;
        void* arg = callback_arg;
        l.unlock();
        if (fn) fn(arg, &c);
        l.lock();
    }

    void run() {
        cudaSetDevice(cfg.device);
        std::exponential_distribution<double> expo(cfg.delay_mean_us > 0.f ? 1.0 / double(cfg.delay_mean_us) : 1.0);
        std::unique_lock<std::mutex> l(m);
        while (!stop) {
            bool progressed = false;
            // admissions
            while (active && !closing && !terminal() && !free_events.empty()) {
                const int id = select();
                if (id < 0) break;
                claimed[id] = 1;
                store_state(states() + id, LS_IO_INFLIGHT);
                issue_log.push_back(id);
                const uint32_t ev = free_events.back();
                free_events.pop_back();
                const uint64_t now = mono_ns();
                if (!stats.first_issue_ns) stats.first_issue_ns = now;
                ++stats.admissions;
                if (fd >= 0) {  // the read first; the copy when it returns
                    to_read.emplace_back(id, ev);
                    read_work.notify_one();
                    progressed = true;
                    continue;
                }
                cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(cfg.staging) + uint64_t(id) * cfg.staging_stride,
                                                static_cast<const uint8_t*>(cfg.host_base) + offsets[id],
                                                cfg.group_bytes, cudaMemcpyHostToDevice, stream);
                if (e == cudaSuccess) e = cudaEventRecord(events[ev], stream);
                if (e != cudaSuccess) {
                    free_events.push_back(ev);
                    fail(l, id, int(e));
                    continue;
                }
                inflight.push_back({id, ev, now});
                progressed = true;
            }
            // returned reads: copy the group to HBM
            for (const ReadDone& r : read_done) {
                progressed = true;
                if (r.error) {
                    free_events.push_back(r.event);
                    fail(l, r.id, r.error);
                    continue;
                }
                cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(cfg.staging) + uint64_t(r.id) * cfg.staging_stride,
                                                static_cast<const uint8_t*>(cfg.host_base) + offsets[r.id],
                                                cfg.group_bytes, cudaMemcpyHostToDevice, stream);
                if (e == cudaSuccess) e = cudaEventRecord(events[r.event], stream);
                if (e != cudaSuccess) {
                    free_events.push_back(r.event);
                    fail(l, r.id, int(e));
                    continue;
                }
                inflight.push_back({r.id, r.event, mono_ns()});
            }
            read_done.clear();
            // landings, in issue order (one stream)
            while (!inflight.empty()) {
                const cudaError_t q = cudaEventQuery(events[inflight.front().event]);
                if (q == cudaErrorNotReady) break;
                const Inflight f = inflight.front();
                inflight.pop_front();
                free_events.push_back(f.event);
                const uint64_t now = mono_ns();
                progressed = true;
                if (q != cudaSuccess) {
                    fail(l, f.id, int(q));
                    continue;
                }
                stats.bytes += cfg.group_bytes;
                stats.last_land_ns = now;
                stats.copy_ns += now - f.issued;
                const uint64_t delay = cfg.delay_mean_us > 0.f ? uint64_t(expo(rng) * 1000.0) : 0;
                landed.push_back({f.id, now + delay});
            }
            // publications that are due (all of them once the session closes)
            for (size_t i = 0; i < landed.size();) {
                if (!closing && landed[i].due > mono_ns()) {
                    ++i;
                    continue;
                }
                const int32_t id = landed[i].id;
                landed[i] = landed.back();
                landed.pop_back();
                store_state(states() + id, LS_IO_READY);
                ++stats.completions;
                const ls_io_completion c{epoch, id, id, 0, ++sequence};
                const ls_io_completion_fn fn = callback;
                void* arg = callback_arg;
                l.unlock();
                if (fn) fn(arg, &c);
                l.lock();
                progressed = true;
            }
            stats.outstanding = uint32_t(inflight.size() + to_read.size() + reading);
            if (progressed) {
                changed.notify_all();
                continue;
            }
            if (!inflight.empty() || !landed.empty()) {
                // copies or delayed publications pending: poll (microsecond scale)
                l.unlock();
                std::this_thread::yield();
                l.lock();
            } else {
                changed.notify_all();
                work.wait(l);
            }
        }
    }

    // Reader thread: pread of an admitted group into its host slot (EINTR and
    // short reads retried; a read that ends early is EIO).
    void read_loop() {
        std::unique_lock<std::mutex> l(m);
        for (;;) {
            read_work.wait(l, [&] { return stop || !to_read.empty(); });
            if (to_read.empty()) return;  // stop
            const auto [id, ev] = to_read.front();
            to_read.pop_front();
            ++reading;
            l.unlock();
            uint8_t* dst = static_cast<uint8_t*>(const_cast<void*>(cfg.host_base)) + offsets[id];
            const uint64_t t0 = mono_ns();
            uint64_t done = 0;
            int error = 0;
            while (done < read_size) {
                const ssize_t got = pread(fd, dst + done, read_size - done, off_t(file_offsets[id] + done));
                if (got < 0 && errno == EINTR) continue;
                if (got < 0) {
                    error = errno ? errno : EIO;
                    break;
                }
                if (got == 0) break;
                done += uint64_t(got);
            }
            if (!error && done < cfg.group_bytes) error = EIO;  // the file ends inside the group
            const uint64_t t1 = mono_ns();
            l.lock();
            --reading;
            stats.read_ns += t1 - t0;
            stats.read_bytes += done;
            read_done.push_back({id, ev, error});
            work.notify_one();
        }
    }

    // ------------------------------------------------------------ IOBackend
    int begin(ls_io_completion_fn fn, void* arg, uint32_t e) {
        std::lock_guard<std::mutex> g(m);
        if (active) return EBUSY;
        for (uint32_t i = 0; i <= cfg.group_count; ++i) store_state(states() + i, LS_IO_EMPTY);
        std::fill(claimed.begin(), claimed.end(), 0);
        std::fill(committed_bit.begin(), committed_bit.end(), 0);
        committed.clear();
        rank.clear();
        issue_log.clear();
        cursor = fallback = 0;
        consuming = closing = false;
        rng.seed(cfg.delay_seed ^ (uint64_t(e) * 0x9E3779B97F4A7C15ull));
        stats = ls_b200_stream_counters{};
        callback = fn;
        callback_arg = arg;
        epoch = e;
        active = true;
        return 0;
    }
    int install(ls_group_span ids, bool consume) {
        if (ids.size && !ids.data) return EINVAL;
        std::lock_guard<std::mutex> g(m);
        if (!active) return EINVAL;
        if (closing) return ESHUTDOWN;
        if (terminal()) return EIO;
        for (size_t i = 0; i < ids.size; ++i)
            if (ids.data[i] < 0 || uint32_t(ids.data[i]) >= cfg.group_count) return EINVAL;
        rank.assign(ids.data, ids.data + ids.size);
        cursor = 0;
        if (consume) {
            consuming = true;
            fallback = 0;
            for (size_t i = 0; i < ids.size; ++i)
                if (!committed_bit[ids.data[i]]) {
                    committed_bit[ids.data[i]] = 1;
                    committed.push_back(ids.data[i]);
                }
        }
        work.notify_one();
        return 0;
    }
    int retire() {
        std::unique_lock<std::mutex> l(m);
        if (!active) return EINVAL;
        closing = true;
        work.notify_one();
        changed.wait(l, [&] { return inflight.empty() && landed.empty() && to_read.empty() && !reading &&
                                     read_done.empty(); });
        active = false;
        return int(load_state(states() + cfg.group_count));
    }
    int wait(int timeout_ms) {
        std::unique_lock<std::mutex> l(m);
        const bool ok = changed.wait_for(l, std::chrono::milliseconds(timeout_ms), [&] {
            if (terminal()) return true;
            if (!consuming) return false;
            for (int32_t id : committed)
                if (load_state(states() + id) != LS_IO_READY) return false;
            return true;
        });
        return ok ? int(load_state(states() + cfg.group_count)) : ETIMEDOUT;
    }
};

int io_begin(void* ctx, ls_io_completion_fn fn, void* arg, uint32_t epoch) {
    return ctx ? static_cast<Engine*>(ctx)->begin(fn, arg, epoch) : EINVAL;
}
int io_update(void* ctx, ls_group_span ids) { return ctx ? static_cast<Engine*>(ctx)->install(ids, false) : EINVAL; }
int io_consume(void* ctx, ls_group_span ids) { return ctx ? static_cast<Engine*>(ctx)->install(ids, true) : EINVAL; }
int io_retire(void* ctx) { return ctx ? static_cast<Engine*>(ctx)->retire() : EINVAL; }
int32_t io_ready_slot(void* ctx, int32_t group) {
    // the staging slot of a group is its logical id
    const auto* e = static_cast<Engine*>(ctx);
    return (e && group >= 0 && uint32_t(group) < e->cfg.group_count) ? group : -1;
}
uint64_t io_requests(void* ctx) {
    auto* e = static_cast<Engine*>(ctx);
    if (!e) return 0;
    std::lock_guard<std::mutex> g(e->m);
    return e->stats.admissions;
}
int io_wait(void* ctx, int timeout_ms) { return ctx ? static_cast<Engine*>(ctx)->wait(timeout_ms) : EINVAL; }

}  // namespace
}  // namespace lsb

extern "C" {

void* ls_b200_stream_create(const ls_b200_stream_config* c) {
    using lsb::Engine;
    if (!c || !c->host_base || !c->host_offsets || !c->staging || !c->io_states || !c->group_count ||
        c->group_count > 0x7fffffffu || !c->queue_depth || c->queue_depth > 32 || !c->group_bytes ||
        c->group_bytes > c->staging_stride || !(c->delay_mean_us >= 0.f)) {
        errno = EINVAL;
        return nullptr;
    }
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || c->device < 0 || c->device >= devices) {
        errno = ENODEV;
        return nullptr;
    }
    Engine* e = new (std::nothrow) Engine();
    if (!e) {
        errno = ENOMEM;
        return nullptr;
    }
    e->cfg = *c;
    int previous = 0;
    cudaGetDevice(&previous);
    bool ok = cudaSetDevice(c->device) == cudaSuccess;
    try {
        e->offsets.assign(c->host_offsets, c->host_offsets + c->group_count);
        e->claimed.assign(c->group_count, 0);
        e->committed_bit.assign(c->group_count, 0);
        e->events.assign(c->queue_depth, nullptr);
        e->rank.reserve(c->group_count);
        e->committed.reserve(c->group_count);
        e->issue_log.reserve(c->group_count);
    } catch (...) {
        ok = false;
    }
    if (ok) ok = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) == cudaSuccess;
    for (uint32_t i = 0; ok && i < c->queue_depth; ++i) {
        ok = cudaEventCreateWithFlags(&e->events[i], cudaEventDisableTiming) == cudaSuccess;
        if (ok) e->free_events.push_back(i);
    }
    cudaSetDevice(previous);
    int open_error = 0;
    if (ok && c->file_path) {
        // SSD leg: O_DIRECT when asked for and every offset and host slot is
        // aligned (each read is then rounded up to the alignment), else
        // buffered reads of exactly group_bytes
        const uint64_t align = c->file_alignment ? c->file_alignment : 4096;
        bool aligned = c->file_offsets && (align & (align - 1)) == 0;
        try {
            if (c->file_offsets) e->file_offsets.assign(c->file_offsets, c->file_offsets + c->group_count);
        } catch (...) {
            ok = false;
        }
        for (uint32_t g = 0; ok && aligned && g < c->group_count; ++g)
            aligned = e->file_offsets[g] % align == 0 &&
                      (reinterpret_cast<uintptr_t>(c->host_base) + c->host_offsets[g]) % align == 0;
        int fd = -1;
        if (ok && c->file_offsets && c->o_direct && aligned) {
            fd = open(c->file_path, O_RDONLY | O_DIRECT);
            e->direct = fd >= 0;
        }
        if (ok && c->file_offsets && fd < 0) fd = open(c->file_path, O_RDONLY);
        if (fd < 0) {
            open_error = c->file_offsets ? errno : EINVAL;
            ok = false;
        }
        e->fd = fd;
        e->read_size = e->direct ? (c->group_bytes + align - 1) / align * align : c->group_bytes;
        const uint32_t n = c->read_workers ? std::min<uint32_t>(c->read_workers, 16) : 4;
        for (uint32_t i = 0; ok && i < n; ++i) {
            try {
                e->readers.emplace_back([e] { e->read_loop(); });
            } catch (...) {
                ok = false;
            }
        }
    }
    if (ok) {
        try {
            e->worker = std::thread([e] { e->run(); });
        } catch (...) {
            ok = false;
        }
    }
    if (!ok) {
        {
            std::lock_guard<std::mutex> g(e->m);
            e->stop = true;
            e->read_work.notify_all();
        }
        for (std::thread& t : e->readers) t.join();
        if (e->fd >= 0) close(e->fd);
        for (cudaEvent_t ev : e->events)
            if (ev) cudaEventDestroy(ev);
        if (e->stream) cudaStreamDestroy(e->stream);
        delete e;
        errno = open_error ? open_error : ENOMEM;
        return nullptr;
    }
    return e;
}

int ls_b200_stream_view(void* engine, ls_io_backend* out) {
    if (!engine || !out) return EINVAL;
    out->context = engine;
    out->begin = lsb::io_begin;
    out->update = lsb::io_update;
    out->consume = lsb::io_consume;
    out->retire = lsb::io_retire;
    out->ready_slot = lsb::io_ready_slot;
    out->requests = lsb::io_requests;
    out->wait = lsb::io_wait;
    return 0;
}

int ls_b200_stream_stats(void* engine, ls_b200_stream_counters* out) {
    if (!engine || !out) return EINVAL;
    auto* e = static_cast<lsb::Engine*>(engine);
    std::lock_guard<std::mutex> g(e->m);
    *out = e->stats;
    out->outstanding = uint32_t(e->inflight.size() + e->to_read.size() + e->reading);
    out->direct = e->direct ? 1u : 0u;
    return 0;
}

uint32_t ls_b200_stream_issue_log(void* engine, int32_t* out, uint32_t capacity) {
    if (!engine || (capacity && !out)) return 0;
    auto* e = static_cast<lsb::Engine*>(engine);
    std::lock_guard<std::mutex> g(e->m);
    const uint32_t n = uint32_t(std::min<size_t>(capacity, e->issue_log.size()));
    std::copy(e->issue_log.begin(), e->issue_log.begin() + n, out);
    return n;
}

void ls_b200_stream_destroy(void* engine) {
    if (!engine) return;
    auto* e = static_cast<lsb::Engine*>(engine);
    {
        std::unique_lock<std::mutex> l(e->m);
        e->closing = true;
        e->work.notify_all();
        e->changed.wait(l, [&] {
            return e->inflight.empty() && e->landed.empty() && e->to_read.empty() && !e->reading &&
                   e->read_done.empty();
        });
        e->stop = true;
        e->work.notify_all();
        e->read_work.notify_all();
    }
    e->worker.join();
    for (std::thread& t : e->readers) t.join();
    if (e->fd >= 0) close(e->fd);
    int previous = 0;
    cudaGetDevice(&previous);
    cudaSetDevice(e->cfg.device);
    for (cudaEvent_t ev : e->events) cudaEventDestroy(ev);
    cudaStreamDestroy(e->stream);
    cudaSetDevice(previous);
    delete e;
}

}  // extern "C"
