// C-ABI plumbing: thread-local error messages, the per-device status word
// that bounded device waits report into, and small shared helpers.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"

namespace rdb {

static thread_local char g_err[1024] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int num_sms() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (v <= 0) v = 148;
    if (dev >= 0 && dev < 64) cached[dev] = v;
    return v;
}

size_t elem_size(int dtype) {
    switch (dtype) {
        case RDB_F32: return 4;
        case RDB_F16: return 2;
        case RDB_BF16: return 2;
        default: return 0;
    }
}

// One zero-initialised status word per device, allocated on first use.
unsigned* device_status_word() {
    static std::mutex mu;
    static unsigned* words[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!words[dev]) {
        unsigned* p = nullptr;
        if (cudaMalloc(&p, sizeof(unsigned)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(unsigned)) != cudaSuccess) return nullptr;
        words[dev] = p;
    }
    return words[dev];
}

// One word of mapped pinned host memory per device (allocated on first use,
// kept until exit): kernels copy a nonzero status word into it, the host reads
// it without synchronising.
struct Mirror {
    volatile unsigned* host = nullptr;
    unsigned* dev = nullptr;
};
static Mirror* mirror_of_current() {
    static std::mutex mu;
    static Mirror mirrors[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    Mirror& m = mirrors[dev];
    if (!m.host) {
        void* h = nullptr;
        if (cudaHostAlloc(&h, sizeof(unsigned), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        void* d = nullptr;
        if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
            cudaGetLastError();
            cudaFreeHost(h);
            return nullptr;
        }
        *static_cast<volatile unsigned*>(h) = 0u;
        m.host = static_cast<volatile unsigned*>(h);
        m.dev = static_cast<unsigned*>(d);
    }
    return &m;
}

unsigned* status_mirror_device() {
    Mirror* m = mirror_of_current();
    return m ? m->dev : nullptr;
}

volatile unsigned* status_mirror_host() {
    Mirror* m = mirror_of_current();
    return m ? m->host : nullptr;
}

// Four pinned host words per host thread (allocated on first use, kept until
// exit) for asynchronous device-to-host reads of flags.
unsigned* host_words() {
    static thread_local unsigned* words = nullptr;
    if (!words) {
        void* p = nullptr;
        if (cudaMallocHost(&p, 4 * sizeof(unsigned)) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        words = static_cast<unsigned*>(p);
    }
    return words;
}

struct TimedLaunch {
    cudaEvent_t start, stop;
    int tag;
};

struct Timing {
    int mask = 0;
    std::vector<TimedLaunch> ev;
    size_t used = 0;
    std::mutex mu;
};
static Timing g_timing;

int timing_begin(int tag, cudaStream_t s, cudaEvent_t* stop) {
    *stop = nullptr;
    if (!(g_timing.mask & tag)) return RDB_OK;
    std::lock_guard<std::mutex> lock(g_timing.mu);
    if (g_timing.used == g_timing.ev.size()) {
        cudaEvent_t a, b;
        RDB_CUDA_TRY(cudaEventCreate(&a));
        RDB_CUDA_TRY(cudaEventCreate(&b));
        g_timing.ev.push_back({a, b, 0});
    }
    auto& p = g_timing.ev[g_timing.used++];
    p.tag = tag;
    RDB_CUDA_TRY(cudaEventRecord(p.start, s));
    *stop = p.stop;
    return RDB_OK;
}

static int timing_sum(int mask, double* total_ms, int* launches) {
    double tot = 0.0;
    int n = 0;
    for (size_t i = 0; i < g_timing.used; ++i) {
        if (!(g_timing.ev[i].tag & mask)) continue;
        RDB_CUDA_TRY(cudaEventSynchronize(g_timing.ev[i].stop));
        float ms = 0.f;
        RDB_CUDA_TRY(cudaEventElapsedTime(&ms, g_timing.ev[i].start, g_timing.ev[i].stop));
        tot += ms;
        ++n;
    }
    *total_ms = tot;
    *launches = n;
    return RDB_OK;
}

}  // namespace rdb

extern "C" {

int rdb_timing_enable(int mask) {
    std::lock_guard<std::mutex> lock(rdb::g_timing.mu);
    rdb::g_timing.mask = mask;
    rdb::g_timing.used = 0;
    // the event pairs are created here, before the launches that record them,
    // so that no event creation (a driver call that can stall behind other
    // driver work) falls between the timed launches; more are created on demand
    constexpr size_t kReserve = 1024;
    while (mask && rdb::g_timing.ev.size() < kReserve) {
        cudaEvent_t a, b;
        RDB_CUDA_TRY(cudaEventCreate(&a));
        RDB_CUDA_TRY(cudaEventCreate(&b));
        rdb::g_timing.ev.push_back({a, b, 0});
    }
    return RDB_OK;
}

int rdb_timing_read(double* total_ms, int* launches, int reset) {
    RDB_CHECK_ARG(total_ms && launches, "NULL pointer");
    std::lock_guard<std::mutex> lock(rdb::g_timing.mu);
    RDB_TRY(rdb::timing_sum(~0, total_ms, launches));
    if (reset) rdb::g_timing.used = 0;
    return RDB_OK;
}

int rdb_timing_read_tags(int mask, double* total_ms, int* launches) {
    RDB_CHECK_ARG(total_ms && launches, "NULL pointer");
    std::lock_guard<std::mutex> lock(rdb::g_timing.mu);
    return rdb::timing_sum(mask, total_ms, launches);
}

const char* rdb_last_error(void) { return rdb::g_err; }

unsigned long long rdb_launch_count(void) { return rdb::g_launches.load(std::memory_order_relaxed); }

int rdb_version(void) { return 200; }  // 2.00: IVF scans take list_end

int rdb_device_status(unsigned* out_host, int clear) {
    RDB_CHECK_ARG(out_host != nullptr, "out_host is NULL");
    unsigned* w = rdb::device_status_word();
    if (!w) return rdb::set_error(RDB_ERR_CUDA, "cannot allocate the device status word");
    RDB_CUDA_TRY(cudaDeviceSynchronize());
    RDB_CUDA_TRY(cudaMemcpy(out_host, w, sizeof(unsigned), cudaMemcpyDeviceToHost));
    if (clear) {
        RDB_CUDA_TRY(cudaMemset(w, 0, sizeof(unsigned)));
        RDB_CUDA_TRY(cudaDeviceSynchronize());
        volatile unsigned* m = rdb::status_mirror_host();
        if (m) *m = 0u;
    }
    return RDB_OK;
}

int rdb_pending_status(unsigned* out_host) {
    RDB_CHECK_ARG(out_host != nullptr, "out_host is NULL");
    volatile unsigned* m = rdb::status_mirror_host();
    if (!m) return rdb::set_error(RDB_ERR_CUDA, "cannot allocate the host status word");
    *out_host = *m;
    return RDB_OK;
}

int rdb_probe_bounded_wait(unsigned long long limit_ns, void* stream) {
    RDB_CHECK_ARG(limit_ns >= 1000ull && limit_ns <= 1000000000ull, "limit_ns must be in [1 us, 1 s]");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned* host = rdb::host_words();
    if (!host) return rdb::set_error(RDB_ERR_CUDA, "cannot allocate pinned host words");
    unsigned* flag = nullptr;
    RDB_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&flag), sizeof(unsigned), s));
    int st = rdb::launch_wait_probe(limit_ns, flag, s);
    if (st == RDB_OK) {
        host[2] = 0;
        cudaError_t e = cudaMemcpyAsync(&host[2], flag, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) {
            cudaGetLastError();
            st = rdb::set_error(RDB_ERR_CUDA, "bounded-wait probe: %s", cudaGetErrorString(e));
        }
    }
    cudaFreeAsync(flag, s);
    cudaStreamSynchronize(s);
    if (st != RDB_OK) return st;
    if (host[2]) return rdb::set_error(RDB_ERR_TIMEOUT, "the probe's device wait ran out after %llu ns", limit_ns);
    return RDB_OK;
}

}  // extern "C"
