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

struct Timing {
    int mask = 0;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
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
        g_timing.ev.emplace_back(a, b);
    }
    auto& p = g_timing.ev[g_timing.used++];
    RDB_CUDA_TRY(cudaEventRecord(p.first, s));
    *stop = p.second;
    return RDB_OK;
}

}  // namespace rdb

extern "C" {

int rdb_timing_enable(int mask) {
    std::lock_guard<std::mutex> lock(rdb::g_timing.mu);
    rdb::g_timing.mask = mask;
    rdb::g_timing.used = 0;
    return RDB_OK;
}

int rdb_timing_read(double* total_ms, int* launches, int reset) {
    RDB_CHECK_ARG(total_ms && launches, "NULL pointer");
    std::lock_guard<std::mutex> lock(rdb::g_timing.mu);
    double tot = 0.0;
    for (size_t i = 0; i < rdb::g_timing.used; ++i) {
        RDB_CUDA_TRY(cudaEventSynchronize(rdb::g_timing.ev[i].second));
        float ms = 0.f;
        RDB_CUDA_TRY(cudaEventElapsedTime(&ms, rdb::g_timing.ev[i].first, rdb::g_timing.ev[i].second));
        tot += ms;
    }
    *total_ms = tot;
    *launches = static_cast<int>(rdb::g_timing.used);
    if (reset) rdb::g_timing.used = 0;
    return RDB_OK;
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
    if (clear) RDB_CUDA_TRY(cudaMemset(w, 0, sizeof(unsigned)));
    return RDB_OK;
}

}  // extern "C"
