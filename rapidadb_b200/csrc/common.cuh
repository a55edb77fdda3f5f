// Shared helpers for the RapidaDB B200 kernels: status reporting, metric
// score algebra, orderable sort keys and bounded spin-waits.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "rapidadb_b200.h"

namespace rdb {

// ---------------------------------------------------------------- errors --

// Records a message for rdb_last_error() (thread-local) and returns `code`.
int set_error(int code, const char* fmt, ...);
void note_launch();
unsigned* host_words();

#define RDB_CHECK_ARG(cond, ...)                                   \
    do {                                                           \
        if (!(cond)) return ::rdb::set_error(RDB_ERR_INVALID, __VA_ARGS__); \
    } while (0)

// On failure the runtime's (non-sticky) last-error state is cleared, so a
// later launch check does not report this failure a second time.
#define RDB_CUDA_TRY(expr)                                                        \
    do {                                                                          \
        cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess) {                                                  \
            (void)cudaGetLastError();                                             \
            return ::rdb::set_error(RDB_ERR_CUDA, "%s: %s (%s:%d)", #expr,        \
                                    cudaGetErrorString(e_), __FILE__, __LINE__);  \
        }                                                                         \
    } while (0)

// After every kernel launch of the library (exactly one per launch site):
// reports a launch error, else counts the launch (rdb_launch_count).
#define RDB_LAUNCH_CHECK()                                                        \
    do {                                                                          \
        cudaError_t e_ = cudaGetLastError();                                      \
        if (e_ != cudaSuccess)                                                    \
            return ::rdb::set_error(RDB_ERR_CUDA, "kernel launch: %s (%s:%d)",    \
                                    cudaGetErrorString(e_), __FILE__, __LINE__);  \
        ::rdb::note_launch();                                                     \
    } while (0)

#define RDB_TRY(expr)              \
    do {                           \
        int s_ = (expr);           \
        if (s_ != RDB_OK) return s_; \
    } while (0)

int num_sms();
size_t elem_size(int dtype);
// |x_i|^2 over the first d columns of n rows with a stride of ld elements
int row_sqnorms_ld(int dtype, const void* x, int64_t n, int d, int64_t ld, float* out, cudaStream_t s);

// Optional CUDA-event timing of selected kernel launches (rdb_timing_*):
// when the launch's tag is enabled, timing_begin records a start event on the
// launching stream and returns the stop event to record after the launch
// (nullptr when timing is off).
enum TimingTag : int {
    TIMING_FLAT_SCAN = 1,      // main pass of rdb_flat_search
    TIMING_IVF_SCAN = 2,       // rdb_ivf_flat_scan list scan
    TIMING_PQ_SCAN = 4,        // rdb_ivfpq_scan list scan
    TIMING_KMEANS_ASSIGN = 8,  // rdb_kmeans_assign scan
    TIMING_KMEANS_UPDATE = 16, // rdb_kmeans_update segment sums
    TIMING_FLAT_PREP = 32,     // rdb_flat_search per-query values
    TIMING_FLAT_SAMPLE = 64,   // rdb_flat_search sample pass + threshold select
    TIMING_FLAT_SELECT = 128,  // rdb_flat_search candidate select
    TIMING_FLAT_REPAIR = 256,  // rdb_flat_search overflow repair (scan + select; idle launches when none)
};
int timing_begin(int tag, cudaStream_t s, cudaEvent_t* stop);

// Device status word: kernels that give up on a bounded wait OR in a code here
// instead of hanging; the host reads it with read_device_status().
enum DeviceStatus : unsigned {
    DEV_OK = 0,
    DEV_TIMEOUT_PRODUCER = 1u << 0,
    DEV_TIMEOUT_MMA = 1u << 1,
    DEV_TIMEOUT_EPILOGUE = 1u << 2,
    DEV_OVERFLOW = 1u << 3,
    DEV_TIMEOUT_SIMT = 1u << 4,  // TMA-fed CUDA-core scan
    DEV_TIMEOUT_PROBE = 1u << 5,  // rdb_probe_bounded_wait
    DEV_TIMEOUT_PEER = 1u << 6,   // rdb_peer_gather: another rank did not signal in time
};
unsigned* device_status_word();  // per-device, zero-initialised
// Per-device word in mapped pinned host memory (device address) that the
// flat-search repair kernel copies a nonzero status word into, so the host
// can see it without synchronising; status_mirror_host() is its host address.
unsigned* status_mirror_device();
volatile unsigned* status_mirror_host();
// Test probe of the bounded mbarrier wait (flat_tc.cu).
int launch_wait_probe(uint64_t limit_ns, unsigned* out_waited_out, cudaStream_t s);
// Load kernels into the current context ahead of use (simt.cu, ivf.cu).
int norms_preload();
int ivf_flat_scan_preload();

// ------------------------------------------------------- score algebra --
//
// Every metric's final score is a function of the raw dot product <q, x> and
// two per-vector scalars (the reference formulas, csrc/kernels/distance.cu):
//   L2      : qv + xv - 2 dot          qv = |q|^2,  xv = |x|^2
//   DOT     : dot
//   COSINE  : d >  128: dot / (qv xv + 1e-8)      qv = sqrt|q|^2,  xv = sqrt|x|^2
//             d <= 128: dot / (qv xv)             qv = sqrt(|q|^2 + 1e-8), ...
// "xv" is the per-row value the index stores beside each row.

__host__ __device__ inline bool metric_largest(int metric) { return metric != RDB_METRIC_L2; }

__host__ __device__ inline float vec_value(int metric, int cos_small, float sq) {
    if (metric == RDB_METRIC_L2) return sq;
    if (metric == RDB_METRIC_COSINE) return cos_small ? sqrtf(sq + 1e-8f) : sqrtf(sq);
    return 0.f;
}

__device__ __forceinline__ float final_score(int metric, int cos_small, float dot, float qv,
                                             float xv) {
    if (metric == RDB_METRIC_L2) return fmaxf(qv + xv - 2.f * dot, 0.f);
    if (metric == RDB_METRIC_COSINE) return cos_small ? dot / (qv * xv) : dot / (qv * xv + 1e-8f);
    return dot;
}

// Filter coefficients: a row passes when dot >= A * xv + B.  Derived from a
// threshold `thr` in final-score units, with a relative slack of 2^-16 so
// that rounding can never reject a row whose final score reaches thr.
struct FilterCoef {
    float A, B;
};

__device__ __forceinline__ FilterCoef filter_coef(int metric, int cos_small, float thr, float qv) {
    FilterCoef f;
    const float eps = 1.52587890625e-05f;  // 2^-16
    if (metric == RDB_METRIC_L2) {
        // qv + xv - 2 dot <= thr  <=>  dot >= 0.5 xv + 0.5 (qv - thr)
        f.A = 0.5f;
        f.B = 0.5f * (qv - thr);
    } else if (metric == RDB_METRIC_COSINE) {
        f.A = thr * qv;
        f.B = cos_small ? 0.f : thr * 1e-8f;
    } else {
        f.A = 0.f;
        f.B = thr;
    }
    f.A -= fabsf(f.A) * eps;  // xv >= 0, so lowering A lowers the bound
    f.B -= fabsf(f.B) * eps + 1e-30f;
    if (!(thr == thr) || isinf(thr)) {  // "accept all"
        f.A = 0.f;
        f.B = -INFINITY;
    }
    return f;
}

// ------------------------------------------------------------- bit casts --

__host__ __device__ inline uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}

__host__ __device__ inline float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

// ------------------------------------------------------------- sort keys --
// 32-bit key, ascending = better.  Ties are broken by the row index in the
// low half of a 64-bit key, so every key is unique.

__host__ __device__ inline uint32_t float_asc_key(float f) {
    uint32_t u = f2u(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__host__ __device__ inline float asc_key_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return u2f(u);
}

__host__ __device__ inline uint32_t score_key(float s, bool largest) {
    uint32_t k = float_asc_key(s);
    return largest ? ~k : k;
}

__host__ __device__ inline float key_score(uint32_t k, bool largest) {
    return asc_key_float(largest ? ~k : k);
}

// ------------------------------------------------- paired fp32 (sm_100) --
//
// Two fp32 lanes in one 64-bit register: one fma.rn.f32x2 / mul.rn.f32x2
// instruction does two independent, individually rounded operations, so the
// results equal two scalar fmaf / multiplications.

__device__ __forceinline__ uint64_t pack2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}


// --------------------------------------------------------- spin waits --

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Upper bound on any single pipeline wait: a healthy wait lasts microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

}  // namespace rdb
