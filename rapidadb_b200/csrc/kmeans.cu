// k-means kernels: GEMM-fused assignment and an atomic-free update.
//
// Replaces the reference's naive Lloyd kernels (csrc/kernels/kmeans.cu:11-45
// assign, :48-94 update), which have no host launcher there.
//
// assign  - points are the "queries" and centroids the "rows" of the fused
//           scan in ARGMIN mode: fp16 / bf16 on tcgen05 (argmin of
//           |c|^2 - 2 x.c fused into the epilogue), fp32 on CUDA cores; the
//           per-split winners are reduced to (label, squared distance) with
//           ties to the lower centroid, as the reference's strict '<'.
//           rdb_assign_exact instead sums sum (x - c)^2 sequentially with one
//           fused multiply-add per element -- the reference assign arithmetic
//           bit for bit -- which the IVF indices use for list assignment.
// update  - a stable counting sort of point ids by label (block histograms ->
//           offsets -> per-block stable scatter through a shared-memory
//           bitonic sort), then one CTA per centroid sums its points in
//           ascending point order.  No floating-point atomics: the sums are
//           deterministic, and the [K, d] sums + [K] counts are what a
//           multi-GPU caller all-reduces before rdb_kmeans_finalize.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "scan.cuh"
#include "sort.cuh"

namespace rdb {
namespace {

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }


template <typename T>
__device__ __forceinline__ float ld_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_f<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}

// winners of nsplit splits -> label, squared distance (ties: lower centroid)
__global__ void argmin_reduce_kernel(const unsigned long long* best, int nsplit, int64_t n, int32_t* labels,
                                     float* sqdist) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    unsigned long long b = ~0ull;
    for (int s = 0; s < nsplit; ++s) b = min(b, best[(int64_t)s * n + i]);
    labels[i] = (int32_t)(uint32_t)b;
    if (sqdist) sqdist[i] = asc_key_float((uint32_t)(b >> 32));
}

// one CTA per centroid: sums of its points in ascending point order
template <typename T>
__global__ void segment_sum_kernel(const T* __restrict__ x, int64_t ldx, int d, const int64_t* __restrict__ perm,
                                   const int64_t* __restrict__ seg_start, float* __restrict__ sums) {
    const int c = blockIdx.x;
    const int64_t j0 = seg_start[c], j1 = seg_start[c + 1];
    for (int t0 = blockIdx.y * blockDim.x; t0 < d; t0 += gridDim.y * blockDim.x) {
        const int t = t0 + threadIdx.x;
        float acc0 = 0.f, acc1 = 0.f;
        int64_t j = j0;
        if (t < d) {
            for (; j + 1 < j1; j += 2) {
                acc0 += ld_f<T>(x, perm[j] * ldx + t);
                acc1 += ld_f<T>(x, perm[j + 1] * ldx + t);
            }
            if (j < j1) acc0 += ld_f<T>(x, perm[j] * ldx + t);
            sums[(int64_t)c * d + t] = acc0 + acc1;
        }
    }
}

__global__ void finalize_kernel(const float* __restrict__ sums, const int64_t* __restrict__ counts, int K, int d,
                                float* __restrict__ centroids) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)K * d) return;
    const int c = (int)(i / d);
    if (counts[c] > 0) centroids[i] = sums[i] / (float)counts[c];
}

size_t update_ws_bytes(int64_t n, int K) {
    return align_up(label_sort_workspace(n, K), 256) + align_up(sizeof(int64_t) * (K + 1), 256) +
           align_up(sizeof(int64_t) * (size_t)std::max<int64_t>(n, 1), 256);
}

bool tc_ok_layout(int dtype, const void* a, int64_t lda, const void* b, int64_t ldb, int d) {
    if (dtype != RDB_F16 && dtype != RDB_BF16) return false;
    if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15)) return false;
    return (lda * 2) % 16 == 0 && (ldb * 2) % 16 == 0 && d >= 8;
}

int assign_impl(int dtype, const void* x, int64_t n, int64_t ldx, int d, const void* c, int K, int64_t ldc,
                const float* c_sq, int exact, int32_t* labels, float* sqdist, void* ws, size_t ws_bytes,
                cudaStream_t s) {
    const bool tc = !exact && tc_ok_layout(dtype, x, ldx, c, ldc, d);
    const int qtile = tc ? (tc_use_pair(n) ? 2 * kTcQueries : kTcQueries) : kSimtQueries;
    const int rtile = tc ? kTcRows : kSimtRows;
    const int64_t nqb = (n + qtile - 1) / qtile;
    const int64_t ntiles = (K + rtile - 1) / rtile;
    const int64_t target = tc ? (tc_use_pair(n) ? num_sms() / 2 : num_sms()) : 2LL * num_sms();
    int64_t nsplit = std::max<int64_t>(1, std::min<int64_t>(target / std::max<int64_t>(nqb, 1), ntiles));
    const int64_t rps = (ntiles + nsplit - 1) / nsplit * rtile;
    nsplit = (K + rps - 1) / rps;
    const size_t need = align_up(sizeof(float) * n, 256) + sizeof(unsigned long long) * (size_t)nsplit * n;
    if (ws_bytes < need) return set_error(RDB_ERR_WORKSPACE, "workspace too small: %zu bytes, need %zu", ws_bytes, need);
    float* qv = static_cast<float*>(ws);
    unsigned long long* best =
        reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + align_up(sizeof(float) * n, 256));
    // |x|^2 of each point (row stride ldx)
    RDB_TRY(row_sqnorms_ld(dtype, x, n, d, ldx, qv, s));
    ScanArgs a = {};
    a.metric = RDB_METRIC_L2;
    a.dtype = dtype;
    a.q = x;
    a.nq = n;
    a.ldq = ldx;
    a.x = c;
    a.n = K;
    a.ldx = ldc;
    a.row_step = 1;
    a.d = d;
    a.qv = qv;
    a.xv = c_sq;
    a.nsplit = (int)nsplit;
    a.rows_per_split = rps;
    a.best = best;
    cudaEvent_t stop_ev;
    RDB_TRY(timing_begin(TIMING_KMEANS_ASSIGN, s, &stop_ev));
    if (tc) {
        RDB_TRY(launch_scan_tc(a, SCAN_ARGMIN, s));
    } else if (exact) {
        RDB_TRY(launch_scan_simt(a, SCAN_ARGMIN_EXACT, s));
    } else {
        RDB_TRY(launch_scan_simt(a, SCAN_ARGMIN, s));
    }
    if (stop_ev) RDB_CUDA_TRY(cudaEventRecord(stop_ev, s));
    argmin_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(best, (int)nsplit, n, labels, sqdist);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

size_t assign_ws(int64_t n, int K, int dtype, int exact) {
    const bool tc_possible = !exact && (dtype == RDB_F16 || dtype == RDB_BF16);
    const int rtile = tc_possible ? kTcRows : kSimtRows;
    const int64_t ntiles = (K + rtile - 1) / rtile;
    // upper bound on the split count of any plan: one split per row tile, at most 2 per SM
    const int64_t nsplit = std::min<int64_t>(ntiles, 2LL * num_sms());
    return align_up(sizeof(float) * n, 256) + sizeof(unsigned long long) * (size_t)nsplit * n + 256;
}

}  // namespace
}  // namespace rdb

using namespace rdb;

extern "C" {

size_t rdb_kmeans_assign_workspace(int dtype, int64_t n, int K, int d) {
    (void)d;
    return assign_ws(n, K, dtype, 0);
}

int rdb_kmeans_assign(int dtype, const void* x, int64_t n, int64_t ldx, int d, const void* centroids, int K,
                      int64_t ldc, const float* c_sqnorms, int32_t* labels, float* sqdist, void* ws,
                      size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(elem_size(dtype) != 0, "unknown dtype %d", dtype);
    RDB_CHECK_ARG(n >= 0 && d >= 1 && K >= 1, "bad shape");
    RDB_CHECK_ARG(ldx >= d && ldc >= d, "row strides must be >= d");
    RDB_CHECK_ARG(K < (1LL << 31), "too many centroids");
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(x && centroids && c_sqnorms && labels && ws, "NULL pointer");
    return assign_impl(dtype, x, n, ldx, d, centroids, K, ldc, c_sqnorms, 0, labels, sqdist, ws, ws_bytes,
                       static_cast<cudaStream_t>(stream));
}

size_t rdb_assign_exact_workspace(int64_t n, int K, int d) {
    (void)d;
    return assign_ws(n, K, RDB_F32, 1);
}

int rdb_assign_exact(const float* x, int64_t n, int64_t ldx, int d, const float* centroids, int K, int64_t ldc,
                     int32_t* labels, float* sqdist, void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(n >= 0 && d >= 1 && K >= 1, "bad shape");
    RDB_CHECK_ARG(ldx >= d && ldc >= d, "row strides must be >= d");
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(x && centroids && labels && ws, "NULL pointer");
    // the exact kernel ignores per-row values; pass the centroids as their own
    // (unused) value array to keep the argument checks uniform
    return assign_impl(RDB_F32, x, n, ldx, d, centroids, K, ldc, centroids, 1, labels, sqdist, ws, ws_bytes,
                       static_cast<cudaStream_t>(stream));
}

size_t rdb_kmeans_update_workspace(int64_t n, int K) { return update_ws_bytes(n, K); }

int rdb_kmeans_update(int dtype, const void* x, int64_t n, int64_t ldx, int d, const int32_t* labels, int K,
                      float* sums, int64_t* counts, void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(elem_size(dtype) != 0, "unknown dtype %d", dtype);
    RDB_CHECK_ARG(n >= 0 && d >= 1 && K >= 1, "bad shape");
    RDB_CHECK_ARG(K <= kMaxLabels, "at most %d clusters", kMaxLabels);
    RDB_CHECK_ARG(sums && counts, "NULL pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t need = update_ws_bytes(n, K);
    if (ws_bytes < need) return set_error(RDB_ERR_WORKSPACE, "workspace too small: %zu < %zu", ws_bytes, need);
    if (n == 0) {
        RDB_CUDA_TRY(cudaMemsetAsync(sums, 0, sizeof(float) * (size_t)K * d, s));
        RDB_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int64_t) * K, s));
        return RDB_OK;
    }
    RDB_CHECK_ARG(x && labels && ws, "NULL pointer");
    char* base = static_cast<char*>(ws);
    const size_t sort_b = align_up(label_sort_workspace(n, K), 256);
    int64_t* seg = reinterpret_cast<int64_t*>(base + sort_b);
    int64_t* perm = reinterpret_cast<int64_t*>(base + sort_b + align_up(sizeof(int64_t) * (K + 1), 256));
    RDB_TRY(label_sort(labels, n, K, seg, perm, counts, base, sort_b, s));
    const int threads = d >= 256 ? 256 : ((d + 31) / 32) * 32;
    dim3 grid(K, 1);
    cudaEvent_t stop_ev;
    RDB_TRY(timing_begin(TIMING_KMEANS_UPDATE, s, &stop_ev));
    switch (dtype) {
        case RDB_F32: segment_sum_kernel<float><<<grid, threads, 0, s>>>((const float*)x, ldx, d, perm, seg, sums); break;
        case RDB_F16: segment_sum_kernel<__half><<<grid, threads, 0, s>>>((const __half*)x, ldx, d, perm, seg, sums); break;
        default:
            segment_sum_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>((const __nv_bfloat16*)x, ldx, d, perm, seg, sums);
    }
    RDB_LAUNCH_CHECK();
    if (stop_ev) RDB_CUDA_TRY(cudaEventRecord(stop_ev, s));
    return RDB_OK;
}

int rdb_kmeans_finalize(const float* sums, const int64_t* counts, int K, int d, float* centroids, void* stream) {
    RDB_CHECK_ARG(K >= 1 && d >= 1, "bad shape");
    RDB_CHECK_ARG(sums && counts && centroids, "NULL pointer");
    const int64_t tot = (int64_t)K * d;
    finalize_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(sums, counts, K, d,
                                                                                                   centroids);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // extern "C"
