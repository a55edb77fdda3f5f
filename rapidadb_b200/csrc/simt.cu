// CUDA-core kernels: row norms, the dense reference-formula distance matrix
// (the raw ops of csrc/kernels/distance.cu), and the fused fp32 scan used by
// flat search for fp32 storage.
//
// The scan tiles 32 queries x 256 rows per CTA (256 threads, 8 x 4 outputs per
// thread) over K chunks of 32 staged through shared memory; each CTA walks a
// contiguous split of rows so its per-query candidate counters stay private.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "scan.cuh"

namespace rdb {
namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// ------------------------------------------------------------ row norms --

template <typename T>
__global__ void row_sqnorms_kernel(const T* __restrict__ x, int64_t n, int d, int64_t ld,
                                   float* __restrict__ out) {
    int lane = threadIdx.x & 31;
    int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const T* p = x + row * ld;
    float acc = 0.f;
    for (int t = lane; t < d; t += 32) {
        float v = to_f<T>(p[t]);
        acc = fmaf(v, v, acc);
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[row] = acc;
}

__global__ void vec_values_kernel(int metric, int cos_small, const float* sq, int64_t n,
                                  float* out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = vec_value(metric, cos_small, sq[i]);
}

// --------------------------------------------------------------- scan --
//
// CTA tile: 32 queries x 256 rows, 256 threads, K chunks of 32 staged in
// shared memory (the next chunk is loaded into registers while the current
// one is consumed).  Warp w owns queries 8 (w mod 4) .. + 7 and rows
// 128 (w / 4) + lane + 32 j (j < 4): its query operands are shared-memory
// broadcasts (two 16-byte loads per k) and each lane loads 4 row values per
// k for 32 multiply-adds.

constexpr int BQ = kSimtQueries;  // 32
constexpr int BN = kSimtRows;     // 256
constexpr int BK = 32;
constexpr int NT = 256;
constexpr int XS = BN + 1;  // Xs row stride (conflict-free transposing stores)
static_assert(BQ == 32 && BN == 256, "thread mapping assumes 32 x 256 tiles");

// four consecutive elements (k .. k + 3 < kmax) as floats; vector loads when
// the caller knows the address is aligned
template <typename T>
__device__ __forceinline__ float4 load4(const T* p, bool vec, int nvalid) {
    if (vec && nvalid >= 4) {
        if constexpr (sizeof(T) == 4) {
            return __ldg(reinterpret_cast<const float4*>(p));
        } else {
            const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
            const T* e = reinterpret_cast<const T*>(&u);
            return make_float4(to_f<T>(e[0]), to_f<T>(e[1]), to_f<T>(e[2]), to_f<T>(e[3]));
        }
    }
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = i < nvalid ? to_f<T>(p[i]) : 0.f;
    return make_float4(v[0], v[1], v[2], v[3]);
}

template <typename T, int MODE, bool DIRECT_L2>
__global__ void __launch_bounds__(NT, 2) simt_scan_kernel(ScanArgs a) {
    __shared__ __align__(16) float Qs[BK][BQ];
    __shared__ float Xs[BK][XS];
    __shared__ float sA[BQ], sB[BQ], sQv[BQ];
    __shared__ int scnt[BQ];
    __shared__ unsigned long long sbest[BQ];

    const T* __restrict__ qp = static_cast<const T*>(a.q);
    const T* __restrict__ xp = static_cast<const T*>(a.x);
    const int split = blockIdx.x;
    // query blocks run along y, continuing in z past the 65535 limit of y
    const int64_t q0 = ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * BQ;
    if (q0 >= a.nq) return;
    const int64_t r_begin = (int64_t)split * a.rows_per_split;
    const int64_t r_end = min(a.n, r_begin + a.rows_per_split);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qg = (warp & 3) * 8;     // first query of this warp
    const int rb = (warp >> 2) * 128;  // first row (in the tile) of this warp
    const int64_t xstride = a.ldx * a.row_step;
    const bool vec_q = (reinterpret_cast<uintptr_t>(qp) % 16 == 0) && (a.ldq % 4 == 0);
    const bool vec_x = (reinterpret_cast<uintptr_t>(xp) % 16 == 0) && (xstride % 4 == 0);

    if (tid < BQ) {
        int64_t q = q0 + tid;
        float qv = (q < a.nq && a.qv) ? a.qv[q] : 0.f;
        float thr = (a.thr && q < a.nq) ? a.thr[q] : __int_as_float(0x7fc00000);
        FilterCoef f = filter_coef(a.metric, a.cos_small, thr, qv);
        sA[tid] = f.A;
        sB[tid] = f.B;
        sQv[tid] = qv;
        scnt[tid] = 0;
        sbest[tid] = ~0ull;
    }
    // ARGMIN: best (distance key, row) of each of this thread's 8 queries
    unsigned long long best[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) best[i] = ~0ull;

    // staging map: queries -> thread (query t / 8, k 4 (t mod 8) .. + 3);
    // rows -> thread (rows t / 8 + 32 i, same k)
    const int sq = tid >> 3, sk = (tid & 7) * 4;
    for (int64_t r0 = r_begin; r0 < r_end; r0 += BN) {
        float acc[8][4];
        float qsq[8], xsq[4];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qsq[i] = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) xsq[j] = 0.f;

        float4 pq, px[8];
        auto fetch = [&](int k0) {
            const int k = k0 + sk;
            const int nv = min(4, a.d - k);
            const int64_t q = q0 + sq;
            pq = (q < a.nq && nv > 0) ? load4<T>(qp + q * a.ldq + k, vec_q, nv) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int64_t r = r0 + sq + 32 * i;
                px[i] = (r < r_end && nv > 0) ? load4<T>(xp + r * xstride + k, vec_x, nv)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        fetch(0);
        for (int k0 = 0; k0 < a.d; k0 += BK) {
            __syncthreads();  // the previous chunk is consumed
            Qs[sk + 0][sq] = pq.x;
            Qs[sk + 1][sq] = pq.y;
            Qs[sk + 2][sq] = pq.z;
            Qs[sk + 3][sq] = pq.w;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                Xs[sk + 0][sq + 32 * i] = px[i].x;
                Xs[sk + 1][sq + 32 * i] = px[i].y;
                Xs[sk + 2][sq + 32 * i] = px[i].z;
                Xs[sk + 3][sq + 32 * i] = px[i].w;
            }
            __syncthreads();
            if (k0 + BK < a.d) fetch(k0 + BK);
#pragma unroll 4
            for (int kk = 0; kk < BK; ++kk) {
                const float4 a0 = *reinterpret_cast<const float4*>(&Qs[kk][qg]);
                const float4 a1 = *reinterpret_cast<const float4*>(&Qs[kk][qg + 4]);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                float bv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) bv[j] = Xs[kk][rb + lane + 32 * j];
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (DIRECT_L2) {
                            const float df = av[i] - bv[j];
                            acc[i][j] = fmaf(df, df, acc[i][j]);
                        } else {
                            acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                        }
                    }
                if (MODE == SCAN_DENSE && !DIRECT_L2 && a.metric == RDB_METRIC_COSINE) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) qsq[i] = fmaf(av[i], av[i], qsq[i]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) xsq[j] = fmaf(bv[j], bv[j], xsq[j]);
                }
            }
        }
        // ---- epilogue ----
        float xvr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t r = r0 + rb + lane + 32 * j;
            xvr[j] = (r < r_end && a.xv && MODE != SCAN_DENSE) ? a.xv[r * a.row_step] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int qi = qg + i;
            const int64_t q = q0 + qi;
            if (q >= a.nq) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t r = r0 + rb + lane + 32 * j;
                if (r >= r_end) continue;
                const float v = acc[i][j];
                if (MODE == SCAN_DENSE) {
                    float s;
                    if (DIRECT_L2) {
                        s = v;
                    } else if (a.metric == RDB_METRIC_COSINE) {
                        const float qn = vec_value(RDB_METRIC_COSINE, a.cos_small, qsq[i]);
                        const float xn = vec_value(RDB_METRIC_COSINE, a.cos_small, xsq[j]);
                        s = final_score(RDB_METRIC_COSINE, a.cos_small, v, qn, xn);
                    } else {
                        s = v;
                    }
                    a.dense_out[q * a.ld_out + r] = s;
                } else if (MODE == SCAN_FILTER) {
                    if (v >= fmaf(sA[qi], xvr[j], sB[qi])) {
                        const int slot = atomicAdd(&scnt[qi], 1);
                        if (slot < a.cap)
                            a.cand[((int64_t)split * a.nq + q) * a.cap + slot] = make_uint2(
                                __float_as_uint(final_score(a.metric, a.cos_small, v, sQv[qi], xvr[j])), (uint32_t)r);
                    }
                } else {  // SCAN_ARGMIN (squared L2; exact: summed directly)
                    const float dist = DIRECT_L2 ? v : fmaxf(sQv[qi] + xvr[j] - 2.f * v, 0.f);
                    const unsigned long long key = ((unsigned long long)float_asc_key(dist) << 32) | (uint32_t)r;
                    best[i] = min(best[i], key);
                }
            }
        }
    }
    if (MODE == SCAN_ARGMIN) {
        // the 32 lanes of a warp share its 8 queries
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            unsigned long long b = best[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) b = min(b, __shfl_xor_sync(0xffffffffu, b, o));
            if (lane == 0) atomicMin(&sbest[qg + i], b);
        }
    }
    __syncthreads();
    if (tid < BQ && q0 + tid < a.nq) {
        if (MODE == SCAN_FILTER) a.counts[(int64_t)split * a.nq + q0 + tid] = scnt[tid];
        if (MODE == SCAN_ARGMIN) a.best[(int64_t)split * a.nq + q0 + tid] = sbest[tid];
    }
}

template <typename T>
int launch_typed(const ScanArgs& a, int mode, cudaStream_t s, dim3 grid) {
    if (mode == SCAN_FILTER)
        simt_scan_kernel<T, SCAN_FILTER, false><<<grid, NT, 0, s>>>(a);
    else if (mode == SCAN_ARGMIN)
        simt_scan_kernel<T, SCAN_ARGMIN, false><<<grid, NT, 0, s>>>(a);
    else if (mode == SCAN_ARGMIN_EXACT)
        simt_scan_kernel<T, SCAN_ARGMIN, true><<<grid, NT, 0, s>>>(a);
    else if (a.metric == RDB_METRIC_L2)
        simt_scan_kernel<T, SCAN_DENSE, true><<<grid, NT, 0, s>>>(a);
    else
        simt_scan_kernel<T, SCAN_DENSE, false><<<grid, NT, 0, s>>>(a);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // namespace

int launch_scan_simt(const ScanArgs& a, int mode, cudaStream_t s) {
    if (a.nq <= 0 || a.n <= 0) return RDB_OK;
    RDB_CHECK_ARG(a.rows_per_split % kSimtRows == 0, "rows_per_split must be a multiple of %d",
                  kSimtRows);
    const int64_t gq = (a.nq + BQ - 1) / BQ;
    const int64_t gy = std::min<int64_t>(gq, 65535), gz = (gq + gy - 1) / gy;
    RDB_CHECK_ARG(gz <= 65535, "too many queries for one launch (%lld)", (long long)a.nq);
    dim3 grid(a.nsplit, (unsigned)gy, (unsigned)gz);
    switch (a.dtype) {
        case RDB_F32: return launch_typed<float>(a, mode, s, grid);
        case RDB_F16: return launch_typed<__half>(a, mode, s, grid);
        case RDB_BF16: return launch_typed<__nv_bfloat16>(a, mode, s, grid);
        default: return set_error(RDB_ERR_INVALID, "unknown dtype %d", a.dtype);
    }
}

}  // namespace rdb

using namespace rdb;

extern "C" {

int rdb_row_sqnorms(int dtype, const void* x, int64_t n, int d, float* out, void* stream) {
    RDB_CHECK_ARG(n >= 0 && d >= 1, "bad shape n=%lld d=%d", (long long)n, d);
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(x && out, "NULL pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned blocks = (unsigned)((n + 7) / 8);
    switch (dtype) {
        case RDB_F32: row_sqnorms_kernel<float><<<blocks, 256, 0, s>>>((const float*)x, n, d, d, out); break;
        case RDB_F16: row_sqnorms_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)x, n, d, d, out); break;
        case RDB_BF16:
            row_sqnorms_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)x, n, d, d, out);
            break;
        default: return set_error(RDB_ERR_INVALID, "unknown dtype %d", dtype);
    }
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int rdb_vec_values(int metric, int d, const float* sq, int64_t n, float* out, void* stream) {
    RDB_CHECK_ARG(metric >= 0 && metric <= 2, "unknown metric %d", metric);
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(sq && out, "NULL pointer");
    vec_values_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        metric, d <= 128 ? 1 : 0, sq, n, out);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int rdb_distance(int metric, int dtype, const void* q, int64_t nq, const void* x, int64_t nx,
                 int d, float* out, void* stream) {
    RDB_CHECK_ARG(metric >= 0 && metric <= 2, "unknown metric %d", metric);
    RDB_CHECK_ARG(nq >= 0 && nx >= 0 && d >= 1, "bad shapes");
    if (nq == 0 || nx == 0) return RDB_OK;
    RDB_CHECK_ARG(q && x && out, "NULL pointer");
    ScanArgs a = {};
    a.metric = metric;
    a.cos_small = d <= 128 ? 1 : 0;
    a.dtype = dtype;
    a.q = q;
    a.nq = nq;
    a.ldq = d;
    a.x = x;
    a.n = nx;
    a.ldx = d;
    a.row_step = 1;
    a.d = d;
    a.rows_per_split = kSimtRows;
    int64_t nsplit = (nx + kSimtRows - 1) / kSimtRows;
    a.dense_out = out;
    a.ld_out = nx;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // grid.x is limited to 2^31-1 splits; chunk the rows for the 65535-query limit only
    for (int64_t qc = 0; qc < nq; qc += 65535LL * kSimtQueries) {
        ScanArgs c = a;
        c.nq = std::min<int64_t>(nq - qc, 65535LL * kSimtQueries);
        c.q = static_cast<const char*>(q) + qc * d * elem_size(dtype);
        c.dense_out = out + qc * nx;
        c.nsplit = (int)nsplit;
        RDB_CHECK_ARG(nsplit < (1LL << 31), "too many rows");
        RDB_TRY(launch_scan_simt(c, SCAN_DENSE, s));
    }
    return RDB_OK;
}

}  // extern "C"
