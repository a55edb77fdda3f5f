// Device-side completion of flat search, so rdb_flat_search never waits on
// the host.
//
//   query_prep_kernel   per-query metric value qv[q] (squared norm, norm or
//                       0, any row stride) and the chunk's overflow word
//                       cleared, in one launch.
//   flat_repair_kernel  runs after the candidate select.  When no candidate
//                       list of the chunk overflowed (the overflow word is 0)
//                       every CTA returns at once.  Otherwise each (split,
//                       marked query) pair is rescanned on CUDA cores: the
//                       split's rows are scored with the reference formulas
//                       (L2 summed directly as sum (q - x)^2) and an exact
//                       streaming top-min(k, cap) -- keys (score, row), ties
//                       to the lower row, kept in a shared-memory buffer
//                       that is sorted and cut to k whenever it fills -- is
//                       written back into that pair's candidate list, which
//                       then holds at most cap entries.  A second select
//                       pass limited to the marked queries produces their
//                       answers.
//
// The exact top-k of every split is a superset of that split's share of the
// global top-k, so the second select returns exactly what an unfiltered
// search returns.  The repair costs one rescan of the marked queries' rows
// (adversarial inputs, e.g. many identical rows); the common case costs two
// launches that exit immediately.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "repair.cuh"

namespace rdb {
namespace {

constexpr int NT = 256;
constexpr int NWARP = NT / 32;
constexpr int kRowsPerWarp = 4;  // rows a warp scores between two buffer checks

__device__ __forceinline__ float ld_f(int dtype, const void* p, int64_t i) {
    if (dtype == RDB_F32) return static_cast<const float*>(p)[i];
    if (dtype == RDB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(static_cast<const __half*>(p)[i]);
}

// Element t of stored row r (SQ8 codes dequantised with the row's scale).
__device__ __forceinline__ float ld_row(const RepairArgs& a, int64_t r, int t) {
    if (a.x_i8) return __fmul_rn(a.x_scale[r], static_cast<float>(static_cast<const int8_t*>(a.x)[r * a.ldx + t]));
    return ld_f(a.dtype, a.x, r * a.ldx + t);
}

__global__ void __launch_bounds__(NT) query_prep_kernel(int metric, int cos_small, int dtype, const void* q,
                                                        int64_t nq, int64_t ldq, int d, float* qv,
                                                        unsigned* flag) {
    const int lane = threadIdx.x & 31;
    if (flag && blockIdx.x == 0 && threadIdx.x == 0) *flag = 0u;
    const int64_t row = (int64_t)blockIdx.x * NWARP + (threadIdx.x >> 5);
    if (row >= nq) return;
    float acc = 0.f;
    for (int t = lane; t < d; t += 32) {
        const float v = ld_f(dtype, q, row * ldq + t);
        acc = fmaf(v, v, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) qv[row] = vec_value(metric, cos_small, acc);
}

// Bitonic sort of n (power of two) keys in shared memory, all threads.
__device__ void sort_keys(unsigned long long* keys, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n >> 1); i += NT) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = ((lo & size) == 0);
                const unsigned long long x = keys[lo], y = keys[hi];
                if ((x > y) == up) {
                    keys[lo] = y;
                    keys[hi] = x;
                }
            }
            __syncthreads();
        }
    }
}

struct RepairShared {
    unsigned long long tkey;  // keys >= tkey cannot enter the top-kk
    int nb;                   // keys in the buffer
};

// Sort the buffer, keep the best kk keys and tighten the admission key.
__device__ void compact(unsigned long long* buf, int B, int kk, RepairShared& S) {
    __syncthreads();
    const int nb = min(S.nb, B);
    for (int i = nb + threadIdx.x; i < B; i += NT) buf[i] = ~0ull;
    __syncthreads();
    sort_keys(buf, B);
    if (threadIdx.x == 0) {
        S.nb = min(nb, kk);
        if (nb >= kk) S.tkey = buf[kk - 1];  // later rows must beat the kk-th best key
    }
    __syncthreads();
}

__global__ void __launch_bounds__(NT) flat_repair_kernel(RepairArgs a) {
    extern __shared__ __align__(16) unsigned long long rbuf[];
    __shared__ RepairShared S;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool largest = metric_largest(a.metric);
    if (blockIdx.x == 0 && threadIdx.x == 0 && a.status && a.status_mirror) {
        // forward a bounded-wait failure of this call's kernels to the host
        // word that the host checks without synchronising
        const unsigned st = *reinterpret_cast<volatile const unsigned*>(a.status);
        if (st) *reinterpret_cast<volatile unsigned*>(a.status_mirror) = st;
    }
    if (*reinterpret_cast<volatile const unsigned*>(a.flag) == 0u) return;
    const int64_t work = (int64_t)a.nq * a.nsplit;
    for (int64_t w = blockIdx.x; w < work; w += gridDim.x) {
        const int64_t q = w / a.nsplit;
        const int s = (int)(w % a.nsplit);
        if (a.mark_q[q] == 0u) continue;  // uniform across the CTA
        const int64_t r0 = (int64_t)s * a.rows_per_split;
        const int64_t r1 = min(r0 + a.rows_per_split, a.n);
        if (r1 <= r0) {
            if (threadIdx.x == 0) a.counts[(int64_t)s * a.nq + q] = 0;
            continue;
        }
        const int kk = (int)min(min((int64_t)a.k, a.cap), r1 - r0);
        if (threadIdx.x == 0) {
            S.nb = 0;
            S.tkey = ~0ull;
        }
        __syncthreads();
        const float qv = a.metric == RDB_METRIC_L2 ? 0.f : a.qv[q];
        for (int64_t base = r0; base < r1; base += NWARP * kRowsPerWarp) {
#pragma unroll 1
            for (int j = 0; j < kRowsPerWarp; ++j) {
                const int64_t r = base + (int64_t)warp * kRowsPerWarp + j;
                if (r >= r1) break;
                float acc = 0.f;
                if (a.metric == RDB_METRIC_L2) {
                    for (int t = lane; t < a.d; t += 32) {
                        const float df = ld_f(a.dtype, a.q, q * a.ldq + t) - ld_row(a, r, t);
                        acc = fmaf(df, df, acc);
                    }
                } else {
                    for (int t = lane; t < a.d; t += 32)
                        acc = fmaf(ld_f(a.dtype, a.q, q * a.ldq + t), ld_row(a, r, t), acc);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (lane == 0) {
                    const float sc = a.metric == RDB_METRIC_L2 ? acc
                                                               : final_score(a.metric, a.cos_small, acc, qv, a.xv ? a.xv[r] : 0.f);
                    const unsigned long long key = ((unsigned long long)score_key(sc, largest) << 32) | (uint32_t)r;
                    if (key < S.tkey) {
                        const int slot = atomicAdd(&S.nb, 1);
                        rbuf[slot] = key;  // slot < B: the buffer keeps NWARP * kRowsPerWarp free entries
                    }
                }
            }
            __syncthreads();
            if (S.nb > a.buf_keys - NWARP * kRowsPerWarp) compact(rbuf, a.buf_keys, kk, S);
        }
        compact(rbuf, a.buf_keys, kk, S);
        const int nb = S.nb;
        uint2* out = a.cand + ((int64_t)s * a.nq + q) * a.cap;
        for (int i = threadIdx.x; i < nb; i += NT) {
            const unsigned long long key = rbuf[i];
            out[i] = make_uint2(f2u(key_score((uint32_t)(key >> 32), largest)), (uint32_t)key);
        }
        if (threadIdx.x == 0) a.counts[(int64_t)s * a.nq + q] = nb;
        __syncthreads();
    }
}

}  // namespace

int launch_query_prep(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d, float* qv,
                      unsigned* flag, cudaStream_t s) {
    if (nq <= 0) return RDB_OK;
    const unsigned blocks = (unsigned)((nq + NWARP - 1) / NWARP);
    query_prep_kernel<<<blocks, NT, 0, s>>>(metric, d <= 128 ? 1 : 0, dtype, q, nq, ldq, d, qv, flag);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int repair_buffer_keys(int k, int64_t cap) {
    int kk = (int)std::min<int64_t>(k, cap);
    int p = 1;
    while (p < kk) p <<= 1;
    return std::max(1024, 2 * p);
}

int launch_flat_repair(const RepairArgs& a, cudaStream_t s) {
    if (a.nq <= 0) return RDB_OK;
    RDB_CHECK_ARG(a.buf_keys >= 2 * std::min<int64_t>(a.k, a.cap) && a.buf_keys >= 1024 &&
                      (a.buf_keys & (a.buf_keys - 1)) == 0,
                  "repair buffer of %d keys too small", a.buf_keys);
    const size_t smem = sizeof(unsigned long long) * (size_t)a.buf_keys;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        RDB_CUDA_TRY(cudaFuncSetAttribute(flat_repair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)(sizeof(unsigned long long) * 2 * 8192)));
        attr_set[dev] = true;
    }
    const int64_t work = a.nq * (int64_t)a.nsplit;
    const unsigned grid = (unsigned)std::min<int64_t>(work, 2LL * num_sms());
    flat_repair_kernel<<<grid, NT, smem, s>>>(a);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // namespace rdb
