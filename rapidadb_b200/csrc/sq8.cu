// INT8 storage: per-row symmetric scalar quantisation (SQ8).
//
// The reference lists INT8 among its storage precisions
// (csrc/include/rapidadb/core/types.h:9-14, python/rapidadb/config.py:21-26,
// README.md:13) without defining it.  Here a row x is stored as
//   scale = max_i |x_i| / 127                (fp32 division; 0 for a zero row)
//   code_i = rint(x_i / scale), clamped to [-127, 127]   (ties to even; 0 if scale == 0)
// and stands for the dequantised row  x^_i = fl(scale * code_i).  Searches over
// SQ8 rows are exact searches over x^ with fp32 queries (the reference
// formulas), one byte per element in HBM instead of four.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace rdb {
namespace {

__device__ __forceinline__ float ld_any(int dtype, const void* p, int64_t i) {
    if (dtype == RDB_F32) return static_cast<const float*>(p)[i];
    if (dtype == RDB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(static_cast<const __half*>(p)[i]);
}

// one warp per row
__global__ void sq8_encode_kernel(int dtype, const void* x, int64_t n, int64_t ldx, int d, int8_t* codes, int64_t ldc,
                                  float* scales) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    float amax = 0.f;
    for (int t = lane; t < d; t += 32) amax = fmaxf(amax, fabsf(ld_any(dtype, x, row * ldx + t)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = __fdiv_rn(amax, 127.f);
    for (int t = lane; t < (int)ldc; t += 32) {
        int c = 0;
        if (t < d && scale > 0.f) {
            const float v = rintf(__fdiv_rn(ld_any(dtype, x, row * ldx + t), scale));
            c = (int)fminf(fmaxf(v, -127.f), 127.f);
        }
        codes[row * ldc + t] = static_cast<int8_t>(c);
    }
    if (lane == 0) scales[row] = scale;
}

// per-row metric value of the dequantised row: |x^|^2 (L2), |x^| or
// sqrt(|x^|^2 + 1e-8) (cosine), 0 (dot)
__global__ void sq8_values_kernel(int metric, int cos_small, const int8_t* codes, const float* scales, int64_t n,
                                  int64_t ldc, int d, float* out) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const float s = scales[row];
    float acc = 0.f;
    for (int t = lane; t < d; t += 32) {
        const float v = __fmul_rn(s, static_cast<float>(codes[row * ldc + t]));
        acc = fmaf(v, v, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[row] = vec_value(metric, cos_small, acc);
}

}  // namespace
}  // namespace rdb

using namespace rdb;

extern "C" {

int rdb_sq8_encode(int dtype, const void* x, int64_t n, int64_t ldx, int d, int8_t* codes, int64_t ldc, float* scales,
                   void* stream) {
    RDB_CHECK_ARG(elem_size(dtype) != 0, "unknown dtype %d", dtype);
    RDB_CHECK_ARG(n >= 0 && d >= 1 && ldx >= d && ldc >= d, "bad shape");
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(x && codes && scales, "NULL pointer");
    const unsigned blocks = (unsigned)((n + 7) / 8);
    sq8_encode_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(dtype, x, n, ldx, d, codes, ldc, scales);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int rdb_sq8_row_values(int metric, const int8_t* codes, const float* scales, int64_t n, int64_t ldc, int d,
                       float* out, void* stream) {
    RDB_CHECK_ARG(metric >= 0 && metric <= 2, "unknown metric %d", metric);
    RDB_CHECK_ARG(n >= 0 && d >= 1 && ldc >= d, "bad shape");
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(codes && scales && out, "NULL pointer");
    const unsigned blocks = (unsigned)((n + 7) / 8);
    sq8_values_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(metric, d <= 128 ? 1 : 0, codes, scales,
                                                                             n, ldc, d, out);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // extern "C"
