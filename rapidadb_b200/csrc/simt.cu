// CUDA-core kernels: row norms, the dense reference-formula distance matrix
// (the raw ops of csrc/kernels/distance.cu), and the fused fp32 scan used by
// flat search for fp32 storage.
//
// The scan tiles 32 queries x 256 rows per CTA (256 threads, 8 x 4 outputs per
// thread) over K chunks of 32 staged through shared memory; each CTA walks a
// contiguous split of rows so its per-query candidate counters stay private.
// fp32 operands with TMA-compatible layouts go through simt_tma_scan_kernel
// (a 4-stage TMA ring, one CTA per SM); other dtypes / layouts and the dense
// distance matrix through simt_scan_kernel (register-staged chunks).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "scan.cuh"
#include "tma.cuh"

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
template <>
__device__ __forceinline__ float to_f<int8_t>(int8_t v) { return static_cast<float>(v); }

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
        if constexpr (sizeof(T) == 1) {
            const char4 c = __ldg(reinterpret_cast<const char4*>(p));
            return make_float4(c.x, c.y, c.z, c.w);
        } else if constexpr (sizeof(T) == 4) {
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

// SCAN_FILTER / SCAN_ARGMIN handling of one tile score: v = dot product (or
// the directly summed squared distance) of query q = q0 + qi and logical row r
template <int MODE, bool DIRECT_L2>
__device__ __forceinline__ void emit_score(const ScanArgs& a, float v, int qi, int64_t q, int64_t r, float xr,
                                           int split, const float* sA, const float* sB, const float* sQv, int* scnt,
                                           unsigned long long& best) {
    if (MODE == SCAN_FILTER) {
        if (v >= fmaf(sA[qi], xr, sB[qi])) {
            const int slot = atomicAdd(&scnt[qi], 1);
            if (slot < a.cap)
                a.cand[((int64_t)split * a.nq + q) * a.cap + slot] =
                    make_uint2(__float_as_uint(final_score(a.metric, a.cos_small, v, sQv[qi], xr)), (uint32_t)r);
        }
    } else {  // SCAN_ARGMIN (squared L2; exact: summed directly)
        const float dist = DIRECT_L2 ? v : fmaxf(sQv[qi] + xr - 2.f * v, 0.f);
        const unsigned long long key = ((unsigned long long)float_asc_key(dist) << 32) | (uint32_t)r;
        best = min(best, key);
    }
}

// end of a CTA's split: per-query candidate counts / arg-best to global memory
template <int MODE>
__device__ __forceinline__ void finish_split(const ScanArgs& a, int64_t q0, int split, int qg, int lane, int tid,
                                             const int* scnt, unsigned long long* sbest,
                                             const unsigned long long (&best)[8]) {
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

// T: query (and row) element type; TX = int8_t: rows are SQ8 codes, each
// dequantised as fl(x_scale[row] * code) while it is staged, so the arithmetic
// that follows is the fp32 scan over the dequantised rows
template <typename T, int MODE, bool DIRECT_L2, typename TX = T>
__global__ void __launch_bounds__(NT, 2) simt_scan_kernel(ScanArgs a) {
    __shared__ __align__(16) float Qs[BK][BQ];
    __shared__ float Xs[BK][XS];
    __shared__ float sA[BQ], sB[BQ], sQv[BQ];
    __shared__ int scnt[BQ];
    __shared__ unsigned long long sbest[BQ];

    const T* __restrict__ qp = static_cast<const T*>(a.q);
    const TX* __restrict__ xp = static_cast<const TX*>(a.x);
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
                px[i] = (r < r_end && nv > 0) ? load4<TX>(xp + r * xstride + k, vec_x, nv)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                if constexpr (sizeof(TX) == 1) {
                    const float sc = r < r_end ? __ldg(a.x_scale + r * a.row_step) : 0.f;
                    px[i] = make_float4(__fmul_rn(sc, px[i].x), __fmul_rn(sc, px[i].y), __fmul_rn(sc, px[i].z),
                                        __fmul_rn(sc, px[i].w));
                }
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
                } else {
                    emit_score<MODE, DIRECT_L2>(a, v, qi, q, r, xvr[j], split, sA, sB, sQv, scnt, best[i]);
                }
            }
        }
    }
    finish_split<MODE>(a, q0, split, qg, lane, tid, scnt, sbest, best);
}

// ------------------------------------------------- TMA-fed fp32 scan --
//
// simt_scan_kernel's tile and thread mapping (32 queries x 256 rows, 8 x 4
// outputs per thread) for fp32 rows, with the operands delivered by TMA: a
// ring of kTmaStages stages, each holding one K chunk of 32 floats (one
// 128-byte line per row, 128-byte swizzle) of the query tile and of the row
// tile, so that several chunks are in flight per CTA and the DRAM latency
// hides behind the multiply-adds of earlier chunks.  One CTA per SM walks
// its split of rows tile by tile, the ring running on across tiles; thread 0
// refills a stage after the CTA barrier that ends its use.  Swizzled reads:
// 16-byte group g of line L sits at group g ^ (L mod 8), so the lanes of a
// warp (rows L = lane + 32 j) read 8 distinct groups per 128 bytes and the
// query reads are broadcasts.  Summation order per (query, row) is
// k = 0, 1, ..., d - 1 as in simt_scan_kernel (bit-identical results);
// columns past d and rows past n read as zero.

constexpr int kTmaStages = 4;
constexpr int kTmaXBytes = BN * BK * 4;  // 32 KB
constexpr int kTmaQBytes = BQ * BK * 4;  // 4 KB
constexpr int kTmaStageBytes = kTmaXBytes + kTmaQBytes;
constexpr int kTmaSmemBytes = kTmaStages * kTmaStageBytes + 1024 /* alignment */ + 64 /* barriers */;
static_assert(BK * 4 == 128, "one 128-byte swizzle line per row and chunk");

template <int MODE, bool DIRECT_L2>
__global__ void __launch_bounds__(NT, 1)
    simt_tma_scan_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_x,
                         const ScanArgs a, unsigned* status) {
    extern __shared__ unsigned char tma_smem_raw[];
    __shared__ float sA[BQ], sB[BQ], sQv[BQ];
    __shared__ int scnt[BQ];
    __shared__ unsigned long long sbest[BQ];

    // 1024-byte aligned ring (the swizzle atom); an offset from the shared
    // array itself keeps the accesses in the shared window (LDS, not generic)
    unsigned char* smem = tma_smem_raw + ((1024u - (tma::smem_addr(tma_smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTmaStages * kTmaStageBytes);

    // SCAN_PARTIAL: CTA x covers split x / ksplit over its share of the K chunks
    const int ks = MODE == SCAN_PARTIAL ? max(1, a.ksplit) : 1;
    const int split = blockIdx.x / ks;
    const int64_t q0 = ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * BQ;
    if (q0 >= a.nq) return;
    const int64_t r_begin = (int64_t)split * a.rows_per_split;
    const int64_t r_end = min(a.n, r_begin + a.rows_per_split);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qg = (warp & 3) * 8;
    const int rb = (warp >> 2) * 128;
    const int nchunk_all = (a.d + BK - 1) / BK;
    const int kpart = blockIdx.x - split * ks;
    const int c_first = (int)((int64_t)kpart * nchunk_all / ks);
    const int nchunk = (int)((int64_t)(kpart + 1) * nchunk_all / ks) - c_first;
    if (nchunk <= 0) return;
    const int ntile = (int)((r_end - r_begin + BN - 1) / BN);
    const int nitems = ntile * nchunk;  // (tile, chunk) pairs in ring order

    auto issue = [&](int it) {
        const int st = it % kTmaStages;
        const int t = it / nchunk, c = it - t * nchunk;
        unsigned char* dst = smem + st * kTmaStageBytes;
        tma::bar_expect_tx(&full[st], kTmaStageBytes);
        tma::load_2d(&tmap_x, &full[st], dst, (c_first + c) * BK, (int)(r_begin + (int64_t)t * BN));
        tma::load_2d(&tmap_q, &full[st], dst + kTmaXBytes, (c_first + c) * BK, (int)q0);
    };
    if (tid == 0) {
        tma::prefetch_map(&tmap_x);
        tma::prefetch_map(&tmap_q);
        for (int st = 0; st < kTmaStages; ++st) tma::bar_init(&full[st], 1);
        tma::fence_init();
    }
    if (tid < BQ) {
        const int64_t q = q0 + tid;
        const float qv = (q < a.nq && a.qv) ? a.qv[q] : 0.f;
        const float thr = (a.thr && q < a.nq) ? a.thr[q] : __int_as_float(0x7fc00000);
        const FilterCoef f = filter_coef(a.metric, a.cos_small, thr, qv);
        sA[tid] = f.A;
        sB[tid] = f.B;
        sQv[tid] = qv;
        scnt[tid] = 0;
        sbest[tid] = ~0ull;
    }
    __syncthreads();
    if (tid == 0)
        for (int it = 0; it < min(kTmaStages, nitems); ++it) issue(it);

    unsigned long long best[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) best[i] = ~0ull;
    const int sw = lane & 7;  // (row line) mod 8 of every row this lane reads
    int it = 0;
    for (int t = 0; t < ntile; ++t) {
        const int64_t r0 = r_begin + (int64_t)t * BN;
        float acc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
        for (int c = 0; c < nchunk; ++c, ++it) {
            const int st = it % kTmaStages;
            const bool ok = tma::bar_wait(&full[st], (uint32_t)((it / kTmaStages) & 1));
            const float* Xs = reinterpret_cast<const float*>(smem + st * kTmaStageBytes);
            const float* Qs = reinterpret_cast<const float*>(smem + st * kTmaStageBytes + kTmaXBytes);
            if (ok) {
#pragma unroll 2
                for (int g = 0; g < BK / 4; ++g) {
                    float4 xb[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        xb[j] = *reinterpret_cast<const float4*>(Xs + (rb + lane + 32 * j) * BK + ((g ^ sw) << 2));
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 qa = *reinterpret_cast<const float4*>(Qs + (qg + i) * BK + ((g ^ i) << 2));
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            if (DIRECT_L2) {
                                float df = qa.x - xb[j].x;
                                acc[i][j] = fmaf(df, df, acc[i][j]);
                                df = qa.y - xb[j].y;
                                acc[i][j] = fmaf(df, df, acc[i][j]);
                                df = qa.z - xb[j].z;
                                acc[i][j] = fmaf(df, df, acc[i][j]);
                                df = qa.w - xb[j].w;
                                acc[i][j] = fmaf(df, df, acc[i][j]);
                            } else {
                                acc[i][j] = fmaf(qa.x, xb[j].x, acc[i][j]);
                                acc[i][j] = fmaf(qa.y, xb[j].y, acc[i][j]);
                                acc[i][j] = fmaf(qa.z, xb[j].z, acc[i][j]);
                                acc[i][j] = fmaf(qa.w, xb[j].w, acc[i][j]);
                            }
                        }
                    }
                }
            }
            // every thread is done with stage st (and agrees whether a wait gave up)
            if (__syncthreads_or(!ok)) {
                if (tid == 0) {
                    if (status) atomicOr(status, DEV_TIMEOUT_SIMT);
                    // bounded wait for the copies still in flight, then leave
                    for (int j = it; j < min(it + kTmaStages, nitems); ++j)
                        tma::bar_wait(&full[j % kTmaStages], (uint32_t)((j / kTmaStages) & 1));
                }
                __syncthreads();
                return;
            }
            if (tid == 0 && it + kTmaStages < nitems) issue(it + kTmaStages);
        }
        if (MODE == SCAN_PARTIAL) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int64_t q = q0 + qg + i;
                if (q >= a.nq) continue;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t r = r0 + rb + lane + 32 * j;
                    if (r < r_end) atomicAdd(&a.dense_out[q * a.ld_out + r], acc[i][j]);
                }
            }
            continue;
        }
        float xvr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t r = r0 + rb + lane + 32 * j;
            xvr[j] = (r < r_end && a.xv) ? a.xv[r * a.row_step] : 0.f;
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
                emit_score<MODE, DIRECT_L2>(a, acc[i][j], qi, q, r, xvr[j], split, sA, sB, sQv, scnt, best[i]);
            }
        }
    }
    finish_split<MODE>(a, q0, split, qg, lane, tid, scnt, sbest, best);
}

__global__ void partial_finalize_kernel(int metric, int cos_small, float* __restrict__ dense, int64_t nq, int64_t n,
                                        int64_t ld, const float* __restrict__ qv, const float* __restrict__ xv,
                                        int64_t row_step) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nq * n) return;
    const int64_t q = i / n, r = i - q * n;
    float* p = dense + q * ld + r;
    if (metric != RDB_METRIC_DOT) *p = final_score(metric, cos_small, *p, qv[q], xv[r * row_step]);
}

// fp32 rows and queries whose layout suits the TMA maps (16-byte aligned
// bases and strides, coordinates within int32)
bool tma_scan_ok(const ScanArgs& a, int mode) {
    if (a.dtype != RDB_F32 || a.x_i8) return false;
    if (mode != SCAN_FILTER && mode != SCAN_ARGMIN && mode != SCAN_ARGMIN_EXACT && mode != SCAN_PARTIAL) return false;
    if ((reinterpret_cast<uintptr_t>(a.q) & 15) || (reinterpret_cast<uintptr_t>(a.x) & 15)) return false;
    if (a.ldq % 4 || (a.ldx * a.row_step) % 4) return false;
    if (a.nq >= (1LL << 31) - BQ || a.n >= (1LL << 31) - 2 * BN) return false;
    if (a.ldx * a.row_step * 4 >= (1LL << 40) || a.ldq * 4 >= (1LL << 40)) return false;
    return tma::encode_tiled() != nullptr;
}

template <int MODE, bool DIRECT_L2>
int launch_tma_typed(const ScanArgs& a, dim3 grid, cudaStream_t s) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        RDB_CUDA_TRY(cudaFuncSetAttribute(simt_tma_scan_kernel<MODE, DIRECT_L2>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kTmaSmemBytes));
        attr[dev] = true;
    }
    CUtensorMap mq, mx;
    RDB_TRY(tma::map_f32_2d(&mq, a.q, a.nq, a.d, a.ldq * 4, BK, BQ));
    RDB_TRY(tma::map_f32_2d(&mx, a.x, a.n, a.d, a.ldx * a.row_step * 4, BK, BN));
    simt_tma_scan_kernel<MODE, DIRECT_L2><<<grid, NT, kTmaSmemBytes, s>>>(mq, mx, a, device_status_word());
    RDB_LAUNCH_CHECK();
    return RDB_OK;
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

bool simt_tma_ok(const ScanArgs& a, int mode) { return tma_scan_ok(a, mode); }

int norms_preload() {
    cudaFuncAttributes fa;
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, row_sqnorms_kernel<float>));
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, row_sqnorms_kernel<__half>));
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, row_sqnorms_kernel<__nv_bfloat16>));
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, vec_values_kernel));
    return RDB_OK;
}

int launch_partial_finalize(const ScanArgs& a, cudaStream_t s) {
    const int64_t total = a.nq * a.n;
    if (total == 0) return RDB_OK;
    partial_finalize_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(a.metric, a.cos_small, a.dense_out, a.nq,
                                                                          a.n, a.ld_out, a.qv, a.xv, a.row_step);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int launch_scan_simt(const ScanArgs& a, int mode, cudaStream_t s) {
    if (a.nq <= 0 || a.n <= 0) return RDB_OK;
    RDB_CHECK_ARG(a.rows_per_split % kSimtRows == 0, "rows_per_split must be a multiple of %d",
                  kSimtRows);
    const int64_t gq = (a.nq + BQ - 1) / BQ;
    const int64_t gy = std::min<int64_t>(gq, 65535), gz = (gq + gy - 1) / gy;
    RDB_CHECK_ARG(gz <= 65535, "too many queries for one launch (%lld)", (long long)a.nq);
    dim3 grid(a.nsplit, (unsigned)gy, (unsigned)gz);
    if (tma_scan_ok(a, mode)) {
        if (mode == SCAN_FILTER) return launch_tma_typed<SCAN_FILTER, false>(a, grid, s);
        if (mode == SCAN_ARGMIN) return launch_tma_typed<SCAN_ARGMIN, false>(a, grid, s);
        if (mode == SCAN_PARTIAL) {
            RDB_CHECK_ARG(a.dense_out && a.ksplit >= 1 && a.ksplit <= (a.d + BK - 1) / BK, "bad partial scan");
            RDB_CHECK_ARG((int64_t)a.nsplit * a.ksplit <= 0x7fffffffLL, "too many CTAs");
            dim3 g2(a.nsplit * a.ksplit, grid.y, grid.z);
            return launch_tma_typed<SCAN_PARTIAL, false>(a, g2, s);
        }
        return launch_tma_typed<SCAN_ARGMIN, true>(a, grid, s);
    }
    RDB_CHECK_ARG(mode != SCAN_PARTIAL, "SCAN_PARTIAL needs fp32 operands in a TMA layout");
    if (a.x_i8) {
        RDB_CHECK_ARG(a.dtype == RDB_F32 && a.x_scale, "SQ8 rows need fp32 queries and per-row scales");
        RDB_CHECK_ARG(mode == SCAN_FILTER, "SQ8 rows support the filter scan only");
        simt_scan_kernel<float, SCAN_FILTER, false, int8_t><<<grid, NT, 0, s>>>(a);
        RDB_LAUNCH_CHECK();
        return RDB_OK;
    }
    switch (a.dtype) {
        case RDB_F32: return launch_typed<float>(a, mode, s, grid);
        case RDB_F16: return launch_typed<__half>(a, mode, s, grid);
        case RDB_BF16: return launch_typed<__nv_bfloat16>(a, mode, s, grid);
        default: return set_error(RDB_ERR_INVALID, "unknown dtype %d", a.dtype);
    }
}

int row_sqnorms_ld(int dtype, const void* x, int64_t n, int d, int64_t ld, float* out, cudaStream_t s) {
    RDB_CHECK_ARG(n >= 0 && d >= 1 && ld >= d, "bad shape n=%lld d=%d ld=%lld", (long long)n, d, (long long)ld);
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(x && out, "NULL pointer");
    const unsigned blocks = (unsigned)((n + 7) / 8);
    switch (dtype) {
        case RDB_F32: row_sqnorms_kernel<float><<<blocks, 256, 0, s>>>((const float*)x, n, d, ld, out); break;
        case RDB_F16: row_sqnorms_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)x, n, d, ld, out); break;
        case RDB_BF16:
            row_sqnorms_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)x, n, d, ld, out);
            break;
        default: return set_error(RDB_ERR_INVALID, "unknown dtype %d", dtype);
    }
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // namespace rdb

using namespace rdb;

extern "C" {

int rdb_row_sqnorms(int dtype, const void* x, int64_t n, int d, float* out, void* stream) {
    return row_sqnorms_ld(dtype, x, n, d, d, out, static_cast<cudaStream_t>(stream));
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
