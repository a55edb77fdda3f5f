// IVF-Flat and IVF-PQ list scans, PQ encoding.
//
// The reference has no IVF or PQ code (its config fields nlist / nprobe /
// pq_m / pq_k, python/rapidadb/config.py:50-56, are unused); the semantics
// follow the CPU oracle (oracle/cpu_oracle.c: orc_ivf_flat_search,
// orc_pq_encode, orc_ivfpq_search).
//
// Both scans here are LIST-MAJOR: the [Q, nprobe] probe table is inverted
// with the stable label sort (entries grouped by list), and a CTA scores a
// list's rows (IVF-Flat) or codes (IVF-PQ) for a chunk of the queries that
// probe it, so a list crosses HBM once per chunk instead of once per probing
// query (IVF-Flat deals a popular list's chunks to several CTAs).  Each
// (query, probed list) pair yields its best k (k <= 32, kept sorted in the
// registers of one warp: lane i holds the i-th best), written to
// out[probe slot][query][k]; the merge kernel (rdb_topk_merge) then keeps the
// best k of the nprobe lists.  The IVF-PQ scan here serves code widths that
// the query-major search (ivfpq.cu) does not.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "ivf.cuh"
#include "scan.cuh"
#include "sort.cuh"

namespace rdb {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int kMaxIvfK = 32;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

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

// a ranks before b; ties to the lower row
__device__ __forceinline__ bool ranks_before(float a, int64_t ia, float b, int64_t ib, bool largest) {
    if (a != b) return largest ? (a > b) : (a < b);
    return ia < ib;
}

// Sorted best-k of one query held by one warp: lane i < k keeps the i-th best.
struct WarpTopK {
    float v;
    int64_t id;
    __device__ __forceinline__ void init(bool largest) {
        v = largest ? -INFINITY : INFINITY;
        id = INT64_MAX;
    }
    // every lane offers (s, sid) when `valid`; the warp inserts those that
    // beat the current k-th, lowest lane first
    __device__ __forceinline__ void offer(float s, int64_t sid, bool valid, int k, bool largest, int lane) {
        float kv = __shfl_sync(FULL, v, k - 1);
        int64_t kid = __shfl_sync(FULL, id, k - 1);
        unsigned m = __ballot_sync(FULL, valid && ranks_before(s, sid, kv, kid, largest));
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const float cs = __shfl_sync(FULL, s, src);
            const int64_t cid = __shfl_sync(FULL, sid, src);
            kv = __shfl_sync(FULL, v, k - 1);
            kid = __shfl_sync(FULL, id, k - 1);
            if (!ranks_before(cs, cid, kv, kid, largest)) continue;
            const unsigned bm = __ballot_sync(FULL, lane < k && ranks_before(v, id, cs, cid, largest));
            const int pos = __popc(bm);
            const float pv = __shfl_up_sync(FULL, v, 1);
            const int64_t pid = __shfl_up_sync(FULL, id, 1);
            if (lane == pos) {
                v = cs;
                id = cid;
            } else if (lane > pos && lane < k) {
                v = pv;
                id = pid;
            }
        }
    }
};

__global__ void probe_to_labels_kernel(const int64_t* __restrict__ probe, int64_t n, int nlist,
                                       int32_t* __restrict__ labels) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int64_t l = probe[i];
    labels[i] = (l >= 0 && l < nlist) ? (int32_t)l : 0;
}

// ------------------------------------------------------------- IVF-Flat scan
//
// CTA = one list x a chunk of FQ = 32 probing queries, rows walked in tiles
// of FR = 256 over K chunks of FK = 32 staged in shared memory (the next
// chunk loaded into registers while the current one is consumed).  Warp w
// computes queries 8 (w mod 4) .. + 7 against rows 128 (w / 4) + lane + 32 j
// (j < 4): query operands are shared-memory broadcasts, each lane loads 4 row
// values per k for 32 multiply-adds.  The tile's scores go through shared
// memory to the per-query warp top-k lists (warp w keeps queries 4 w .. + 3).
//
// L2 with k <= kL2ExpandMaxK uses the expansion |q|^2 + |x|^2 - 2 q.x (one
// multiply-add per element instead of a subtract and a multiply-add) and
// keeps k + kL2Margin rows per (query, list); once the list is scanned, each
// kept row is rescored with the direct sum of (q - x)^2 in dimension order
// and the best k of those are written, so the reported distances are the
// direct ones.  Larger k accumulates (q - x)^2 directly.

constexpr int FQ = 32;   // queries per chunk
constexpr int FR = 256;  // rows per tile
constexpr int FK = 32;   // K chunk
constexpr int FNT = 256;
constexpr int FXS = FR + 1;  // row stride of the transposed row tile
constexpr int kL2Margin = 8;
constexpr int kL2ExpandMaxK = kMaxIvfK - kL2Margin;

template <typename T>
__device__ __forceinline__ float4 load4f(const T* p, bool vec, int nvalid) {
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

struct IvfFlatSmem {
    float Qs[FK][FQ];
    float Xs[FK][FXS];
    float S[FQ][FXS];
    int64_t s_q[FQ];
    int s_p[FQ];
    float s_qv[FQ];
};

// four row elements as floats; SQ8 rows (TX = int8_t) dequantised with the
// row's scale, fl(scale * code)
template <typename TX>
__device__ __forceinline__ float4 load_row4(const TX* p, int64_t r, const float* x_scale, bool vec, int nvalid) {
    float4 v = load4f<TX>(p, vec, nvalid);
    if constexpr (sizeof(TX) == 1) {
        const float sc = __ldg(x_scale + r);
        v = make_float4(__fmul_rn(sc, v.x), __fmul_rn(sc, v.y), __fmul_rn(sc, v.z), __fmul_rn(sc, v.w));
    }
    return v;
}

// EXPAND: accumulate q.x (every metric but direct L2); false: accumulate (q - x)^2.
// T: query (and row) type; TX = int8_t: rows are SQ8 codes with x_scale.
template <typename T, bool EXPAND, typename TX = T>
__global__ void __launch_bounds__(FNT, 2) ivf_flat_scan_kernel(
    int metric, int cos_small, const T* __restrict__ q, int64_t Q, int64_t ldq, int d, const float* __restrict__ qv,
    int nprobe, const int64_t* __restrict__ eperm, const int64_t* __restrict__ eseg, const TX* __restrict__ rows,
    int64_t ldx, const float* __restrict__ x_scale, const float* __restrict__ xv, const int64_t* __restrict__ list_off,
    const int64_t* __restrict__ list_end, int nlist,
    const int64_t* __restrict__ ids, int k, float* __restrict__ out_v, int64_t* __restrict__ out_i) {
    extern __shared__ __align__(16) unsigned char ivf_smem[];
    IvfFlatSmem& sh = *reinterpret_cast<IvfFlatSmem*>(ivf_smem);
    const bool largest = metric != RDB_METRIC_L2;
    const bool rescore = EXPAND && metric == RDB_METRIC_L2;
    const int kk = rescore ? min(kMaxIvfK, k + kL2Margin) : k;  // rows kept per (query, list)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qg = (warp & 3) * 8;     // this warp's first query
    const int rb = (warp >> 2) * 128;  // this warp's first tile row
    const int sq = tid >> 3, sk = (tid & 7) * 4;  // staging: query / row t / 8 (+ 32 i), k 4 (t mod 8)
    const bool vec_q = (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (ldq % 4 == 0);
    const bool vec_x = (reinterpret_cast<uintptr_t>(rows) % 16 == 0) && (ldx % 4 == 0);

    for (int l = blockIdx.x; l < nlist; l += gridDim.x) {
        const int64_t e0 = eseg[l], e1 = eseg[l + 1];
        const int64_t r0 = list_off[l], r1 = list_end ? list_end[l] : list_off[l + 1];
        // chunks of FQ probing queries, dealt round-robin to the gridDim.y
        // CTAs of this list (a popular list is shared by several SMs)
        for (int64_t ec = e0 + (int64_t)blockIdx.y * FQ; ec < e1; ec += (int64_t)gridDim.y * FQ) {
            const int nqc = (int)min((int64_t)FQ, e1 - ec);
            __syncthreads();
            if (tid < FQ) {
                if (tid < nqc) {
                    const int64_t e = eperm[ec + tid];
                    sh.s_q[tid] = e / nprobe;
                    sh.s_p[tid] = (int)(e % nprobe);
                    sh.s_qv[tid] = qv ? qv[e / nprobe] : 0.f;
                } else {
                    sh.s_q[tid] = -1;
                    sh.s_p[tid] = 0;
                    sh.s_qv[tid] = 0.f;
                }
            }
            WarpTopK st[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) st[j].init(largest);
            __syncthreads();
            const int64_t my_q = sh.s_q[sq];
            for (int64_t t0 = r0; t0 < r1; t0 += FR) {
                float acc[8][4];
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
                float4 pq, px[8];
                auto fetch = [&](int k0) {
                    const int kx = k0 + sk;
                    const int nv = min(4, d - kx);
                    pq = (my_q >= 0 && nv > 0) ? load4f<T>(q + my_q * ldq + kx, vec_q, nv)
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int64_t r = t0 + sq + 32 * i;
                        px[i] = (r < r1 && nv > 0) ? load_row4<TX>(rows + r * ldx + kx, r, x_scale, vec_x, nv)
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                };
                fetch(0);
                for (int k0 = 0; k0 < d; k0 += FK) {
                    __syncthreads();  // the previous chunk (and tile's scores) are consumed
                    sh.Qs[sk + 0][sq] = pq.x;
                    sh.Qs[sk + 1][sq] = pq.y;
                    sh.Qs[sk + 2][sq] = pq.z;
                    sh.Qs[sk + 3][sq] = pq.w;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        sh.Xs[sk + 0][sq + 32 * i] = px[i].x;
                        sh.Xs[sk + 1][sq + 32 * i] = px[i].y;
                        sh.Xs[sk + 2][sq + 32 * i] = px[i].z;
                        sh.Xs[sk + 3][sq + 32 * i] = px[i].w;
                    }
                    __syncthreads();
                    if (k0 + FK < d) fetch(k0 + FK);
#pragma unroll 4
                    for (int kk = 0; kk < FK; ++kk) {
                        const float4 a0 = *reinterpret_cast<const float4*>(&sh.Qs[kk][qg]);
                        const float4 a1 = *reinterpret_cast<const float4*>(&sh.Qs[kk][qg + 4]);
                        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                        float bv[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) bv[j] = sh.Xs[kk][rb + lane + 32 * j];
#pragma unroll
                        for (int i = 0; i < 8; ++i)
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                if constexpr (EXPAND) {
                                    acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                                } else {
                                    const float df = av[i] - bv[j];
                                    acc[i][j] = fmaf(df, df, acc[i][j]);
                                }
                            }
                    }
                }
                // final scores of the tile -> S
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int ri = rb + lane + 32 * j;
                    const int64_t r = t0 + ri;
                    const bool need_xv = metric == RDB_METRIC_COSINE || rescore;
                    const float xr = (need_xv && r < r1) ? xv[r] : 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int qi = qg + i;
                        float sc = acc[i][j];
                        if (metric == RDB_METRIC_COSINE && r < r1) sc = final_score(metric, cos_small, sc, sh.s_qv[qi], xr);
                        if (rescore) sc = sh.s_qv[qi] + xr - 2.f * sc;  // ranking only: rescored below
                        sh.S[qi][ri] = sc;
                    }
                }
                __syncthreads();
                // warp w keeps queries 4w .. 4w + 3
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int qi = warp * 4 + j;
#pragma unroll
                    for (int b = 0; b < FR / 32; ++b) {
                        const int64_t r = t0 + 32 * b + lane;
                        st[j].offer(sh.S[qi][32 * b + lane], r, r < r1, kk, largest, lane);
                    }
                }
            }
            if (rescore) {
                // direct (q - x)^2 of the kept rows, then their best k
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t qq = sh.s_q[warp * 4 + j];
                    const bool has = qq >= 0 && lane < kk && st[j].id != INT64_MAX;
                    float dist = INFINITY;
                    if (has) {
                        const T* qp = q + qq * ldq;
                        const TX* xp = rows + st[j].id * ldx;
                        float a = 0.f;
                        int c = 0;
                        if (vec_q && vec_x) {
#pragma unroll 8
                            for (; c + 4 <= d; c += 4) {
                                const float4 u = load4f<T>(qp + c, true, 4);
                                const float4 v = load_row4<TX>(xp + c, st[j].id, x_scale, true, 4);
                                float df = u.x - v.x;
                                a = fmaf(df, df, a);
                                df = u.y - v.y;
                                a = fmaf(df, df, a);
                                df = u.z - v.z;
                                a = fmaf(df, df, a);
                                df = u.w - v.w;
                                a = fmaf(df, df, a);
                            }
                        }
                        for (; c < d; ++c) {
                            float xe = to_f<TX>(xp[c]);
                            if constexpr (sizeof(TX) == 1) xe = __fmul_rn(__ldg(x_scale + st[j].id), xe);
                            const float df = to_f<T>(qp[c]) - xe;
                            a = fmaf(df, df, a);
                        }
                        dist = a;
                    }
                    WarpTopK fin;
                    fin.init(false);
                    fin.offer(dist, st[j].id, has, k, false, lane);
                    st[j] = fin;
                }
            }
            // write the (query, probe slot) lists
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int qi = warp * 4 + j;
                const int64_t qq = sh.s_q[qi];
                if (qq >= 0 && lane < k) {
                    const int64_t o = ((int64_t)sh.s_p[qi] * Q + qq) * k + lane;
                    const bool has = st[j].id != INT64_MAX;
                    out_v[o] = st[j].v;
                    out_i[o] = has ? (ids ? ids[st[j].id] : st[j].id) : -1;
                }
            }
        }
    }
}

// ------------------------------------------------------------- PQ encode

// One thread per (row, subspace): argmin over codewords of the sequential
// fused-FMA squared distance to the residual sub-vector (ties: lower codeword).
__global__ void pq_encode_kernel(const float* __restrict__ x, int64_t n, int64_t ldx, int d,
                                 const int32_t* __restrict__ labels, const float* __restrict__ centroids,
                                 const float* __restrict__ codebooks, int M, int ksub, uint8_t* __restrict__ codes) {
    extern __shared__ float cb[];  // [M][ksub][dsub]
    const int dsub = d / M;
    for (int i = threadIdx.x; i < M * ksub * dsub; i += blockDim.x) cb[i] = codebooks[i];
    __syncthreads();
    const int64_t pairs = n * M;
    for (int64_t pi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; pi < pairs; pi += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = pi / M;
        const int m = (int)(pi % M);
        const float* xr = x + row * ldx + m * dsub;
        const float* cr = centroids + (int64_t)labels[row] * d + m * dsub;
        float r[32];
#pragma unroll 4
        for (int u = 0; u < dsub; ++u) r[u] = xr[u] - cr[u];
        const float* cbm = cb + (int64_t)m * ksub * dsub;
        float best = INFINITY;
        int bj = 0;
        for (int j = 0; j < ksub; ++j) {
            const float* p = cbm + j * dsub;
            float s = 0.f;
            for (int u = 0; u < dsub; ++u) {
                const float t = r[u] - p[u];
                s = fmaf(t, t, s);
            }
            if (s < best) {
                best = s;
                bj = j;
            }
        }
        codes[row * M + m] = (uint8_t)bj;
    }
}

// ------------------------------------------------------------- IVF-PQ scan

constexpr int PNT = 512;
constexpr int PNW = PNT / 32;

__global__ void __launch_bounds__(PNT) ivfpq_scan_kernel(
    const float* __restrict__ q, int64_t Q, int64_t ldq, int d, int nprobe, const int64_t* __restrict__ eperm,
    const int64_t* __restrict__ eseg, const float* __restrict__ centroids, const float* __restrict__ codebooks, int M,
    int ksub, const uint8_t* __restrict__ codes, const int64_t* __restrict__ list_off,
    const int64_t* __restrict__ list_end, int nlist,
    const int64_t* __restrict__ ids, int k, float* __restrict__ out_v, int64_t* __restrict__ out_i) {
    extern __shared__ float psm[];
    const int dsub = d / M;
    float* cb = psm;                                  // M * ksub * dsub
    float* lut = cb + (size_t)M * ksub * dsub;        // M * ksub
    float* res = lut + (size_t)M * ksub;              // d
    unsigned long long* mkey = reinterpret_cast<unsigned long long*>(
        (reinterpret_cast<uintptr_t>(res + ((d + 3) & ~3)) + 7) & ~uintptr_t(7));  // PNW * kMaxIvfK
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // codebooks transposed to [m][u][j]: the LUT build reads them with
    // consecutive codewords j in consecutive threads (no bank conflicts)
    for (int i = tid; i < M * ksub * dsub; i += PNT) {
        const int m = i / (ksub * dsub), r = i % (ksub * dsub), j = r / dsub, u = r % dsub;
        cb[((size_t)m * dsub + u) * ksub + j] = codebooks[i];
    }
    __syncthreads();
    const bool m16 = (M % 16) == 0;

    for (int l = blockIdx.x; l < nlist; l += gridDim.x) {
        const int64_t e0 = eseg[l], e1 = eseg[l + 1];
        const int64_t r0 = list_off[l], r1 = list_end ? list_end[l] : list_off[l + 1];
        const float* cl = centroids + (int64_t)l * d;
        for (int64_t e = e0; e < e1; ++e) {
            const int64_t ent = eperm[e];
            const int64_t qq = ent / nprobe;
            const int p = (int)(ent % nprobe);
            __syncthreads();
            for (int t = tid; t < d; t += PNT) res[t] = q[qq * ldq + t] - cl[t];
            __syncthreads();
            // LUT[m][j] = |res_m - codeword_mj|^2
            for (int i = tid; i < M * ksub; i += PNT) {
                const int m = i / ksub, j = i % ksub;
                const float* pv = cb + (size_t)m * dsub * ksub + j;
                const float* rv = res + m * dsub;
                float s = 0.f;
                for (int u = 0; u < dsub; ++u) {
                    const float t = rv[u] - pv[(size_t)u * ksub];
                    s = fmaf(t, t, s);
                }
                lut[i] = s;
            }
            __syncthreads();
            WarpTopK st;
            st.init(false);
            // rows of the list, 32 per warp step (one 128-bit code load per row when M % 16 == 0)
            for (int64_t base = r0 + (int64_t)warp * 32; base < r1; base += (int64_t)PNT) {
                const int64_t row = base + lane;
                float dist = INFINITY;
                const bool valid = row < r1;
                if (valid) {
                    const uint8_t* cr = codes + row * M;
                    dist = 0.f;
                    if (m16) {
                        for (int m0 = 0; m0 < M; m0 += 16) {
                            const uint4 w4 = *reinterpret_cast<const uint4*>(cr + m0);
                            const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                            for (int b = 0; b < 16; ++b) {
                                const uint32_t c = (w[b >> 2] >> (8 * (b & 3))) & 0xffu;
                                dist += lut[(m0 + b) * ksub + c];
                            }
                        }
                    } else {
                        for (int m = 0; m < M; ++m) dist += lut[m * ksub + cr[m]];
                    }
                }
                st.offer(dist, row, valid, k, false, lane);
            }
            // merge the warps' sorted lists: block bitonic sort of the
            // PNW x k (score key, row) keys, best k written out
            if (lane < kMaxIvfK) {
                const bool has = lane < k && st.id != INT64_MAX;
                mkey[warp * kMaxIvfK + lane] =
                    has ? (((unsigned long long)float_asc_key(st.v) << 32) | (uint32_t)st.id) : ~0ull;
            }
            __syncthreads();
            for (int size = 2; size <= PNW * kMaxIvfK; size <<= 1)
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    const int t = tid, o = tid ^ stride;
                    if (o > t) {
                        const bool up = (t & size) == 0;
                        const unsigned long long a = mkey[t], b = mkey[o];
                        if ((a > b) == up) {
                            mkey[t] = b;
                            mkey[o] = a;
                        }
                    }
                    __syncthreads();
                }
            if (tid < k) {
                const unsigned long long key = mkey[tid];
                const int64_t o = ((int64_t)p * Q + qq) * k + tid;
                const bool has = key != ~0ull;
                out_v[o] = has ? asc_key_float((uint32_t)(key >> 32)) : INFINITY;
                const int64_t row = (int64_t)(uint32_t)key;
                out_i[o] = has ? (ids ? ids[row] : row) : -1;
            }
        }
    }
}

}  // namespace

IvfWs ivf_ws(int64_t Q, int nprobe, int nlist) {
    IvfWs w;
    const int64_t ne = Q * nprobe;
    size_t off = 0;
    w.off_lab = off;
    off = align_up(off + sizeof(int32_t) * std::max<int64_t>(ne, 1), 256);
    w.off_perm = off;
    off = align_up(off + sizeof(int64_t) * std::max<int64_t>(ne, 1), 256);
    w.off_seg = off;
    off = align_up(off + sizeof(int64_t) * (nlist + 1), 256);
    w.off_qv = off;
    off = align_up(off + sizeof(float) * std::max<int64_t>(Q, 1), 256);
    w.off_sort = off;
    off = align_up(off + label_sort_workspace(ne, nlist), 256);
    w.bytes = off;
    return w;
}

// group the Q x nprobe probe entries by list
int invert_probes(const int64_t* probe, int64_t Q, int nprobe, int nlist, const IvfWs& w, char* base,
                  cudaStream_t s) {
    const int64_t ne = Q * nprobe;
    int32_t* lab = reinterpret_cast<int32_t*>(base + w.off_lab);
    probe_to_labels_kernel<<<(unsigned)((ne + 255) / 256), 256, 0, s>>>(probe, ne, nlist, lab);
    RDB_LAUNCH_CHECK();
    return label_sort(lab, ne, nlist, reinterpret_cast<int64_t*>(base + w.off_seg),
                      reinterpret_cast<int64_t*>(base + w.off_perm), nullptr, base + w.off_sort,
                      label_sort_workspace(ne, nlist), s);
}

namespace {

template <typename T, typename TX = T>
int ivf_flat_smem_attr(int bytes) {
    RDB_CUDA_TRY(cudaFuncSetAttribute(ivf_flat_scan_kernel<T, true, TX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      bytes));
    RDB_CUDA_TRY(cudaFuncSetAttribute(ivf_flat_scan_kernel<T, false, TX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      bytes));
    return RDB_OK;
}

template <typename T, typename TX = T>
void launch_ivf_flat(bool expand, dim3 grid, cudaStream_t s, int metric, int cos_small, const void* q, int64_t nq,
                     int64_t ldq, int d, const float* qv, int nprobe, const int64_t* eperm, const int64_t* eseg,
                     const void* rows, int64_t ldx, const float* x_scale, const float* xv, const int64_t* list_off,
                     const int64_t* list_end, int nlist,
                     const int64_t* ids, int k, float* out_v, int64_t* out_i) {
    auto kern = expand ? ivf_flat_scan_kernel<T, true, TX> : ivf_flat_scan_kernel<T, false, TX>;
    kern<<<grid, FNT, sizeof(IvfFlatSmem), s>>>(metric, cos_small, static_cast<const T*>(q), nq, ldq, d, qv, nprobe,
                                                eperm, eseg, static_cast<const TX*>(rows), ldx, x_scale, xv, list_off,
                                                list_end, nlist,
                                                ids, k, out_v, out_i);
}

bool g_ivf_flat_attr[64] = {false};

// shared-memory opt-in of the list-scan kernels, once per device
int ivf_flat_attrs() {
    int dev = 0;
    RDB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && g_ivf_flat_attr[dev]) return RDB_OK;
    const int bytes = (int)sizeof(IvfFlatSmem);
    RDB_TRY(ivf_flat_smem_attr<float>(bytes));
    RDB_TRY(ivf_flat_smem_attr<__half>(bytes));
    RDB_TRY(ivf_flat_smem_attr<__nv_bfloat16>(bytes));
    RDB_TRY((ivf_flat_smem_attr<float, int8_t>(bytes)));
    if (dev >= 0 && dev < 64) g_ivf_flat_attr[dev] = true;
    return RDB_OK;
}

size_t pq_smem(int d, int M, int ksub) {
    return sizeof(float) * ((size_t)ksub * d + (size_t)M * ksub + ((d + 3) & ~3)) +
           sizeof(unsigned long long) * (PNW * kMaxIvfK + 1);
}

}  // namespace

// Loads every kernel rdb_ivf_flat_scan can launch into the current context
// and sets their attributes (CUDA loads kernels lazily, on first use).
int ivf_flat_scan_preload() {
    RDB_TRY(ivf_flat_attrs());
    cudaFuncAttributes fa;
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, probe_to_labels_kernel));
    RDB_TRY(label_sort_preload());
    return norms_preload();
}

}  // namespace rdb

using namespace rdb;

extern "C" {

size_t rdb_ivf_scan_workspace(int64_t nq, int nprobe, int nlist) { return ivf_ws(nq, nprobe, nlist).bytes; }

}  // extern "C"

namespace rdb {
namespace {

// x_scale != NULL: rows are SQ8 codes (int8, stride ldx bytes) with per-row
// scales, queries fp32
int ivf_flat_scan_impl(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d, const int64_t* probe,
                       int nprobe, const void* rows, int64_t ldx, const float* x_scale, const float* xv,
                       const int64_t* list_off, const int64_t* list_end, int nlist, const int64_t* ids, int k,
                       float* out_v, int64_t* out_i, void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(metric >= 0 && metric <= 2, "unknown metric %d", metric);
    RDB_CHECK_ARG(elem_size(dtype) != 0, "unknown dtype %d", dtype);
    RDB_CHECK_ARG(nq >= 0 && d >= 1 && nprobe >= 1 && nlist >= 1 && nlist <= kMaxLabels, "bad shape");
    RDB_CHECK_ARG(k >= 1 && k <= kMaxIvfK, "IVF search supports k in [1, %d]", kMaxIvfK);
    if (nq == 0) return RDB_OK;
    RDB_CHECK_ARG(q && probe && list_off && out_v && out_i && ws, "NULL pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    IvfWs w = ivf_ws(nq, nprobe, nlist);
    if (ws_bytes < w.bytes) return set_error(RDB_ERR_WORKSPACE, "workspace too small: %zu < %zu", ws_bytes, w.bytes);
    char* base = static_cast<char*>(ws);
    RDB_TRY(invert_probes(probe, nq, nprobe, nlist, w, base, s));
    float* qv = reinterpret_cast<float*>(base + w.off_qv);
    const int cos_small = d <= 128 ? 1 : 0;
    // L2 with k <= kL2ExpandMaxK ranks by |q|^2 + |x|^2 - 2 q.x, then rescores
    const bool expand = metric != RDB_METRIC_L2 || (k <= kL2ExpandMaxK && xv != nullptr);
    if (metric == RDB_METRIC_COSINE || (metric == RDB_METRIC_L2 && expand)) {
        RDB_CHECK_ARG(xv, "cosine needs per-row values");
        RDB_TRY(row_sqnorms_ld(dtype, q, nq, d, ldq, qv, s));
        if (metric == RDB_METRIC_COSINE) RDB_TRY(rdb_vec_values(metric, d, qv, nq, qv, s));
    }
    // x: lists; y: CTAs sharing a list's query chunks, ~4x the mean chunk count
    const int64_t mean_chunks = (nq * nprobe + (int64_t)nlist * FQ - 1) / ((int64_t)nlist * FQ);
    const dim3 grid((unsigned)nlist, (unsigned)std::min<int64_t>(64, std::max<int64_t>(1, 4 * mean_chunks)));
    const int64_t* eperm = reinterpret_cast<const int64_t*>(base + w.off_perm);
    const int64_t* eseg = reinterpret_cast<const int64_t*>(base + w.off_seg);
    RDB_TRY(ivf_flat_attrs());
    cudaEvent_t stop_ev;
    RDB_TRY(timing_begin(TIMING_IVF_SCAN, s, &stop_ev));
    if (x_scale) {
        launch_ivf_flat<float, int8_t>(expand, grid, s, metric, cos_small, q, nq, ldq, d, qv, nprobe, eperm, eseg, rows,
                                       ldx, x_scale, xv, list_off, list_end, nlist, ids, k, out_v, out_i);
    } else {
        switch (dtype) {
            case RDB_F32:
                launch_ivf_flat<float>(expand, grid, s, metric, cos_small, q, nq, ldq, d, qv, nprobe, eperm, eseg,
                                       rows, ldx, nullptr, xv, list_off, list_end, nlist, ids, k, out_v, out_i);
                break;
            case RDB_F16:
                launch_ivf_flat<__half>(expand, grid, s, metric, cos_small, q, nq, ldq, d, qv, nprobe, eperm, eseg,
                                        rows, ldx, nullptr, xv, list_off, list_end, nlist, ids, k, out_v, out_i);
                break;
            default:
                launch_ivf_flat<__nv_bfloat16>(expand, grid, s, metric, cos_small, q, nq, ldq, d, qv, nprobe, eperm,
                                               eseg, rows, ldx, nullptr, xv, list_off, list_end, nlist, ids, k, out_v,
                                               out_i);
        }
    }
    RDB_LAUNCH_CHECK();
    if (stop_ev) RDB_CUDA_TRY(cudaEventRecord(stop_ev, s));
    return RDB_OK;
}

}  // namespace
}  // namespace rdb

extern "C" {

int rdb_ivf_flat_scan(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d, const int64_t* probe,
                      int nprobe, const void* rows, int64_t ldx, const float* xv, const int64_t* list_off,
                      const int64_t* list_end, int nlist,
                      const int64_t* ids, int k, float* out_v, int64_t* out_i, void* ws, size_t ws_bytes,
                      void* stream) {
    return ivf_flat_scan_impl(metric, dtype, q, nq, ldq, d, probe, nprobe, rows, ldx, nullptr, xv, list_off, list_end,
                              nlist, ids, k, out_v, out_i, ws, ws_bytes, stream);
}

int rdb_ivf_flat_scan_sq8(int metric, const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe,
                          int nprobe, const int8_t* codes, int64_t ldx, const float* scales, const float* xv,
                          const int64_t* list_off, const int64_t* list_end, int nlist, const int64_t* ids, int k,
                          float* out_v, int64_t* out_i, void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(scales != nullptr, "scales is NULL");
    RDB_CHECK_ARG(ldx % 4 == 0, "SQ8 row stride must be a multiple of 4 bytes");
    return ivf_flat_scan_impl(metric, RDB_F32, q, nq, ldq, d, probe, nprobe, codes, ldx, scales, xv, list_off,
                              list_end, nlist, ids, k, out_v, out_i, ws, ws_bytes, stream);
}

int rdb_pq_encode(const float* x, int64_t n, int64_t ldx, int d, const int32_t* labels, const float* centroids,
                  const float* codebooks, int M, int ksub, uint8_t* codes, void* stream) {
    RDB_CHECK_ARG(n >= 0 && d >= 1 && M >= 1 && d % M == 0, "d must be a multiple of M");
    RDB_CHECK_ARG(d / M <= 32, "sub-vector dimension d / M must be <= 32");
    RDB_CHECK_ARG(ksub >= 1 && ksub <= 256, "ksub must be in [1, 256] (8-bit codes)");
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(x && labels && centroids && codebooks && codes, "NULL pointer");
    const size_t smem = sizeof(float) * (size_t)ksub * d;
    RDB_CHECK_ARG(smem <= 200 * 1024, "codebooks too large for shared memory (ksub * d <= 51200)");
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        RDB_CUDA_TRY(cudaFuncSetAttribute(pq_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr[dev] = true;
    }
    const int64_t pairs = n * M;
    const unsigned grid = (unsigned)std::min<int64_t>((pairs + 255) / 256, 4LL * num_sms());
    pq_encode_kernel<<<grid, 256, smem, static_cast<cudaStream_t>(stream)>>>(x, n, ldx, d, labels, centroids,
                                                                           codebooks, M, ksub, codes);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int rdb_ivfpq_scan(const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe, int nprobe,
                   const float* centroids, int nlist, const float* codebooks, int M, int ksub, const uint8_t* codes,
                   const int64_t* list_off, const int64_t* list_end, const int64_t* ids, int k, float* out_v,
                   int64_t* out_i, void* ws,
                   size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(nq >= 0 && d >= 1 && M >= 1 && d % M == 0, "d must be a multiple of M");
    RDB_CHECK_ARG(ksub >= 1 && ksub <= 256, "ksub must be in [1, 256]");
    RDB_CHECK_ARG(nprobe >= 1 && nlist >= 1 && nlist <= kMaxLabels, "bad shape");
    RDB_CHECK_ARG(k >= 1 && k <= kMaxIvfK, "IVF-PQ search supports k in [1, %d]", kMaxIvfK);
    if (nq == 0) return RDB_OK;
    RDB_CHECK_ARG(q && probe && centroids && codebooks && codes && list_off && out_v && out_i && ws, "NULL pointer");
    const size_t smem = pq_smem(d, M, ksub);
    RDB_CHECK_ARG(smem <= 220 * 1024, "codebooks + tables too large for shared memory");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    IvfWs w = ivf_ws(nq, nprobe, nlist);
    if (ws_bytes < w.bytes) return set_error(RDB_ERR_WORKSPACE, "workspace too small: %zu < %zu", ws_bytes, w.bytes);
    char* base = static_cast<char*>(ws);
    RDB_TRY(invert_probes(probe, nq, nprobe, nlist, w, base, s));
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        RDB_CUDA_TRY(cudaFuncSetAttribute(ivfpq_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
        attr[dev] = true;
    }
    const unsigned grid = (unsigned)std::min<int64_t>(nlist, (int64_t)num_sms());
    cudaEvent_t stop_ev;
    RDB_TRY(timing_begin(TIMING_PQ_SCAN, s, &stop_ev));
    ivfpq_scan_kernel<<<grid, PNT, smem, s>>>(q, nq, ldq, d, nprobe, reinterpret_cast<const int64_t*>(base + w.off_perm),
                                            reinterpret_cast<const int64_t*>(base + w.off_seg), centroids, codebooks, M,
                                            ksub, codes, list_off, list_end, nlist, ids, k, out_v, out_i);
    RDB_LAUNCH_CHECK();
    if (stop_ev) RDB_CUDA_TRY(cudaEventRecord(stop_ev, s));
    return RDB_OK;
}

}  // extern "C"
