// Query-major IVF-PQ search (squared L2, residual product quantisation).
//
// The reference has no IVF-PQ code (python/rapidadb/config.py:50-56 declares
// nlist / nprobe / pq_m / pq_k and nothing reads them); the scores follow the
// CPU oracle's asymmetric distance (oracle/cpu_oracle.c: orc_ivfpq_search),
//
//   dist(q, row) = sum_m |(q - c_l)_m - cb[m][code_m]|^2,
//
// regrouped so that a query's lookup table does not depend on the list:
//
//   dist = |q - c_l|^2 + T[row] + sum_m QT[m][code_m]
//   T[row]    = sum_m |cb[m][code_m]|^2 + 2 <(c_l)_m, cb[m][code_m]>  (once per
//               stored row, rdb_pq_row_terms, at add time)
//   QT[m][j]  = -2 <q_m, cb[m][j]>                                   (once per
//               query, in shared memory)
//
// so one CTA builds QT once and scans all nprobe lists of the query with no
// per-(query, list) table.  QT is held as 32-bit fixed point (a power-of-two
// scale per query, |sum| < 2^30): the code sum is exact integer arithmetic, so
// rows with identical codes in one list score identically whatever order the
// lanes add in, and ties fall to the lower stored row as in the oracle.  The
// regrouping and the fixed point change rounding only (~1e-7 of the terms);
// codes, centroids and codebooks are the oracle's.
//
// Conflict-free table lookups: in each group of G = min(M, 32) code bytes,
// row i is stored rotated by i mod G (stored byte s = code[(i + s) mod G]).
// A warp scores 32 consecutive rows whose first row is a multiple of 32, so at
// step s lane L reads subquantiser (L + s) mod G; the table holds NC = 32 / G
// copies of each entry arranged so that the 32 lanes of a step hit 32
// different banks whatever the codes are (layout below, before pq_smem).
#include <algorithm>

#include "scan.cuh"
#include "sort.cuh"

namespace rdb {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr int SNT = 512;
constexpr int SNW = SNT / 32;
constexpr int kMaxPqK = 32;
constexpr int kMaxPqProbe = 4096;
constexpr int RPL = 4;  // rows per lane in a scan chunk (chunks of 128 rows)
constexpr int kMaxPqSmem = 227 * 1024;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <int M>
struct PqLayout {
    static constexpr int G = M < 32 ? M : 32;  // rotation group
    static constexpr int NC = 32 / G;          // table copies
    static constexpr int NG = M / G;           // groups per code
    static_assert(M % G == 0 && 32 % G == 0, "M must be a power of two <= 32 or a multiple of 32");
};

// Best k 64-bit keys of a warp, ascending: lane i holds the i-th smallest;
// kth (every lane) caches lane k - 1's key, refreshed after insertions.
struct WarpKeys {
    unsigned long long key, kth;
    __device__ __forceinline__ void init() { key = kth = ~0ull; }
    __device__ __forceinline__ void offer(unsigned long long c, bool valid, int k, int lane) {
        unsigned m = __ballot_sync(FULL, valid && c < kth);
        if (!m) return;
        do {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const unsigned long long x = __shfl_sync(FULL, c, src);
            if (x >= kth) continue;
            const int pos = __popc(__ballot_sync(FULL, lane < k && key < x));
            const unsigned long long prev = __shfl_up_sync(FULL, key, 1);
            if (lane == pos)
                key = x;
            else if (lane > pos && lane < k)
                key = prev;
            kth = __shfl_sync(FULL, key, k - 1);
        } while (m);
    }
};

template <int M>
__device__ __forceinline__ void load_codes(const uint8_t* p, uint32_t (&w)[M / 4]) {
    if constexpr (M % 16 == 0) {
#pragma unroll
        for (int i = 0; i < M / 16; ++i) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + i);
            w[4 * i] = v.x;
            w[4 * i + 1] = v.y;
            w[4 * i + 2] = v.z;
            w[4 * i + 3] = v.w;
        }
    } else if constexpr (M == 8) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
        w[0] = v.x;
        w[1] = v.y;
    } else {
        w[0] = __ldg(reinterpret_cast<const unsigned int*>(p));
    }
}

// Table layout: per group g of G subquantisers, 256 rows (one per code value j)
// of 64 words.  Word w of row j holds QT[g G + (w / NC) mod G][j] (copy w mod NC):
// positions m' = w / NC in [0, 2 G) so that lane L at step s reads position
// (L mod G) + s without wrapping, at byte  256 j + 4 (NC (L mod G) + L / G) + 4 NC s:
// a per-lane base, the code placed in bits 8..15 by one byte permute, and a
// compile-time offset.  For each s the 32 lanes hit 32 different banks.
constexpr int kRowWords = 64;
constexpr int kGroupWords = 256 * kRowWords;

struct PqSmem {
    size_t lut, mk, r0, r1, qs, t1, red, pfx, bytes;
};

PqSmem pq_smem(int M, int d, int nprobe) {
    PqSmem s;
    const int G = M < 32 ? M : 32;
    size_t off = 0;
    s.lut = off;  // at offset 0: lookups address it as pq_shared + (lane offset | code << 8)
    off += sizeof(uint32_t) * (size_t)(M / G) * kGroupWords;
    s.mk = off;
    off += sizeof(unsigned long long) * SNW * kMaxPqK;
    s.r0 = off;
    off += sizeof(uint32_t) * nprobe;
    s.r1 = off;
    off += sizeof(uint32_t) * nprobe;
    s.qs = off;
    off += sizeof(float) * ((d + 3) & ~3);
    s.t1 = off;
    off += sizeof(float) * nprobe;
    s.red = off;
    off += sizeof(float) * SNW;
    s.pfx = off;
    off += sizeof(int) * (nprobe + 1);
    s.bytes = align_up(off, 16);
    return s;
}

template <int M>
__global__ void __launch_bounds__(SNT, (M <= 32 ? 2 : 1)) ivfpq_search_kernel(
    const float* __restrict__ q, int64_t Q, int64_t ldq, int d, const int64_t* __restrict__ probe, int nprobe,
    const float* __restrict__ centroids, int nlist, const float* __restrict__ codebooks, int ksub,
    const uint8_t* __restrict__ codes, const float* __restrict__ row_terms, const int64_t* __restrict__ list_off,
    const int64_t* __restrict__ list_end,
    const int64_t* __restrict__ ids, const int64_t* __restrict__ order, int k, PqSmem sm, float* __restrict__ out_v,
    int64_t* __restrict__ out_i) {
    using L = PqLayout<M>;
    extern __shared__ __align__(16) unsigned char pq_shared[];
    uint32_t* lut = reinterpret_cast<uint32_t*>(pq_shared + sm.lut);  // fp32 bits, then fixed point
    unsigned long long* mk = reinterpret_cast<unsigned long long*>(pq_shared + sm.mk);
    uint32_t* r0s = reinterpret_cast<uint32_t*>(pq_shared + sm.r0);
    uint32_t* r1s = reinterpret_cast<uint32_t*>(pq_shared + sm.r1);
    float* qs = reinterpret_cast<float*>(pq_shared + sm.qs);
    float* t1 = reinterpret_cast<float*>(pq_shared + sm.t1);
    float* red = reinterpret_cast<float*>(pq_shared + sm.red);
    int* pfx = reinterpret_cast<int*>(pq_shared + sm.pfx);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dsub = d / M;
    // this lane's byte offset in a table row: word NC (lane mod G) + lane / G
    // (< 256; the table starts at offset 0 of the dynamic shared memory)
    const uint32_t lane_off = 4u * (L::NC * (lane % L::G) + lane / L::G);

    for (int64_t w = blockIdx.x; w < Q; w += gridDim.x) {
        const int64_t qi = order ? order[w] : w;
        __syncthreads();  // the previous query is done with shared memory
        for (int t = tid; t < d; t += SNT) qs[t] = q[qi * ldq + t];
        for (int p = tid; p < nprobe; p += SNT) {
            const int64_t l = probe[qi * nprobe + p];
            uint32_t r0 = 0, r1 = 0;
            if (l >= 0 && l < nlist) {
                r0 = static_cast<uint32_t>(list_off[l]);
                r1 = static_cast<uint32_t>(list_end ? list_end[l] : list_off[l + 1]);
            }
            r0s[p] = r0;
            r1s[p] = r1;
            // chunks of 32 * RPL rows from the 32-aligned row at or below r0
            pfx[p + 1] = r1 > r0 ? static_cast<int>((r1 - (r0 & ~31u) + (32u * RPL - 1)) / (32u * RPL)) : 0;
        }
        __syncthreads();
        if (warp == 0) {
            // chunk prefix over the probes (in place)
            int carry = 0;
            for (int p0 = 0; p0 < nprobe; p0 += 32) {
                const int p = p0 + lane;
                int v = p < nprobe ? pfx[p + 1] : 0;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int u = __shfl_up_sync(FULL, v, o);
                    if (lane >= o) v += u;
                }
                if (p < nprobe) pfx[p + 1] = v + carry;
                carry += __shfl_sync(FULL, v, 31);
            }
            if (lane == 0) pfx[0] = 0;
        }
        // |q - c_l|^2 per probe
        for (int p = warp; p < nprobe; p += SNW) {
            const int64_t l = probe[qi * nprobe + p];
            float s = 0.f;
            if (l >= 0 && l < nlist) {
                const float* cp = centroids + l * d;
                for (int t = lane; t < d; t += 32) {
                    const float df = qs[t] - __ldg(cp + t);
                    s = fmaf(df, df, s);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
            if (lane == 0) t1[p] = s;
        }
        // QT[m][j] = -2 <q_m, cb[m][j]>: every thread computes whole entries
        // (entry e = j M + m, so the lanes of a warp cover the M subquantisers
        // of consecutive codes and their table stores fall in distinct
        // banks), the dsub codebook loads of an entry independent of each
        // other; entry (m, j) fills its 2 NC words of table row j of group
        // m / G (word w holds position (w / NC) mod G)
        // M <= 32: a thread's entries (at most M / 2 with ksub <= 256) stay in
        // registers until the scale is known and are written once, in fixed
        // point; wider codes store fp32 entries and convert them in a second
        // pass over the table
        constexpr int KREG = M <= 32 ? (M * 256 + SNT - 1) / SNT : 1;
        float vreg[KREG];
        float amax = 0.f;
        auto entry = [&](int e) -> float {
            const int j = e / M, m = e - j * M;
            const float* cbp = codebooks + (static_cast<int64_t>(m) * ksub + j) * dsub;
            const float* qp = qs + m * dsub;
            float s = 0.f;
            for (int u = 0; u < dsub; ++u) s = fmaf(qp[u], __ldg(cbp + u), s);
            return -2.f * s;
        };
        auto store = [&](int e, uint32_t word) {
            const int j = e / M, m = e - j * M;
            const int g = m / L::G, t = m - g * L::G;
            uint32_t* row = lut + g * kGroupWords + j * kRowWords;
#pragma unroll
            for (int c = 0; c < L::NC; ++c) {
                row[L::NC * t + c] = word;
                row[L::NC * (t + L::G) + c] = word;
            }
        };
        if constexpr (M <= 32) {
#pragma unroll
            for (int i = 0; i < KREG; ++i) {
                const int e = tid + i * SNT;
                vreg[i] = e < M * ksub ? entry(e) : 0.f;
                amax = fmaxf(amax, fabsf(vreg[i]));
            }
        } else {
#pragma unroll 2
            for (int e = tid; e < M * ksub; e += SNT) {
                const float val = entry(e);
                amax = fmaxf(amax, fabsf(val));
                store(e, __float_as_uint(val));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(FULL, amax, o));
        if (lane == 0) red[warp] = amax;
        __syncthreads();
        // fixed point: M * max |QT| * scale < 2^30, scale a power of two
        float bound = 0.f;
#pragma unroll
        for (int i = 0; i < SNW; ++i) bound = fmaxf(bound, red[i]);
        bound *= static_cast<float>(M);
        int ex = 0;
        if (bound > 0.f) frexpf(bound, &ex);  // bound < 2^ex
        ex = max(ex, -90);                    // keep 2^(30 - ex) finite
        const float scale = ldexpf(1.f, 30 - ex), inv_scale = ldexpf(1.f, ex - 30);
        if constexpr (M <= 32) {
#pragma unroll
            for (int i = 0; i < KREG; ++i) {
                const int e = tid + i * SNT;
                if (e < M * ksub) store(e, static_cast<uint32_t>(__float2int_rn(vreg[i] * scale)));
            }
        } else {
            for (int rr = warp; rr < L::NG * ksub; rr += SNW) {
                const int g = rr / ksub, j = rr - g * ksub;
                uint32_t* row = lut + g * kGroupWords + j * kRowWords;
                row[lane] = static_cast<uint32_t>(__float2int_rn(__uint_as_float(row[lane]) * scale));
                row[lane + 32] = static_cast<uint32_t>(__float2int_rn(__uint_as_float(row[lane + 32]) * scale));
            }
        }
        __syncthreads();

        // ---- scan: warps take chunks of 32 * RPL rows of the probed lists in
        // turn (the 16 warps of a CTA read 16 consecutive chunks together);
        // lane L scores rows L, L + 32, ... of its chunk (all rotated alike)
        WarpKeys tk;
        tk.init();
        float kth_d = INFINITY;  // distance of the warp's current k-th best
        const int total = pfx[nprobe];
        int p = 0;
        for (int c = warp; c < total; c += SNW) {
            while (pfx[p + 1] <= c) ++p;
            const uint32_t r0 = r0s[p], r1 = r1s[p];
            const uint32_t base = (r0 & ~31u) + 32u * RPL * static_cast<uint32_t>(c - pfx[p]) + lane;
            uint32_t cw[RPL][M / 4];
            float term[RPL];
            bool valid[RPL];
#pragma unroll
            for (int h = 0; h < RPL; ++h) {
                const uint32_t row = base + 32u * h;
                valid[h] = row >= r0 && row < r1;
                // rows outside the list read the list's first row (always
                // valid) and are masked from the top-k
                const uint32_t rr = valid[h] ? row : r0;
                load_codes<M>(codes + static_cast<size_t>(rr) * M, cw[h]);
                term[h] = __ldg(row_terms + rr);
            }
            uint32_t acc[RPL];
#pragma unroll
            for (int h = 0; h < RPL; ++h) acc[h] = 0;  // two's-complement sums of fixed-point entries
#pragma unroll
            for (int g = 0; g < L::NG; ++g) {
#pragma unroll
                for (int s = 0; s < L::G; ++s) {
                    const int b = g * L::G + s;
#pragma unroll
                    for (int h = 0; h < RPL; ++h) {
                        // byte 0: this lane's word offset, byte 1: the code (= code * 256 bytes)
                        const uint32_t a = __byte_perm(cw[h][b >> 2], lane_off, 0x5504u | ((b & 3) << 4));
                        acc[h] += *reinterpret_cast<const uint32_t*>(pq_shared + a + 4 * (g * kGroupWords + L::NC * s));
                    }
                }
            }
            const float tl = t1[p];
            float dist[RPL];
            bool hit = false;
#pragma unroll
            for (int h = 0; h < RPL; ++h) {
                dist[h] = fmaf(static_cast<float>(static_cast<int>(acc[h])), inv_scale, tl + term[h]);
                hit |= valid[h] && dist[h] <= kth_d;
            }
            if (__any_sync(FULL, hit)) {
#pragma unroll
                for (int h = 0; h < RPL; ++h) {
                    const unsigned long long key =
                        valid[h] ? (static_cast<unsigned long long>(float_asc_key(dist[h])) << 32) | (base + 32u * h)
                                 : ~0ull;
                    tk.offer(key, valid[h], k, lane);
                }
                kth_d = tk.kth == ~0ull ? INFINITY : asc_key_float(static_cast<uint32_t>(tk.kth >> 32));
            }
        }
        if (lane < k) mk[warp * kMaxPqK + lane] = tk.key;
        __syncthreads();
        if (warp == 0) {
            // best k of the SNW warp lists
            WarpKeys f;
            f.init();
            for (int i0 = 0; i0 < SNW * k; i0 += 32) {
                const int i = i0 + lane;
                const unsigned long long key = i < SNW * k ? mk[(i / k) * kMaxPqK + i % k] : ~0ull;
                f.offer(key, key != ~0ull, k, lane);
            }
            if (lane < k) {
                const bool has = f.key != ~0ull;
                const int64_t r = static_cast<int64_t>(static_cast<uint32_t>(f.key));
                out_v[qi * k + lane] = has ? asc_key_float(static_cast<uint32_t>(f.key >> 32)) : INFINITY;
                out_i[qi * k + lane] = has ? (ids ? ids[r] : r) : -1;
            }
        }
    }
}

__global__ void pq_row_terms_kernel(const uint8_t* __restrict__ codes, int64_t n, int M,
                                    const int32_t* __restrict__ labels, const float* __restrict__ centroids,
                                    int d, const float* __restrict__ codebooks, int ksub, float* __restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int dsub = d / M;
    const float* c = centroids + static_cast<int64_t>(labels[i]) * d;
    float s = 0.f;
    for (int m = 0; m < M; ++m) {
        const float* cb = codebooks + (static_cast<int64_t>(m) * ksub + codes[i * M + m]) * dsub;
        for (int u = 0; u < dsub; ++u) {
            const float v = cb[u];
            s = fmaf(v, fmaf(2.f, c[m * dsub + u], v), s);
        }
    }
    out[i] = s;
}

// rotate the bytes of row i by i mod G inside each group of G (inverse undoes it)
__global__ void pq_rotate_kernel(uint8_t* __restrict__ codes, int64_t n, int M, int G, int inverse) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint8_t* r = codes + i * M;
    const int sh = static_cast<int>(i % G);
    uint8_t tmp[32];
    for (int g = 0; g < M / G; ++g) {
        uint8_t* rg = r + g * G;
        for (int s = 0; s < G; ++s) tmp[s] = rg[s];
        for (int s = 0; s < G; ++s) {
            if (inverse)
                rg[(s + sh) % G] = tmp[s];
            else
                rg[s] = tmp[(s + sh) % G];
        }
    }
}

// dst row dest[i] = src row i, rotated by dest[i] mod G when G > 0 (the
// stored layout of pq_rotate_kernel for that row)
__global__ void pq_scatter_kernel(const uint8_t* __restrict__ src, int64_t n, int M, const int64_t* __restrict__ dest,
                                  uint8_t* __restrict__ dst, int G) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t o = dest[i];
    const uint8_t* r = src + i * M;
    uint8_t* w = dst + o * M;
    if (G <= 0) {
        for (int s = 0; s < M; ++s) w[s] = r[s];
        return;
    }
    const int sh = static_cast<int>(o % G);
    for (int g = 0; g < M / G; ++g)
        for (int s = 0; s < G; ++s) w[g * G + s] = r[g * G + (s + sh) % G];
}

__global__ void first_probe_kernel(const int64_t* __restrict__ probe, int64_t nq, int nprobe, int nlist,
                                   int32_t* __restrict__ labels) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nq) return;
    const int64_t l = probe[i * nprobe];
    labels[i] = (l >= 0 && l < nlist) ? static_cast<int32_t>(l) : 0;
}

bool fast_m(int M) { return M == 4 || M == 8 || M == 16 || M == 32 || M == 64 || M == 96; }

struct PqSearchWs {
    size_t off_lab, off_order, off_seg, off_sort, bytes;
};

PqSearchWs pq_search_ws(int64_t nq, int nlist) {
    PqSearchWs w;
    size_t off = 0;
    w.off_lab = off;
    off = align_up(off + sizeof(int32_t) * std::max<int64_t>(nq, 1), 256);
    w.off_order = off;
    off = align_up(off + sizeof(int64_t) * std::max<int64_t>(nq, 1), 256);
    w.off_seg = off;
    off = align_up(off + sizeof(int64_t) * (nlist + 1), 256);
    w.off_sort = off;
    off = align_up(off + label_sort_workspace(nq, nlist), 256);
    w.bytes = off;
    return w;
}

template <int M>
int launch_search(const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe, int nprobe,
                  const float* centroids, int nlist, const float* codebooks, int ksub, const uint8_t* codes,
                  const float* row_terms, const int64_t* list_off, const int64_t* list_end, const int64_t* ids,
                  const int64_t* order, int k,
                  float* out_v, int64_t* out_i, cudaStream_t s) {
    const PqSmem sm = pq_smem(M, d, nprobe);
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        RDB_CUDA_TRY(cudaFuncSetAttribute(ivfpq_search_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kMaxPqSmem));
        attr[dev] = true;
    }
    RDB_CHECK_ARG(sm.bytes <= static_cast<size_t>(kMaxPqSmem),
                  "IVF-PQ search tables need %zu bytes of shared memory (max %d): lower nprobe", sm.bytes, kMaxPqSmem);
    // two CTAs per SM when registers (__launch_bounds__) and 228 KB of shared memory allow
    const int per_sm = (M <= 32 && sm.bytes <= 112 * 1024) ? 2 : 1;
    const int64_t grid = std::min<int64_t>(nq, static_cast<int64_t>(per_sm) * num_sms());
    cudaEvent_t stop_ev;
    RDB_TRY(timing_begin(TIMING_PQ_SCAN, s, &stop_ev));
    ivfpq_search_kernel<M><<<static_cast<unsigned>(grid), SNT, sm.bytes, s>>>(
        q, nq, ldq, d, probe, nprobe, centroids, nlist, codebooks, ksub, codes, row_terms, list_off, list_end, ids, order,
        k,
        sm, out_v, out_i);
    RDB_LAUNCH_CHECK();
    if (stop_ev) RDB_CUDA_TRY(cudaEventRecord(stop_ev, s));
    return RDB_OK;
}

}  // namespace
}  // namespace rdb

using namespace rdb;

extern "C" {

int rdb_pq_fast_layout(int M) { return fast_m(M) ? 1 : 0; }

int rdb_pq_row_terms(const uint8_t* codes, int64_t n, int M, const int32_t* labels, const float* centroids,
                     int d, const float* codebooks, int ksub, float* out_terms, void* stream) {
    RDB_CHECK_ARG(n >= 0 && M >= 1 && d >= M && d % M == 0 && ksub >= 1 && ksub <= 256, "bad PQ shape");
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(codes && labels && centroids && codebooks && out_terms, "NULL pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    pq_row_terms_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(codes, n, M, labels, centroids, d,
                                                                              codebooks, ksub, out_terms);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int rdb_pq_rotate_codes(uint8_t* codes, int64_t n, int M, int inverse, void* stream) {
    RDB_CHECK_ARG(fast_m(M), "no rotated code layout for pq_m = %d", M);
    RDB_CHECK_ARG(n >= 0, "bad row count");
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(codes, "NULL pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int G = M < 32 ? M : 32;
    pq_rotate_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(codes, n, M, G, inverse ? 1 : 0);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int rdb_pq_scatter_codes(const uint8_t* src, int64_t n, int M, const int64_t* dest, uint8_t* dst, int rotated,
                         void* stream) {
    RDB_CHECK_ARG(M >= 1 && n >= 0, "bad shape");
    RDB_CHECK_ARG(!rotated || fast_m(M), "no rotated code layout for pq_m = %d", M);
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(src && dest && dst, "NULL pointer");
    const int G = rotated ? (M < 32 ? M : 32) : 0;
    pq_scatter_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        src, n, M, dest, dst, G);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

size_t rdb_ivfpq_search_workspace(int64_t nq, int nlist) {
    if (nq <= 0 || nlist <= 0) return 256;
    return pq_search_ws(nq, nlist).bytes;
}

int rdb_ivfpq_search(const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe, int nprobe,
                     const float* centroids, int nlist, const float* codebooks, int M, int ksub,
                     const uint8_t* codes, const float* row_terms, const int64_t* list_off, const int64_t* list_end,
                     const int64_t* ids,
                     int k, float* out_v, int64_t* out_i, void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(fast_m(M), "rdb_ivfpq_search needs pq_m in {4, 8, 16, 32, 64, 96}, got %d", M);
    RDB_CHECK_ARG(d >= M && d % M == 0 && ldq >= d, "bad shape");
    RDB_CHECK_ARG(ksub >= 1 && ksub <= 256, "pq_k must be in [1, 256]");
    RDB_CHECK_ARG(k >= 1 && k <= kMaxPqK, "k must be in [1, %d]", kMaxPqK);
    RDB_CHECK_ARG(nprobe >= 1 && nprobe <= kMaxPqProbe, "nprobe must be in [1, %d]", kMaxPqProbe);
    RDB_CHECK_ARG(nlist >= 1 && nlist <= kMaxLabels, "nlist must be in [1, %d]", kMaxLabels);
    if (nq <= 0) return RDB_OK;
    RDB_CHECK_ARG(q && probe && centroids && codebooks && codes && row_terms && list_off && out_v && out_i && ws,
                  "NULL pointer");
    const PqSearchWs w = pq_search_ws(nq, nlist);
    RDB_CHECK_ARG(ws_bytes >= w.bytes, "workspace too small: %zu bytes, need %zu", ws_bytes, w.bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* base = static_cast<char*>(ws);
    // queries ordered by their nearest list: CTAs running at the same time
    // share lists, which then stay in L2
    int32_t* lab = reinterpret_cast<int32_t*>(base + w.off_lab);
    int64_t* order = reinterpret_cast<int64_t*>(base + w.off_order);
    first_probe_kernel<<<static_cast<unsigned>((nq + 255) / 256), 256, 0, s>>>(probe, nq, nprobe, nlist, lab);
    RDB_LAUNCH_CHECK();
    RDB_TRY(label_sort(lab, nq, nlist, reinterpret_cast<int64_t*>(base + w.off_seg), order, nullptr,
                       base + w.off_sort, label_sort_workspace(nq, nlist), s));
    switch (M) {
        case 4:
            return launch_search<4>(q, nq, ldq, d, probe, nprobe, centroids, nlist, codebooks, ksub, codes, row_terms,
                                    list_off, list_end, ids, order, k, out_v, out_i, s);
        case 8:
            return launch_search<8>(q, nq, ldq, d, probe, nprobe, centroids, nlist, codebooks, ksub, codes, row_terms,
                                    list_off, list_end, ids, order, k, out_v, out_i, s);
        case 16:
            return launch_search<16>(q, nq, ldq, d, probe, nprobe, centroids, nlist, codebooks, ksub, codes,
                                     row_terms, list_off, list_end, ids, order, k, out_v, out_i, s);
        case 32:
            return launch_search<32>(q, nq, ldq, d, probe, nprobe, centroids, nlist, codebooks, ksub, codes,
                                     row_terms, list_off, list_end, ids, order, k, out_v, out_i, s);
        case 64:
            return launch_search<64>(q, nq, ldq, d, probe, nprobe, centroids, nlist, codebooks, ksub, codes,
                                     row_terms, list_off, list_end, ids, order, k, out_v, out_i, s);
        default:
            return launch_search<96>(q, nq, ldq, d, probe, nprobe, centroids, nlist, codebooks, ksub, codes,
                                     row_terms, list_off, list_end, ids, order, k, out_v, out_i, s);
    }
}

}  // extern "C"
