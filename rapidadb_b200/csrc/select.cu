// Per-query top-k selection: one CTA per query, or one warp per query for
// small outputs over few elements (select_warp_kernel).
//
// Every element gets a unique 64-bit key  (score key << 32) | index  that
// sorts ascending best-first (csrc/kernels/topk.cu:25 semantics: sorted,
// largest for cosine / dot, smallest for L2; ties go to the lower index).  An
// MSD radix select finds the k-th smallest key in a few passes over the
// elements (shared-memory cached when they fit), the k winners are gathered
// and bitonic-sorted in shared memory.  For L2 over stored vectors the winners
// (plus a margin) are re-scored exactly as sum (q - x)^2 before the final
// sort, which is the reference formula (csrc/kernels/distance.cu:414-438).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "select.cuh"

namespace rdb {
namespace {

constexpr int NT = 256;
constexpr int NWARP = NT / 32;
constexpr int kCacheKeys = 8192;  // keys cached in shared memory when T fits
constexpr int kMaxSeg = 1024;
constexpr int kDigit = 11;  // radix digit width
constexpr int kBins = 1 << kDigit;

struct SelShared {
    int seg_off[kMaxSeg + 1];
    int hist[kBins];
    int wsum[NWARP];
    unsigned long long red_min[NWARP];
    unsigned long long red_max[NWARP];
    unsigned long long prefix;
    int top;
    int remaining;
    int done;
    int nsel;
    int total;
};

__device__ __forceinline__ float load_as_float(int dtype, const void* p, int64_t i) {
    if (dtype == RDB_F32) return static_cast<const float*>(p)[i];
    if (dtype == RDB_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(static_cast<const __half*>(p)[i]);
}

// Element t of stored (physical) row prow as a float: SQ8 codes are
// dequantised with their row's scale (a rounded product, never fused).
__device__ __forceinline__ float load_row_elem(const SelectArgs& a, int64_t prow, int t) {
    if (a.x_i8)
        return __fmul_rn(__ldg(a.x_scale + prow),
                         static_cast<float>(static_cast<const int8_t*>(a.xdata)[prow * a.ldx + t]));
    return load_as_float(a.dtype, a.xdata, prow * a.ldx + t);
}

__device__ __forceinline__ bool hi_eq(unsigned long long a, unsigned long long b, int top) {
    return top >= 64 ? true : ((a >> top) == (b >> top));
}

// Id of element t of merge list g, query q.
__device__ __forceinline__ int64_t merge_id(const SelectArgs& a, int g, int64_t q, int t) {
    const int64_t ld = a.ldi ? a.ldi : a.kin;
    const int64_t gs = a.gstride_i ? a.gstride_i : a.nq * ld;
    return a.merge_i[(int64_t)g * gs + q * ld + t];
}

// Key of element t of segment seg of query q.
__device__ __forceinline__ unsigned long long seg_key(const SelectArgs& a, int64_t q, int seg, int t,
                                                      float qv) {
    const bool largest = a.largest != 0;
    if (a.input == SEL_CANDIDATES) {
        // candidates carry their final score (computed by the scan epilogue)
        uint2 c = a.cand[((int64_t)seg * a.nq + q) * a.cap + t];
        return ((unsigned long long)score_key(__uint_as_float(c.x), largest) << 32) | c.y;
    } else if (a.input == SEL_DENSE) {
        float s = a.dense[q * a.dense_n + t];
        return ((unsigned long long)score_key(s, largest) << 32) | (uint32_t)t;
    } else {
        const int64_t ld = a.ldv ? a.ldv : a.kin;
        const int64_t gs = a.gstride_v ? a.gstride_v : a.nq * ld;
        float s = a.merge_v[(int64_t)seg * gs + q * ld + t];
        return ((unsigned long long)score_key(s, largest) << 32) | (uint32_t)(seg * a.kin + t);
    }
}

// Walks elements e = threadIdx.x, +NT, ... of query q; the segment of e is
// tracked with a monotone cursor (each thread's e only grows).
struct ElemCursor {
    int seg = 0;
    __device__ __forceinline__ unsigned long long key(const SelectArgs& a, const SelShared& S,
                                                      int64_t q, int e, float qv) {
        while (e >= S.seg_off[seg + 1]) ++seg;
        return seg_key(a, q, seg, e - S.seg_off[seg], qv);
    }
};

__device__ void bitonic_sort(unsigned long long* keys, int n /* power of two */) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n >> 1); i += NT) {
                int lo = 2 * i - (i & (stride - 1));
                int hi = lo + stride;
                bool up = ((lo & size) == 0);
                unsigned long long x = keys[lo], y = keys[hi];
                if ((x > y) == up) {
                    keys[lo] = y;
                    keys[hi] = x;
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ int next_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

// seven CTAs per SM (32 registers, a few bytes spilled): with the key cache
// sized from the expected count, 148 x 7 = 1,036 queries run in one wave
__global__ void __launch_bounds__(NT, 7) select_kernel(SelectArgs a) {
    extern __shared__ __align__(16) unsigned char dsm[];
    __shared__ SelShared S;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool largest = a.largest != 0;
    const int out_k_req = a.k + a.rescore_margin;
    const int sel_cap = next_pow2(out_k_req > 0 ? out_k_req : 1);
    unsigned long long* sel = reinterpret_cast<unsigned long long*>(dsm);
    unsigned long long* cache = sel + sel_cap;

    if (a.gate && *a.gate == 0) return;
    for (int64_t q = blockIdx.x; q < a.nq; q += gridDim.x) {
        if (a.only_q && a.only_q[q] == 0) continue;  // uniform across the CTA
        // ---- segment offsets -------------------------------------------
        if (warp == 0) {
            int nseg = a.input == SEL_DENSE ? 1 : (a.input == SEL_MERGE ? a.G : a.nsplit);
            int per = (nseg + 31) / 32;
            int b0 = lane * per, b1 = min(b0 + per, nseg);
            int local = 0;
            bool ovf = false;
            for (int s = b0; s < b1; ++s) {
                int len;
                if (a.input == SEL_CANDIDATES) {
                    int c = a.counts[(int64_t)s * a.nq + q];
                    ovf |= (int64_t)c > a.cap;
                    len = (int)min((int64_t)c, a.cap);
                } else if (a.input == SEL_DENSE) {
                    len = (int)a.dense_n;
                } else {
                    len = a.kin;
                }
                S.seg_off[s] = local;  // provisional (local prefix)
                local += len;
            }
            if (ovf && a.overflow) atomicOr(a.overflow, 1u);
            if (a.mark_q) {
                const bool any_ovf = __any_sync(0xffffffffu, ovf);
                if (lane == 0) a.mark_q[q] = any_ovf ? 1u : 0u;
            }
            int incl = local;
            for (int o = 1; o < 32; o <<= 1) {
                int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            int excl = incl - local;
            for (int s = b0; s < b1; ++s) S.seg_off[s] += excl;
            if (lane == 31) {
                S.seg_off[nseg] = incl;
                S.total = incl;
            }
        }
        __syncthreads();
        const int T = S.total;
        const float qv = (a.input == SEL_CANDIDATES && a.qv) ? a.qv[q] : 0.f;
        const int want = min(out_k_req, T);  // elements to select
        const bool cached = T <= a.cache_keys;

        // ---- pass 0: keys (cached) and min / max ---------------------------
        unsigned long long kmin = ~0ull, kmax = 0ull;
        ElemCursor cur0;
        for (int e = threadIdx.x; e < T; e += NT) {
            unsigned long long key = cur0.key(a, S, q, e, qv);
            if (cached) cache[e] = key;
            kmin = min(kmin, key);
            kmax = max(kmax, key);
        }
        for (int o = 16; o > 0; o >>= 1) {
            kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
            kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
        }
        if (lane == 0) {
            S.red_min[warp] = kmin;
            S.red_max[warp] = kmax;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long mn = ~0ull, mx = 0ull;
            for (int w = 0; w < NWARP; ++w) {
                mn = min(mn, S.red_min[w]);
                mx = max(mx, S.red_max[w]);
            }
            S.prefix = mn;
            S.remaining = want;
            S.nsel = 0;
            // all elements selected, or nothing to select: finish immediately
            if (want >= T || want == 0) {
                S.done = 1;
                S.top = 0;
                S.prefix = mx;  // every key <= max
            } else {
                unsigned long long diff = mn ^ mx;
                S.top = diff ? 64 - __clzll(diff) : 0;  // bits >= top are common
                S.done = diff ? 0 : 1;
            }
        }
        __syncthreads();

        // ---- MSD radix select: 11-bit digits from the highest bit that differs
        int rounds = 0;
        while (!S.done) {
            const int top = S.top;
            const int shift = top > kDigit ? top - kDigit : 0;
            const unsigned width_mask = (1u << (top - shift)) - 1u;
            const unsigned long long prefix = S.prefix;
            const int rem = S.remaining;  // read before the owner below rewrites it
            for (int i = threadIdx.x; i < kBins; i += NT) S.hist[i] = 0;
            __syncthreads();
            ElemCursor cur;
            for (int e = threadIdx.x; e < T; e += NT) {
                const unsigned long long key = cached ? cache[e] : cur.key(a, S, q, e, qv);
                if (hi_eq(key, prefix, top)) atomicAdd(&S.hist[(key >> shift) & width_mask], 1);
            }
            __syncthreads();
            // block-wide scan of the bins: thread t owns bins [8t, 8t + 8)
            constexpr int PER = kBins / NT;
            int c[PER];
            int local = 0;
#pragma unroll
            for (int j = 0; j < PER; ++j) {
                c[j] = S.hist[threadIdx.x * PER + j];
                local += c[j];
            }
            int incl = local;
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            if (lane == 31) S.wsum[warp] = incl;
            __syncthreads();
            int before = 0;
            for (int w = 0; w < warp; ++w) before += S.wsum[w];
            incl += before;
            const int excl = incl - local;
            if (excl < rem && rem <= incl) {
                int cum = excl, b = 0;
#pragma unroll
                for (int j = 0; j < PER; ++j) {
                    if (cum + c[j] >= rem) {
                        b = threadIdx.x * PER + j;
                        break;
                    }
                    cum += c[j];
                }
                const int nrem = rem - cum;
                const int cnt_b = S.hist[b];
                const unsigned long long mask = (unsigned long long)width_mask << shift;
                S.prefix = (prefix & ~mask) | ((unsigned long long)b << shift);
                S.remaining = nrem;
                S.top = shift;
                S.done = (cnt_b == nrem || shift == 0) ? 1 : 0;
            }
            __syncthreads();
            if (++rounds >= 8 && threadIdx.x == 0) S.done = 1;  // 64-bit keys need <= 6 rounds
            __syncthreads();
        }

        // ---- gather the winners: (key >> top) <= (prefix >> top) ------------
        {
            const int top = S.top;
            const unsigned long long pref = top >= 64 ? 0ull : (S.prefix >> top);
            ElemCursor cur;
            for (int e = threadIdx.x; e < T; e += NT) {
                unsigned long long key = cached ? cache[e] : cur.key(a, S, q, e, qv);
                bool take = top >= 64 ? true : ((key >> top) <= pref);
                if (take) {
                    int slot = atomicAdd(&S.nsel, 1);
                    if (slot < sel_cap) sel[slot] = key;
                }
            }
        }
        __syncthreads();
        int nsel = min(S.nsel, sel_cap);

        // ---- exact L2 re-scoring of the winners --------------------------
        if (a.rescore_margin > 0 && a.input == SEL_CANDIDATES && a.metric == RDB_METRIC_L2) {
            for (int i = warp; i < nsel; i += NWARP) {
                unsigned long long key = sel[i];
                uint32_t row = (uint32_t)key;
                int64_t prow = (int64_t)row * a.row_step;
                float acc = 0.f;
                for (int t = lane; t < a.d; t += 32) {
                    float df = load_as_float(a.dtype, a.qdata, q * a.ldq + t) -
                               load_row_elem(a, prow, t);
                    acc = fmaf(df, df, acc);
                }
                for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (lane == 0) sel[i] = ((unsigned long long)score_key(acc, false) << 32) | row;
            }
            __syncthreads();
        }

        // ---- sort + write -------------------------------------------------
        if (a.output == SEL_OUT_THRESHOLD) {
            // the k-th best score (winners hold exactly min(k, T) keys)
            unsigned long long m = 0ull;
            for (int i = threadIdx.x; i < nsel; i += NT) m = max(m, sel[i]);
            for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) S.red_max[warp] = m;
            __syncthreads();
            if (threadIdx.x == 0) {
                unsigned long long mm = 0ull;
                for (int w = 0; w < NWARP; ++w) mm = max(mm, S.red_max[w]);
                float thr = (nsel >= a.k && nsel > 0) ? key_score((uint32_t)(mm >> 32), largest)
                                                      : (largest ? -INFINITY : INFINITY);
                a.out_thr[q] = thr;
            }
        } else {
            int P = next_pow2(nsel > 0 ? nsel : 1);
            for (int i = nsel + threadIdx.x; i < P; i += NT) sel[i] = ~0ull;
            __syncthreads();
            bitonic_sort(sel, P);
            for (int i = threadIdx.x; i < a.k; i += NT) {
                float v;
                int64_t id;
                if (i < nsel) {
                    unsigned long long key = sel[i];
                    v = key_score((uint32_t)(key >> 32), largest);
                    uint32_t idx = (uint32_t)key;
                    if (a.input == SEL_CANDIDATES) {
                        int64_t prow = (int64_t)idx * a.row_step;
                        id = a.ids ? a.ids[prow] : prow + a.id_offset;
                    } else if (a.input == SEL_DENSE) {
                        id = idx;
                    } else {
                        int g = idx / a.kin, t = idx % a.kin;
                        id = merge_id(a, g, q, t);
                    }
                } else {
                    v = largest ? -INFINITY : INFINITY;
                    id = -1;
                }
                a.out_v[q * a.k + i] = v;
                a.out_i[q * a.k + i] = id;
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Warp-per-query selection for small outputs (k + margin <= 128) over at most
// kWarpSeg segments: eight queries per CTA, no block barriers, same keys and
// results as select_kernel.  The want-th smallest score key s* is found by an
// MSD radix select over the 32-bit score keys (8-bit digits, per-warp
// shared-memory histogram); when more elements tie at s* than are needed, a
// second radix select over their indices keeps the lowest.  Up to 1024
// elements per query are held in registers; more are streamed from global
// memory / L2 on every pass.  Winners are gathered in shared memory and
// each goes to the output position given by its rank.

constexpr int kWarpSeg = 64;
constexpr int kWarpOut = 128;

constexpr int kWarpCache = 1024;       // elements per query kept on chip (registers for a dense row)
constexpr int kWarpCacheSmall = 512;   // the small instance: shared memory only, four CTAs per SM

template <int CACHE>
struct WarpSelT {
    int seg_off[kWarpSeg + 1];
    int hist[256];
    int nsel;
    unsigned long long sel[kWarpOut];
    unsigned long long cache[CACHE];  // element keys when T <= CACHE
};

// One histogram pass + bucket search.  Elements are offered through `each`
// (calls fn(key64) for every element of the query).  Among elements with
// pred(key), digit ((field(key) >> shift) & 255) is counted; returns the bucket
// holding the remaining-th smallest field value and updates remaining / the
// count of that bucket.
template <class WarpSel, class Each, class Pred, class Field>
__device__ __forceinline__ uint32_t warp_radix_pass(WarpSel& W, int lane, Each&& each, Pred&& pred, Field&& field,
                                                    int shift, uint32_t match_mask, uint32_t match_val,
                                                    int& remaining, int& cnt_b) {
    const unsigned FULLM = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < 8; ++i) W.hist[lane * 8 + i] = 0;
    __syncwarp();
    each([&](unsigned long long key) {
        const uint32_t f = field(key);
        if (pred(key) && (f & match_mask) == match_val) atomicAdd(&W.hist[(f >> shift) & 255u], 1);
    });
    __syncwarp();
    int c[8], local = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        c[i] = W.hist[lane * 8 + i];
        local += c[i];
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(FULLM, incl, o);
        if (lane >= o) incl += v;
    }
    const int excl = incl - local;
    const unsigned own = __ballot_sync(FULLM, excl < remaining && remaining <= incl);
    const int src = own ? __ffs(own) - 1 : 31;
    int b = 255, before = 0, cb = 0;
    if (lane == src && own) {
        before = excl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (before + c[i] >= remaining) {
                b = lane * 8 + i;
                cb = c[i];
                break;
            }
            before += c[i];
        }
    }
    b = __shfl_sync(FULLM, b, src);
    before = __shfl_sync(FULLM, before, src);
    cb = __shfl_sync(FULLM, cb, src);
    remaining -= before;
    cnt_b = cb;
    __syncwarp();
    return static_cast<uint32_t>(b);
}

// want-th smallest 32-bit field among elements with pred (want >= 1 and at
// most the number of such elements); fmin / fmax bound the field values.
// Returns the value; remaining = how many elements equal to it are needed,
// cnt_eq = how many there are.
template <class WarpSel, class Each, class Pred, class Field>
__device__ __forceinline__ uint32_t warp_select32(WarpSel& W, int lane, Each&& each, Pred&& pred, Field&& field,
                                                  uint32_t fmin, uint32_t fmax, int want, int& remaining,
                                                  int& cnt_eq) {
    uint32_t val = fmin;
    remaining = want;
    cnt_eq = 0;
    const uint32_t diff = fmin ^ fmax;
    int top = diff ? 32 - __clz(diff) : 0;  // bits >= top are common to all
    if (top == 0) {
        // a single value: count it
        int n = 0;
        each([&](unsigned long long key) { n += pred(key) ? 1 : 0; });
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
        cnt_eq = n;
        return val;
    }
    while (top > 0) {
        const int shift = top > 8 ? top - 8 : 0;
        const uint32_t match_mask = top >= 32 ? 0u : (0xffffffffu << top);
        int cb = 0;
        const uint32_t b = warp_radix_pass(W, lane, each, pred, field, shift, match_mask, val & match_mask, remaining,
                                           cb);
        const uint32_t dmask = (top - shift >= 32 ? 0xffffffffu : ((1u << (top - shift)) - 1u)) << shift;
        val = (val & ~dmask) | (b << shift);
        top = shift;
        cnt_eq = cb;
    }
    return val;
}

// CACHE = kWarpCache: up to 1024 elements on chip (a dense row in
// registers), two CTAs per SM; CACHE = kWarpCacheSmall: up to 512, all in
// shared memory (about 6.5 KB per warp), four CTAs per SM, for the small
// candidate lists of row-sharded searches.
template <int CACHE>
__global__ void __launch_bounds__(NT, (CACHE <= kWarpCacheSmall ? 4 : 2)) select_warp_kernel(SelectArgs a) {
    using WarpSel = WarpSelT<CACHE>;
    constexpr bool kRegDense = CACHE == kWarpCache;
    extern __shared__ __align__(16) unsigned char wsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    WarpSel& W = reinterpret_cast<WarpSel*>(wsm)[warp];
    const unsigned FULLM = 0xffffffffu;
    const bool largest = a.largest != 0;
    const int out_k_req = a.k + a.rescore_margin;
    const int nseg = a.input == SEL_DENSE ? 1 : (a.input == SEL_MERGE ? a.G : a.nsplit);

    if (a.gate && *a.gate == 0) return;
    for (int64_t q = (int64_t)blockIdx.x * NWARP + warp; q < a.nq; q += (int64_t)gridDim.x * NWARP) {
        if (a.only_q && a.only_q[q] == 0) continue;  // uniform across the warp
        // ---- segment offsets (two segments per lane at most)
        int len[2] = {0, 0};
        bool ovf = false;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int sgi = lane + 32 * h;
            if (sgi < nseg) {
                if (a.input == SEL_CANDIDATES) {
                    const int c = a.counts[(int64_t)sgi * a.nq + q];
                    ovf |= (int64_t)c > a.cap;
                    len[h] = (int)min((int64_t)c, a.cap);
                } else if (a.input == SEL_DENSE) {
                    len[h] = (int)a.dense_n;
                } else {
                    len[h] = a.kin;
                }
            }
        }
        {
            const bool any_ovf = __any_sync(FULLM, ovf);
            if (any_ovf && lane == 0 && a.overflow) atomicOr(a.overflow, 1u);
            if (a.mark_q && lane == 0) a.mark_q[q] = any_ovf ? 1u : 0u;
        }
        int base = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int incl = len[h];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(FULLM, incl, o);
                if (lane >= o) incl += v;
            }
            if (lane + 32 * h < kWarpSeg) W.seg_off[lane + 32 * h] = base + incl - len[h];
            base += __shfl_sync(FULLM, incl, 31);
        }
        if (lane == 0) {
            W.seg_off[min(nseg, kWarpSeg)] = base;
            W.nsel = 0;
        }
        __syncwarp();
        const int T = base;
        const float qv = (a.input == SEL_CANDIDATES && a.qv) ? a.qv[q] : 0.f;
        const int want = min(out_k_req, T);

        // element keys: a dense row of <= kWarpCache scores in registers
        // (element lane + 32 i: score key kh[i]; CACHE = kWarpCache only),
        // other inputs of <= CACHE elements copied once into W.cache, larger
        // ones re-read from global memory / L2 on every pass
        const int mode = T > CACHE ? 0 : ((kRegDense && a.input == SEL_DENSE) ? 1 : 2);
        uint32_t kh[kRegDense ? kWarpCache / 32 : 1];
        if (kRegDense && mode == 1) {
#pragma unroll
            for (int i = 0; i < kWarpCache / 32; ++i) {
                const int e = lane + 32 * i;
                kh[i] = e < T ? score_key(a.dense[q * a.dense_n + e], largest) : 0xffffffffu;
            }
        } else if (mode == 2) {
            for (int sgi = 0; sgi < nseg; ++sgi) {
                const int o = W.seg_off[sgi], n = W.seg_off[sgi + 1] - o;
                for (int t = lane; t < n; t += 32) W.cache[o + t] = seg_key(a, q, sgi, t, qv);
            }
            __syncwarp();
        }
        auto each = [&](auto&& fn) {
            if (kRegDense && mode == 1) {
#pragma unroll
                for (int i = 0; i < kWarpCache / 32; ++i) {
                    const int e = lane + 32 * i;
                    if (e < T) fn((static_cast<unsigned long long>(kh[i]) << 32) | static_cast<uint32_t>(e));
                }
            } else if (mode == 2) {
                for (int e = lane; e < T; e += 32) fn(W.cache[e]);
            } else {
                int sgc = 0;
                for (int e = lane; e < T; e += 32) {
                    while (e >= W.seg_off[sgc + 1]) ++sgc;
                    fn(seg_key(a, q, sgc, e - W.seg_off[sgc], qv));
                }
            }
        };
        auto& each_score = each;
        auto hi32 = [](unsigned long long key) { return static_cast<uint32_t>(key >> 32); };
        auto lo32 = [](unsigned long long key) { return static_cast<uint32_t>(key); };
        auto all = [](unsigned long long) { return true; };

        // ---- s* = want-th smallest score key, then the index bound r* among ties
        uint32_t s_star = 0xffffffffu, r_star = 0xffffffffu;
        bool any = want > 0;
        if (any && want < T) {
            uint32_t mn = 0xffffffffu, mx = 0u;
            each_score([&](unsigned long long key) {
                mn = min(mn, hi32(key));
                mx = max(mx, hi32(key));
            });
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mn = min(mn, __shfl_xor_sync(FULLM, mn, o));
                mx = max(mx, __shfl_xor_sync(FULLM, mx, o));
            }
            int rem = 0, cnt_eq = 0;
            s_star = warp_select32(W, lane, each_score, all, hi32, mn, mx, want, rem, cnt_eq);
            if (a.output == SEL_OUT_TOPK && cnt_eq > rem) {
                // more ties at s* than needed: keep the rem lowest indices
                auto tie = [&](unsigned long long key) { return hi32(key) == s_star; };
                uint32_t rmn = 0xffffffffu, rmx = 0u;
                each([&](unsigned long long key) {
                    if (tie(key)) {
                        rmn = min(rmn, lo32(key));
                        rmx = max(rmx, lo32(key));
                    }
                });
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    rmn = min(rmn, __shfl_xor_sync(FULLM, rmn, o));
                    rmx = max(rmx, __shfl_xor_sync(FULLM, rmx, o));
                }
                int rem2 = 0, cnt2 = 0;
                r_star = warp_select32(W, lane, each, tie, lo32, rmn, rmx, rem, rem2, cnt2);
            }
        }

        if (a.output == SEL_OUT_THRESHOLD) {
            // the k-th best score: s*, or the largest key when every element wins
            uint32_t mx = 0u;
            if (any && want >= T) {
                each_score([&](unsigned long long key) { mx = max(mx, hi32(key)); });
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(FULLM, mx, o));
            } else {
                mx = s_star;
            }
            if (lane == 0)
                a.out_thr[q] = (want >= a.k && want > 0) ? key_score(mx, largest) : (largest ? -INFINITY : INFINITY);
            __syncwarp();
            continue;
        }

        // ---- gather the winners: score < s*, or score == s* and index <= r*
        each([&](unsigned long long key) {
            const uint32_t h = hi32(key);
            if (h < s_star || (h == s_star && lo32(key) <= r_star)) {
                const int slot = atomicAdd(&W.nsel, 1);
                if (slot < kWarpOut) W.sel[slot] = key;
            }
        });
        __syncwarp();
        const int nsel = min(W.nsel, kWarpOut);
        // ---- exact L2 re-scoring of the winners (one winner per warp step)
        if (a.rescore_margin > 0 && a.input == SEL_CANDIDATES && a.metric == RDB_METRIC_L2) {
            for (int i = 0; i < nsel; ++i) {
                const unsigned long long key = W.sel[i];
                const uint32_t row = (uint32_t)key;
                const int64_t prow = (int64_t)row * a.row_step;
                float acc = 0.f;
                for (int t = lane; t < a.d; t += 32) {
                    const float df = load_as_float(a.dtype, a.qdata, q * a.ldq + t) -
                                     load_row_elem(a, prow, t);
                    acc = fmaf(df, df, acc);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULLM, acc, o);
                if (lane == 0) W.sel[i] = ((unsigned long long)score_key(acc, false) << 32) | row;
                __syncwarp();
            }
        }
        // ---- winner i goes to position rank(i) = #winners with a smaller key
        for (int i = lane; i < nsel; i += 32) {
            const unsigned long long key = W.sel[i];
            int rank = 0;
            for (int j = 0; j < nsel; ++j) rank += W.sel[j] < key ? 1 : 0;
            if (rank < a.k) {
                const float v = key_score((uint32_t)(key >> 32), largest);
                const uint32_t idx = (uint32_t)key;
                int64_t id;
                if (a.input == SEL_CANDIDATES) {
                    const int64_t prow = (int64_t)idx * a.row_step;
                    id = a.ids ? a.ids[prow] : prow + a.id_offset;
                } else if (a.input == SEL_DENSE) {
                    id = idx;
                } else {
                    const int g = idx / a.kin, t = idx % a.kin;
                    id = merge_id(a, g, q, t);
                }
                a.out_v[q * a.k + rank] = v;
                a.out_i[q * a.k + rank] = id;
            }
        }
        for (int i = nsel + lane; i < a.k; i += 32) {
            a.out_v[q * a.k + i] = largest ? -INFINITY : INFINITY;
            a.out_i[q * a.k + i] = -1;
        }
        __syncwarp();
    }
}

}  // namespace

int launch_select(const SelectArgs& a, cudaStream_t stream) {
    if (a.nq <= 0) return RDB_OK;
    int out_k = a.k + a.rescore_margin;
    RDB_CHECK_ARG(a.k >= 1 && out_k <= kMaxK + 64, "k must be in [1, %d], got %d", kMaxK, a.k);
    if (a.input == SEL_CANDIDATES)
        RDB_CHECK_ARG(a.nsplit >= 1 && a.nsplit <= kMaxSeg, "nsplit %d out of range", a.nsplit);
    if (a.input == SEL_MERGE)
        RDB_CHECK_ARG(a.G >= 1 && a.G <= kMaxSeg, "G %d out of range", a.G);
    int P = 1;
    while (P < out_k) P <<= 1;
    // the CTA kernel caches up to kCacheKeys keys per query in shared memory;
    // with an expected count it holds that many plus an eighth and 256 (the
    // count's spread is about its square root), so more CTAs fit on an SM;
    // a query with more elements reads them again from global memory / L2
    SelectArgs ac = a;
    ac.cache_keys = kCacheKeys;
    if (a.expect > 0)
        ac.cache_keys = (int)std::min<int64_t>(kCacheKeys, (a.expect + a.expect / 8 + 256 + 63) / 64 * 64);
    size_t smem = sizeof(unsigned long long) * ((size_t)P + ac.cache_keys);
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
        size_t maxdyn = sizeof(unsigned long long) * (8192 + 64 + kCacheKeys);
        RDB_CUDA_TRY(cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)maxdyn));
        attr_set[dev] = true;
    }
    const int nseg = a.input == SEL_DENSE ? 1 : (a.input == SEL_MERGE ? a.G : a.nsplit);
    // small outputs over few elements per query: one warp per query
    const int64_t max_elems = a.input == SEL_DENSE ? a.dense_n
                              : a.input == SEL_MERGE ? (int64_t)a.G * a.kin
                                                     : a.cap * a.nsplit;
    // a warp re-reads elements beyond its on-chip cache on every pass: larger
    // expected inputs go to the CTA kernel, and so do expected counts above
    // kWarpExpect, where the CTA kernel (seven per SM, keys sized to the
    // count) selects faster (B200: 1,024 queries x ~1,680 candidates in
    // 36 us against 2,048 x ~840 in 72 us for the warp kernel)
    constexpr int64_t kWarpExpect = 512;
    constexpr int64_t kWarpSmallExpect = 384;  // counts rarely above 512 (spread ~ sqrt(expect))
    const bool small = a.expect > 0 ? a.expect <= kWarpExpect : max_elems <= 32768;
    // fewer queries than SMs: a CTA per query spreads them over the GPU (the
    // warp kernel would occupy nq / 8 SMs)
    const bool many = a.nq >= num_sms();
    if (!a.force_cta && out_k <= kWarpOut && nseg <= kWarpSeg && small && many) {
        const int64_t blocks = (a.nq + NWARP - 1) / NWARP;
        const unsigned nb = (unsigned)std::min<int64_t>(blocks, 65535LL * 16);
        // expected counts well under 512 (the per-rank lists of row-sharded
        // searches): the small instance, twice the warps per SM
        if (a.expect > 0 && a.expect <= kWarpSmallExpect) {
            static bool wattr_small[64] = {false};
            if (dev < 64 && !wattr_small[dev]) {
                RDB_CUDA_TRY(cudaFuncSetAttribute(select_warp_kernel<kWarpCacheSmall>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)(sizeof(WarpSelT<kWarpCacheSmall>) * NWARP)));
                wattr_small[dev] = true;
            }
            select_warp_kernel<kWarpCacheSmall><<<nb, NT, sizeof(WarpSelT<kWarpCacheSmall>) * NWARP, stream>>>(a);
        } else {
            static bool wattr[64] = {false};
            if (dev < 64 && !wattr[dev]) {
                RDB_CUDA_TRY(cudaFuncSetAttribute(select_warp_kernel<kWarpCache>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)(sizeof(WarpSelT<kWarpCache>) * NWARP)));
                wattr[dev] = true;
            }
            select_warp_kernel<kWarpCache><<<nb, NT, sizeof(WarpSelT<kWarpCache>) * NWARP, stream>>>(a);
        }
        RDB_LAUNCH_CHECK();
        return RDB_OK;
    }
    int64_t grid = a.nq < 65535 * 4 ? a.nq : 65535 * 4;
    if (a.force_cta) grid = std::min<int64_t>(grid, num_sms());
    select_kernel<<<(unsigned)grid, NT, smem, stream>>>(ac);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // namespace rdb
