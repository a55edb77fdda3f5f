// IVF-Flat list scan on the tcgen05 tensor cores, for fp32 rows with d <= 128.
//
// The CUDA-core list scan (ivf.cu) is a contraction of each list's probing
// queries with the list's rows; here the contraction runs on the tensor cores
// with fp32-level accuracy and the ranking stays exact:
//
//   operands   every fp32 value v of a row (or query) is scaled by a power of
//              two 2^-e (e per row, per query: max |v| 2^-e in [2^13, 2^14),
//              an exact scaling) and split into two fp16 planes,
//              hi = fp16(v 2^-e), lo = fp16(v 2^-e - hi), about 22 significant
//              bits; rows are split once after adds (rdb_f16_split), the
//              probing queries per search, gathered entry by entry (entries =
//              (query, probe slot) pairs grouped by list).
//   contraction q.x ~ 2^(eq + ex) (qh.xh + qh.xl + ql.xh): three
//              tcgen05.mma.kind::f16 per 16-wide K step into an fp32 TMEM
//              accumulator (relative error about 1e-6 of sum |q_i x_i|, below
//              the rounding of an fp32 dot product of length 128).
//   ranking    per entry the best kk = k + 8 rows of the list by that value
//              (L2: |x|^2 - 2 q.x, cosine: the reference's final score, dot:
//              q.x), written to the entry's (query, probe slot) list.
//   answer     ivf_tc_finish_kernel merges a query's nprobe lists into its
//              best kk by ranking value, scores those rows again on CUDA cores
//              with the CUDA-core scan's arithmetic (L2 summed directly as
//              sum (q - x)^2, dot products accumulated in dimension order) and
//              writes the best k, ties to the lower stored row: the merged
//              [nq, k] answer (no per-probe lists, no separate merge).
//
// Work is handed out in units of (list, chunk of 128 entries): a one-block
// kernel lists them, and each CTA of the persistent scan (one per SM) takes
// the next unit from a global counter, so long lists and lists probed by many
// queries spread over the SMs.  Scan kernel roles:
//   warp 0      TMA producer: takes units, publishes them to the other roles
//               through a 4-slot shared-memory queue; loads the unit's query
//               chunk (both planes, whole K) once into a resident buffer, then
//               the list's rows in tiles of 256 through a two-stage ring (both
//               planes of one 64-wide K block per stage); SWIZZLE_128B, no
//               multicast.
//   warp 1      allocates 512 TMEM columns (two 128 x 256 accumulators); one
//               lane issues the MMAs and commits stage / accumulator / buffer
//               releases.
//   warps 2-9   epilogue, two warps per TMEM lane quadrant (32 entries): each
//               reads half of a tile's columns, 32 at a time, into the quad's
//               shared block (entry-major, XOR-swizzled), and after a pair
//               barrier ranks 16 of the quad's entries over all 64 columns
//               with lane = column: a ballot against the entry's kk-th value,
//               and each passing column inserted into the entry's list, held
//               across the warp (lane i: i-th best) -- one shuffle step per
//               insertion.
// Every mbarrier wait is bounded (mbar_wait): a role that gives up sets the
// abort flag and a status bit, and the CTA frees its TMEM and exits.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "ivf.cuh"
#include "sort.cuh"
#include "tc_common.cuh"

namespace rdb {
namespace {

constexpr int TQ = 128;       // entries per task (UMMA M)
constexpr int TR = 256;       // rows per tile (UMMA N)
constexpr int TK = 64;        // fp16 elements per K block: one 128-byte swizzle atom
constexpr int kMaxDp = 128;   // padded dimension limit (query chunk resident in shared memory)
constexpr int kMaxKB = kMaxDp / TK;
constexpr int NSTAGE = 2;
constexpr int EPIW = 8;
constexpr int EPIT = EPIW * 32;
constexpr int NTHR = 64 + EPIT;
constexpr int TMEM_NCOLS = 512;
constexpr int A_BLK = TQ * TK * 2;        // 16 KB: one plane, one K block of the query chunk
constexpr int A_BYTES = 2 * kMaxKB * A_BLK;
constexpr int B_PLANE = TR * TK * 2;      // 32 KB
constexpr int STAGE_BYTES = 2 * B_PLANE;  // both planes of one K block of a row tile
constexpr int BAR_OFF = A_BYTES + NSTAGE * STAGE_BYTES;
constexpr int BAR_BYTES = 256;
constexpr int UQ = 4;                        // unit hand-out slots
constexpr int XS_OFF = BAR_OFF + BAR_BYTES;  // [epilogue warp][row factor, row value][TR / 2] column staging
constexpr int GKMAX = 32;                    // group minima kept per (entry, column half)
constexpr int MG_OFF = XS_OFF + EPIW * TR * 4;  // [4 quads][32 entries][GKMAX] second half's minima
constexpr int TH_OFF = MG_OFF + 4 * 32 * GKMAX * 4;  // [4 quads][32 entries] entry thresholds
constexpr int UR_OFF = TH_OFF + 4 * 32 * 4;  // [UQ] resolved units (rows, entries, tiles)
constexpr int SMEM_BYTES = 1024 + UR_OFF + UQ * 48;
static_assert(SMEM_BYTES <= 232448, "shared memory over 227 KB");
static_assert((11 + 2 * UQ) * 8 + UQ * 4 + 8 <= BAR_BYTES, "barrier region");
constexpr int kMaxKK = 32;  // ranked rows per entry
constexpr int kCap = 32;    // collected rows per (entry, column half)

constexpr int kL2Margin = 8;
constexpr unsigned kNoRow = 0xffffffffu;

__device__ __forceinline__ void mbar_arrive_local(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool epi_and(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pin, pout;\n\t"
        "setp.ne.u32 pin, %1, 0;\n\t"
        "bar.red.and.pred pout, 1, %2, pin;\n\t"
        "selp.u32 %0, 1, 0, pout;\n\t}"
        : "=r"(r)
        : "r"(ok ? 1u : 0u), "n"(EPIT)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void pair_sync(int quad) {
    asm volatile("bar.sync %0, 64;" ::"r"(2 + quad) : "memory");
}

// Power-of-two scale of a vector whose largest |value| is amax: 2^e with
// amax 2^-e in [2^13, 2^14), 1 for a zero vector.
__device__ __forceinline__ float pow2_scale(float amax) {
    if (!(amax > 0.f) || isinf(amax)) return 1.f;
    int e;
    frexpf(amax, &e);  // amax = m 2^e, m in [0.5, 1)
    return ldexpf(1.f, e - 14 < -126 ? -126 : e - 14);  // normal, so that 1 / scale is finite
}

// One warp per vector: scale, hi / lo fp16 planes (columns d .. ldp - 1 zero).
// flag: set when a value is not finite.
__global__ void split_f16_kernel(const float* __restrict__ x, int64_t n, int64_t ldx, int d, __half* __restrict__ hi,
                                 __half* __restrict__ lo, int64_t ldp, float* __restrict__ scale,
                                 const int64_t* __restrict__ gather, int64_t gather_div, unsigned* flag) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n) return;
    const int64_t src = gather ? gather[row] / gather_div : row;
    const float* p = x + src * ldx;
    float amax = 0.f;
    bool finite = true;
    for (int t = lane; t < d; t += 32) {
        const float v = p[t];
        finite &= isfinite(v);
        amax = fmaxf(amax, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    finite = __all_sync(0xffffffffu, finite);
    const float s = pow2_scale(amax), inv = 1.f / s;  // exact: powers of two
    for (int t = lane; t < (int)ldp; t += 32) {
        const float v = t < d ? p[t] * inv : 0.f;
        const __half h = __float2half_rn(v);
        hi[row * ldp + t] = h;
        lo[row * ldp + t] = __float2half_rn(v - __half2float(h));
    }
    if (lane == 0) {
        scale[row] = s;
        if (!finite && flag) atomicOr(flag, 1u);
    }
}

struct IvfTcArgs {
    int metric;
    int cos_small;
    int nkb;                  // K blocks of 64 (padded dimension / 64)
    int planes;               // 2: fp32 values as hi / lo fp16 planes; 1: fp16 / bf16 values as stored
    int kk;                   // ranked rows per entry (k + 8), <= kMaxKK
    const int2* units;        // (list, first entry) of each unit of work
    const int* nunits;
    int* unit_ctr;            // next unit to hand out (zeroed by the unit-table kernel)
    const int64_t* eseg;      // [nlist + 1] entry segments (entries sorted by list)
    const int64_t* eperm;     // [E] entry -> query * nprobe + slot
    int nprobe;
    const int64_t* list_off;  // [nlist + 1]
    const int64_t* list_end;  // [nlist] or NULL
    const float* xv;          // per stored row: |x|^2 (L2), norm (cosine)
    const float* row_scale;   // per stored row: 2^ex
    const float2* colfv;      // per stored row: (f, v) with value = acc * (qf * f) + v (col_factors_kernel)
    const float* qv;          // per query: norm (cosine)
    const float* ent_scale;   // per entry: 2^eq
    float* cand_v;            // [nq * nprobe][2][kCap] ranking values, by (query, slot), column half
    uint32_t* cand_r;         // [nq * nprobe][2][kCap] stored rows
    int* cand_n;              // [nq * nprobe][2] rows collected (> kCap: overflow, the list is rescanned)
    float* dense;             // dense mode: value of entry e, row r at dense[(e - dense_e0) * dense_ld + r]
    int64_t dense_ld, dense_e0, dense_e1;  // dense mode: entries [dense_e0, dense_e1), every unit's "list" a row block
    float* dense_gmin;        // dense mode: minimum of each 32-row group, [entries][dense_ld / 32]
};

// float -> unsigned key with the same order
__device__ __forceinline__ uint32_t fkey(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float tof(float v) { return v; }
__device__ __forceinline__ float tof(__half v) { return __half2float(v); }
__device__ __forceinline__ float tof(__nv_bfloat16 v) { return __bfloat162float(v); }

// (value, row) as one 64-bit key in the order of before(); all ones = empty
__device__ __forceinline__ uint64_t vr_key(float v, uint32_t r) {
    return (static_cast<uint64_t>(fkey(v)) << 32) | r;
}

// Per stored row, the column factor and value of the ranking value
// acc * (qf * f) + v: L2 (-2 s, |x|^2), cosine (-s / xv, 0), dot (-s, 0),
// s the row's power-of-two scale.
__global__ void col_factors_kernel(int metric, const float* __restrict__ row_scale, const float* __restrict__ xv,
                                   int64_t n, float2* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float rs = row_scale ? row_scale[i] : 1.f;
    if (metric == RDB_METRIC_L2)
        out[i] = make_float2(-2.f * rs, xv[i]);
    else if (metric == RDB_METRIC_COSINE)
        out[i] = make_float2(-rs / xv[i], 0.f);
    else
        out[i] = make_float2(-rs, 0.f);
}

// The units of work of one search: each list's entries in chunks of TQ, in
// list order; one block.  Also zeroes the hand-out counter.
__global__ void __launch_bounds__(1024) ivf_tc_units_kernel(const int64_t* __restrict__ eseg, int nlist,
                                                            int2* __restrict__ units, int* nunits, int* ctr) {
    __shared__ int part[1024];
    const int tid = threadIdx.x;
    const int per = (nlist + 1023) / 1024;
    const int l0 = min(nlist, tid * per), l1 = min(nlist, l0 + per);
    int s = 0;
    for (int l = l0; l < l1; ++l) s += static_cast<int>((eseg[l + 1] - eseg[l] + TQ - 1) / TQ);
    part[tid] = s;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
        const int v = tid >= o ? part[tid - o] : 0;
        __syncthreads();
        part[tid] += v;
        __syncthreads();
    }
    int u = part[tid] - s;
    for (int l = l0; l < l1; ++l)
        for (int64_t e = eseg[l]; e < eseg[l + 1]; e += TQ) units[u++] = make_int2(l, static_cast<int>(e));
    if (tid == 1023) {
        *nunits = part[1023];
        *ctr = 0;
    }
}

// Group of rows per minimum in the threshold pass: the largest power of two
// <= 32 that leaves at least 4 kk groups in the list (1 for short lists), so
// that the kk-th smallest minimum sits close to the kk-th smallest value.
__device__ __forceinline__ int group_rows(int64_t n, int kk) {
    int s = 32;
    while (s > 1 && n < static_cast<int64_t>(s) * 4 * kk) s >>= 1;
    return s;
}

// Insert v into the ascending list tv[GK] (values only), dropping the last:
// element i becomes max(min(tv[i], v), tv[i - 1]) -- the old tv[i - 1] when it
// exceeds v (shifted up), v at the insertion point, tv[i] below it; a value
// above tv[GK - 1] leaves the list unchanged.  Branch-free, depth 2.
template <int GK>
__device__ __forceinline__ void insert_sorted(float (&tv)[GK], float v) {
#pragma unroll
    for (int i = GK - 1; i > 0; --i) tv[i] = fmaxf(fminf(tv[i], v), tv[i - 1]);
    tv[0] = fminf(tv[0], v);
}

// Paired fp32 arithmetic (sm_100): two IEEE round-to-nearest operations per
// instruction, each identical to its scalar form.
// A unit of work as the producer resolves it once for the other roles: list
// rows [r0, r1), entries [ec, e1), row tiles.
struct UnitRec {
    int64_t r0, r1, ec, e1;
    int ntiles, pad;
};
static_assert(sizeof(UnitRec) <= 48, "unit record slot");

// A unit whose list fits the two TMEM accumulators (at most two row tiles) is
// computed once: the collecting pass reads the accumulators the threshold
// pass read (no second load and contraction of its tiles).
__device__ __forceinline__ bool unit_reuses_tmem(int ntiles) { return ntiles <= 2; }

// Row tile of step t2 of a unit: the threshold pass walks tiles 0 .. n - 1,
// the collecting pass n - 1 .. 0 (its first tiles are the last ones loaded,
// still in L2).
__device__ __forceinline__ int tile_of(int t2, int ntiles) { return t2 < ntiles ? t2 : 2 * ntiles - 1 - t2; }

// DENSE: one pass that writes every (entry, row) value to a.dense (the coarse
// probe's centroid scan); otherwise the threshold and collecting passes.
template <int METRIC, int GK, bool DENSE>
__global__ void __launch_bounds__(NTHR, 1)
    ivf_tc_scan_kernel(const __grid_constant__ CUtensorMap mqh, const __grid_constant__ CUtensorMap mql,
                       const __grid_constant__ CUtensorMap mxh, const __grid_constant__ CUtensorMap mxl,
                       const IvfTcArgs a, const uint32_t idesc, unsigned* status) {
    extern __shared__ uint8_t ivf_tc_smem[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ivf_tc_smem) + 1023) & ~uintptr_t(1023));
    uint8_t* abuf = smem;
    uint8_t* ring = smem + A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
    uint64_t* empty = full + NSTAGE;
    uint64_t* tfull = empty + NSTAGE;
    uint64_t* tempty = tfull + 2;
    uint64_t* afull = tempty + 2;
    uint64_t* aempty = afull + 1;
    uint64_t* mma_done = aempty + 1;
    uint64_t* ufull = mma_done + 1;
    uint64_t* uempty = ufull + UQ;
    volatile int* unit_slot = reinterpret_cast<volatile int*>(uempty + UQ);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(unit_slot) + UQ);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* xs_s = reinterpret_cast<float*>(smem + XS_OFF);  // [EPIW][2][TR / 2]: row factor, row value
    float* mg_s = reinterpret_cast<float*>(smem + MG_OFF);
    float* th_s = reinterpret_cast<float*>(smem + TH_OFF);
    volatile UnitRec* urec = reinterpret_cast<volatile UnitRec*>(smem + UR_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int c = 0; c < 2; ++c) {
            mbar_init(&tfull[c], 1);
            mbar_init(&tempty[c], EPIW);
        }
        for (int s = 0; s < UQ; ++s) {
            mbar_init(&ufull[s], 1);
            mbar_init(&uempty[s], 1 + EPIW);
        }
        mbar_init(afull, 1);
        mbar_init(aempty, 1);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&mqh);
        tma_prefetch_desc(&mql);
        tma_prefetch_desc(&mxh);
        tma_prefetch_desc(&mxl);
    }
    if (warp == 1) {
        tmem_alloc_t<false>(tmem_slot, TMEM_NCOLS);
        tmem_relinquish_t<false>();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int nkb = a.nkb;
    const int nunits = *a.nunits;
    constexpr int NPASS = DENSE ? 1 : 2;

    // the list range of unit u: rows [r0, r1), entries [ec, e1); its row tiles
    auto unit_info = [&](int u, int64_t& r0, int64_t& r1, int64_t& ec, int64_t& e1) {
        const int2 un = a.units[u];
        const int l = un.x;
        ec = un.y;
        e1 = min(DENSE ? a.dense_e1 : a.eseg[l + 1], ec + TQ);
        r0 = a.list_off[l];
        r1 = a.list_end ? a.list_end[l] : a.list_off[l + 1];
        return r1 > r0 ? static_cast<int>((r1 - r0 + TR - 1) / TR) : 0;
    };

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer
            // each unit's row tiles twice: threshold pass, then collecting pass
            int stage = 0;
            uint32_t phase = 0, at = 0, ui = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool a_pending = false, ok = true;
            for (;;) {
                int u = atomicAdd(a.unit_ctr, 1);
                if (u >= nunits) u = -1;
                const int s = static_cast<int>(ui % UQ);
                if (!mbar_wait(&uempty[s], ((ui / UQ) & 1) ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                int64_t r0 = 0, r1 = 0, ec = 0, e1 = 0;
                const int ntiles = u >= 0 ? unit_info(u, r0, r1, ec, e1) : 0;
                urec[s].r0 = r0;
                urec[s].r1 = r1;
                urec[s].ec = ec;
                urec[s].e1 = e1;
                urec[s].ntiles = ntiles;
                unit_slot[s] = u;
                mbar_arrive_local(&ufull[s]);  // release: the record is visible to the waiting roles
                ++ui;
                if (u < 0) break;
                if (ntiles == 0) continue;
                if (!mbar_wait(aempty, (at & 1) ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(afull, a.planes * nkb * A_BLK);
                for (int kb = 0; kb < nkb; ++kb) {
                    tma_load_2d(&mqh, afull, abuf + kb * A_BLK, kb * TK, static_cast<int>(ec));
                    if (a.planes == 2)
                        tma_load_2d(&mql, afull, abuf + (kMaxKB + kb) * A_BLK, kb * TK, static_cast<int>(ec));
                }
                a_pending = true;
                ++at;
                const int mma_steps = (NPASS == 2 && unit_reuses_tmem(ntiles) ? 1 : NPASS) * ntiles;
                for (int t2 = 0; t2 < mma_steps && ok; ++t2) {
                    const int t = tile_of(t2, ntiles);
                    const int row0 = static_cast<int>(r0 + static_cast<int64_t>(t) * TR);
                    for (int kb = 0; kb < nkb; ++kb) {
                        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        uint8_t* sp = ring + stage * STAGE_BYTES;
                        mbar_arrive_expect_tx(&full[stage], a.planes * B_PLANE);
                        tma_load_2d(&mxh, &full[stage], sp, kb * TK, row0);
                        if (a.planes == 2) tma_load_2d(&mxl, &full[stage], sp + B_PLANE, kb * TK, row0);
                        issued_mask |= 1u << stage;
                        issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                        if (++stage == NSTAGE) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
                if (!ok) break;
            }
            if (!ok) {
                *abort_flag = 1;
                if (status) atomicOr(status, DEV_TIMEOUT_PRODUCER);
                // let the loads tracked by this CTA's barriers land before its
                // shared memory is released
                for (int s = 0; s < NSTAGE; ++s)
                    if (issued_mask & (1u << s)) {
                        const uint64_t t0 = globaltimer_ns();
                        while (!mbar_try_wait(&full[s], (issued_phase >> s) & 1) &&
                               globaltimer_ns() - t0 < kWaitLimitNs) {
                        }
                    }
                if (a_pending) {
                    const uint64_t t0 = globaltimer_ns();
                    while (!mbar_try_wait(afull, (at - 1) & 1) && globaltimer_ns() - t0 < kWaitLimitNs) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0, at = 0, gt = 0, ui = 0;
            bool ok = true, any = false;
            for (;;) {
                const int s = static_cast<int>(ui % UQ);
                if (!mbar_wait(&ufull[s], (ui / UQ) & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                const int u = unit_slot[s];
                const int ntiles = urec[s].ntiles;
                mbar_arrive_local(&uempty[s]);
                ++ui;
                if (u < 0) break;
                if (ntiles == 0) continue;
                if (!mbar_wait(afull, at & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                ++at;
                tc_fence_after();
                const int mma_steps = (NPASS == 2 && unit_reuses_tmem(ntiles) ? 1 : NPASS) * ntiles;
                for (int t2 = 0; t2 < mma_steps && ok; ++t2, ++gt) {
                    const int acc = gt & 1;
                    if (!mbar_wait(&tempty[acc], ((gt >> 1) & 1) ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TR);
                    for (int kb = 0; kb < nkb; ++kb) {
                        if (!mbar_wait(&full[stage], phase, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t ah = make_sdesc(smem_u32(abuf + kb * A_BLK));
                        const uint64_t al = make_sdesc(smem_u32(abuf + (kMaxKB + kb) * A_BLK));
                        const uint32_t b_addr = smem_u32(ring + stage * STAGE_BYTES);
                        const uint64_t bh = make_sdesc(b_addr);
                        const uint64_t bl = make_sdesc(b_addr + B_PLANE);
                        if (a.planes == 2) {
#pragma unroll
                            for (int k = 0; k < TK / 16; ++k) {
                                umma_f16(d_tmem, ah + 2 * k, bh + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                                umma_f16(d_tmem, ah + 2 * k, bl + 2 * k, idesc, 1u);
                                umma_f16(d_tmem, al + 2 * k, bh + 2 * k, idesc, 1u);
                            }
                        } else {
#pragma unroll
                            for (int k = 0; k < TK / 16; ++k)
                                umma_f16(d_tmem, ah + 2 * k, bh + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                        }
                        any = true;
                        umma_commit(&empty[stage]);
                        if (++stage == NSTAGE) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (ok) umma_commit(&tfull[acc]);
                }
                if (!ok) break;
                umma_commit(aempty);  // the query chunk may be replaced
            }
            if (!ok) {
                *abort_flag = 1;
                if (status) atomicOr(status, DEV_TIMEOUT_MMA);
            }
            if (any) {
                // every MMA this thread issued completes before TMEM is freed
                umma_commit(mma_done);
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(mma_done, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
                }
            }
        }
    } else {
        // -------------------------------------------------------- epilogue
        // Warp (quad q, half h): thread = entry 32q + lane of the unit (TMEM
        // lane), columns 128h .. 128h + 127 of each tile, 32 at a time.
        const int ew = warp - 2;
        const int quad = warp & 3;
        const int half = ew >> 2;
        const int kk = a.kk;
        uint32_t gt = 0, ui = 0;
        for (;;) {
            // the one point where the eight epilogue warps agree: every warp
            // leaves here, together, once any role has given up on a wait
            const int s = static_cast<int>(ui % UQ);
            const bool got_unit = mbar_wait(&ufull[s], (ui / UQ) & 1, abort_flag);
            if (!epi_and(got_unit && *abort_flag == 0)) {
                if (!got_unit) {
                    *abort_flag = 1;
                    if (status) atomicOr(status, DEV_TIMEOUT_EPILOGUE);
                }
                break;
            }
            const int u = unit_slot[s];
            const int64_t r0 = urec[s].r0, r1 = urec[s].r1, ec = urec[s].ec, e1 = urec[s].e1;
            const int ntiles = urec[s].ntiles;
            __syncwarp();
            if (lane == 0) mbar_arrive_local(&uempty[s]);
            ++ui;
            if (u < 0) break;
            const int64_t e = ec + quad * 32 + lane;
            const bool evalid = e < e1;
            float qf = 0.f;
            int64_t pe = 0;
            if (evalid) {
                qf = a.ent_scale[e];
                pe = DENSE ? e : a.eperm[e];
                if (METRIC == RDB_METRIC_COSINE) qf /= a.qv[pe / a.nprobe];
            }
            const bool quad_live = ec + quad * 32 < e1;  // same for both warps of the quad
            const int gs = group_rows(r1 - r0, kk);
            float tv[GK];  // smallest group minima of this half (ascending)
#pragma unroll
            for (int i = 0; i < GK; ++i) tv[i] = INFINITY;
            float thr = INFINITY;  // the entry's threshold in the collecting pass
            int cnt = 0;
            float* cv = DENSE ? nullptr : a.cand_v + (pe * 2 + half) * kCap;
            uint32_t* cr = DENSE ? nullptr : a.cand_r + (pe * 2 + half) * kCap;
            // per-column factors of this warp's half of a tile, so that value =
            // acc * (qf * f) + v with the entry's qf: L2 f = -2 * 2^ex, v = |x|^2,
            // qf = 2^eq; cosine f = -2^ex / xv, v = 0, qf = 2^eq / qv; dot
            // f = -2^ex, v = 0, qf = 2^eq.  Lane L loads columns L + 32 j; the
            // warp stages them in its own shared buffer (no cross-warp barrier).
            float* wst = xs_s + ew * TR;  // [f: TR / 2][v: TR / 2]
            auto load_cols = [&](int t, float2 (&fv)[4]) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t r = r0 + static_cast<int64_t>(t) * TR + half * (TR / 2) + lane + 32 * j;
                    fv[j] = r < r1 ? __ldg(a.colfv + r) : make_float2(0.f, 0.f);
                }
            };
            // two tiles of column factors in flight ahead of the tile being ranked
            const int nsteps = NPASS * ntiles;
            float2 fv1[4], fv2[4];
            if (nsteps > 0) load_cols(tile_of(0, ntiles), fv1);
            if (nsteps > 1) load_cols(tile_of(1, ntiles), fv2);
            bool live = true;  // false once a wait gave up: the unit is walked without work
            // tile instance of step t2 in the MMA's sequence: one per step, or one
            // per tile when the collecting pass re-reads the accumulators
            const bool reuse = NPASS == 2 && unit_reuses_tmem(ntiles);
            const uint32_t gt0 = gt;
            for (int t2 = 0; t2 < nsteps; ++t2) {
                const bool collect = t2 >= ntiles;
                const int t = tile_of(t2, ntiles);
                const uint32_t inst = gt0 + static_cast<uint32_t>(reuse ? t : t2);
                const int acc = inst & 1;
                const bool wait_acc = !(reuse && collect);   // the threshold pass waited for it
                const bool free_acc = !reuse || collect;     // last read of this accumulator
                float fc[4], vc[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    fc[j] = fv1[j].x;
                    vc[j] = fv1[j].y;
                    fv1[j] = fv2[j];
                }
                if (t2 + 2 < nsteps) load_cols(tile_of(t2 + 2, ntiles), fv2);
                if (!DENSE && t2 == ntiles && quad_live) {
                    // threshold of each entry: kk-th smallest group minimum over both halves
                    if (half == 1) {
#pragma unroll
                        for (int i = 0; i < GK; ++i) mg_s[(quad * 32 + lane) * GKMAX + i] = tv[i];
                    }
                    pair_sync(quad);
                    if (half == 0) {
                        // kk-th smallest of the two ascending lists A (tv) and B (o):
                        // min over i in [0, kk] of max(A_i, B_{kk-i}) with A_i the
                        // i-th smallest (A_0 = -inf; A_i = +inf past the list)
                        const float* o = mg_s + (quad * 32 + lane) * GKMAX;
                        float kth = o[kk - 1];  // i = 0
#pragma unroll
                        for (int i = 1; i <= GK; ++i) {
                            if (i <= kk) {
                                const float bi = i < kk ? o[kk - i - 1] : -INFINITY;
                                kth = fminf(kth, fmaxf(tv[i - 1], bi));
                            }
                        }
                        th_s[quad * 32 + lane] = kth;
                    }
                    pair_sync(quad);
                    thr = th_s[quad * 32 + lane];
                }
                if (live && wait_acc && !mbar_wait(&tfull[acc], (inst >> 1) & 1, abort_flag)) {
                    if (*abort_flag == 0 && status) atomicOr(status, DEV_TIMEOUT_EPILOGUE);
                    *abort_flag = 1;
                    live = false;
                }
                tc_fence_after();
                __syncwarp();  // the previous tile's reads of the staging buffer are done
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    wst[lane + 32 * j] = fc[j];
                    wst[TR / 2 + lane + 32 * j] = vc[j];
                }
                __syncwarp();
                const int64_t col0 = r0 + static_cast<int64_t>(t) * TR;
                const float* fs = wst;
                const float* vs = wst + TR / 2;
                const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                       static_cast<uint32_t>(acc * TR + half * (TR / 2));
                if (quad_live && live) {
#pragma unroll 1
                    for (int c = 0; c < TR / 2 / 32; ++c) {
                        const int64_t gcol = col0 + half * (TR / 2) + c * 32;  // row of column 0 of the group
                        const int64_t left = r1 - gcol;
                        const int nvc = left <= 0 ? 0 : (left >= 32 ? 32 : static_cast<int>(left));  // valid columns
                        uint32_t rr[32];
                        if (nvc > 0) {
                            tmem_ld32_async(tbase + static_cast<uint32_t>(c * 32), rr);
                            tmem_ld_wait(rr);
                        }
                        if (c == TR / 2 / 32 - 1 && free_acc) {
                            // the accumulator is read: the MMA may overwrite it
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive_local(&tempty[acc]);
                        }
                        if (nvc == 0) continue;  // past the list's end (the rest of the tile too)
                        // value = acc * (qf * f) + v, two columns per paired fp32 operation
                        float key[32];
                        const uint64_t qf2 = pack2(qf, qf);
#pragma unroll
                        for (int j4 = 0; j4 < 8; ++j4) {
                            const float4 f4 = *reinterpret_cast<const float4*>(fs + c * 32 + 4 * j4);
                            const float4 v4 = *reinterpret_cast<const float4*>(vs + c * 32 + 4 * j4);
                            const int j = 4 * j4;
                            const uint64_t a01 = pack2(__uint_as_float(rr[j]), __uint_as_float(rr[j + 1]));
                            const uint64_t a23 = pack2(__uint_as_float(rr[j + 2]), __uint_as_float(rr[j + 3]));
                            const uint64_t m01 = mul_f32x2(qf2, pack2(f4.x, f4.y));
                            const uint64_t m23 = mul_f32x2(qf2, pack2(f4.z, f4.w));
                            uint64_t k01, k23;
                            if (METRIC == RDB_METRIC_L2) {
                                k01 = fma_f32x2(a01, m01, pack2(v4.x, v4.y));
                                k23 = fma_f32x2(a23, m23, pack2(v4.z, v4.w));
                            } else {
                                k01 = mul_f32x2(a01, m01);
                                k23 = mul_f32x2(a23, m23);
                            }
                            unpack2(k01, key[j], key[j + 1]);
                            unpack2(k23, key[j + 2], key[j + 3]);
                        }
                        if (nvc < 32) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) key[j] = j < nvc ? key[j] : INFINITY;
                        }
                        if (DENSE) {
                            if (evalid) {
                                float* out = a.dense + (e - a.dense_e0) * a.dense_ld + gcol;
                                const int64_t room = a.dense_ld - gcol;  // padding columns get +inf
                                if (room >= 32 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
                                    for (int j = 0; j < 32; j += 4)
                                        *reinterpret_cast<float4*>(out + j) =
                                            make_float4(key[j], key[j + 1], key[j + 2], key[j + 3]);
                                } else {
#pragma unroll
                                    for (int j = 0; j < 32; ++j)
                                        if (j < room) out[j] = key[j];
                                }
                                float gmin = key[0];
#pragma unroll
                                for (int j = 1; j < 32; ++j) gmin = fminf(gmin, key[j]);
                                a.dense_gmin[(e - a.dense_e0) * (a.dense_ld / 32) + gcol / 32] = gmin;
                            }
                        } else if (!collect) {
                            // threshold pass: minima of groups of gs rows (gs a power of two <= 32)
#pragma unroll
                            for (int w = 1; w < 32; w <<= 1) {
                                if (w < gs) {
#pragma unroll
                                    for (int i = 0; i < 32; i += 2 * w) key[i] = fminf(key[i], key[i + w]);
                                }
                            }
                            insert_sorted(tv, key[0]);
                            if (gs < 32) {
#pragma unroll
                                for (int i = 1; i < 32; ++i) {
                                    if ((i & (gs - 1)) == 0) insert_sorted(tv, key[i]);
                                }
                            }
                        } else {
                            // collecting pass: every row whose value reaches the entry's threshold
                            float gmin = key[0];
#pragma unroll
                            for (int j = 1; j < 32; ++j) gmin = fminf(gmin, key[j]);
                            if (!evalid || !(gmin <= thr)) continue;
                            unsigned m = 0;
#pragma unroll
                            for (int j = 0; j < 32; ++j) m |= key[j] <= thr ? (1u << j) : 0u;
                            if (nvc < 32) m &= (1u << nvc) - 1;  // columns past the list's end
                            while (m) {
                                const int j = __ffs(m) - 1;
                                m &= m - 1;
                                if (cnt < kCap) {
                                    cv[cnt] = pick32(key, j);
                                    cr[cnt] = static_cast<uint32_t>(gcol + j);
                                }
                                ++cnt;
                            }
                        }
                    }
                } else if (free_acc) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_local(&tempty[acc]);
                }
            }
            gt = gt0 + static_cast<uint32_t>(reuse ? ntiles : nsteps);
            if (!DENSE && evalid && live) a.cand_n[pe * 2 + half] = cnt;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_t<false>(tmem_base, TMEM_NCOLS);
    }
}

// Entries whose collection overflowed and were rescanned (rdb_ivf_tc_overflows),
// and probed queries that scored every centroid exactly.
__device__ unsigned long long g_tc_overflows;
__device__ unsigned long long g_probe_rescans;

// One warp per query: the rows collected for its entries (or, for an entry
// whose collection overflowed, every row of that list, with exact fp32
// ranking values) reduced to the best KF >= kk by ranking value, those rows
// scored again with the CUDA-core scan's arithmetic (L2 as sum (q - x)^2, dot
// products accumulated in dimension order, cosine through final_score), and
// the best k of them (ties to the lower stored row) written to out_v / out_i
// [nq, k].
template <int METRIC, int KF, typename T>
__global__ void ivf_tc_finish_kernel(int cos_small, const T* __restrict__ q, int64_t Q, int64_t ldq, int d,
                                     int nprobe, const int64_t* __restrict__ probe, int nlist,
                                     const int64_t* __restrict__ list_off, const int64_t* __restrict__ list_end,
                                     const T* __restrict__ rows, int64_t ldx, const float* __restrict__ xv,
                                     const float* __restrict__ qv, const float* __restrict__ cand_v,
                                     const uint32_t* __restrict__ cand_r, const int* __restrict__ cand_n,
                                     const int64_t* __restrict__ ids, int k, float* __restrict__ out_v,
                                     int64_t* __restrict__ out_i) {
    static_assert(KF <= 32, "one merged row per lane");
    const int lane = threadIdx.x & 31;
    const int64_t qi = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (qi >= Q) return;
    const T* qp = q + qi * ldq;
    const float qvq = METRIC == RDB_METRIC_COSINE ? qv[qi] : 0.f;
    // this lane's best KF (value, row) keys, ascending; branch-free insertion
    // (element j becomes max(min(tk[j], key), tk[j - 1]))
    uint64_t tk[KF];
#pragma unroll
    for (int i = 0; i < KF; ++i) tk[i] = ~0ull;
    auto offer = [&](float v, uint32_t r) {
        const uint64_t key = vr_key(v, r);
        if (key >= tk[KF - 1]) return;
#pragma unroll
        for (int j = KF - 1; j > 0; --j) tk[j] = max(min(tk[j], key), tk[j - 1]);
        tk[0] = min(tk[0], key);
    };
    auto exact_dot = [&](uint32_t r) {
        const T* xp = rows + static_cast<int64_t>(r) * ldx;
        float acc = 0.f;
        for (int t = 0; t < d; ++t) acc = fmaf(tof(qp[t]), tof(xp[t]), acc);
        return acc;
    };
    // 1. rows collected for this query's entries (lane: probe slots lane, lane + 32, ...)
    for (int p = lane; p < nprobe; p += 32) {
        const int64_t pe = qi * nprobe + p;
        const int n0 = cand_n[pe * 2], n1 = cand_n[pe * 2 + 1];
        if (n0 > kCap || n1 > kCap) continue;  // rescanned below
        for (int h = 0; h < 2; ++h) {
            const int n = h ? n1 : n0;
            const float* v = cand_v + (pe * 2 + h) * kCap;
            const uint32_t* r = cand_r + (pe * 2 + h) * kCap;
            for (int i = 0; i < n; ++i) offer(v[i], r[i]);
        }
    }
    // 2. entries whose collection overflowed: the whole list, rows across the warp
    for (int p0 = 0; p0 < nprobe; p0 += 32) {
        bool over = false;
        if (p0 + lane < nprobe) {
            const int64_t pe = qi * nprobe + p0 + lane;
            over = cand_n[pe * 2] > kCap || cand_n[pe * 2 + 1] > kCap;
        }
        unsigned ob = __ballot_sync(0xffffffffu, over);
        if (ob && lane == 0) atomicAdd(&g_tc_overflows, static_cast<unsigned long long>(__popc(ob)));
        while (ob) {
            const int pl = __ffs(ob) - 1;
            ob &= ob - 1;
            int64_t l = probe[qi * nprobe + p0 + pl];
            if (l < 0 || l >= nlist) l = 0;  // as the entry sort files it
            const int64_t r0 = list_off[l], r1 = list_end ? list_end[l] : list_off[l + 1];
            for (int64_t r = r0 + lane; r < r1; r += 32) {
                const float dot = exact_dot(static_cast<uint32_t>(r));
                float key;
                if (METRIC == RDB_METRIC_L2)
                    key = fmaf(-2.f, dot, xv[r]);
                else if (METRIC == RDB_METRIC_COSINE)
                    key = -final_score(RDB_METRIC_COSINE, cos_small, dot, qvq, xv[r]);
                else
                    key = -dot;
                offer(key, static_cast<uint32_t>(r));
            }
        }
    }
    // 3. the warp's best KF: KF rounds of the best list head, whose lane pops it
    uint32_t mine = kNoRow;  // merged row `lane`
    for (int rnd = 0; rnd < KF; ++rnd) {
        uint64_t best = tk[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
        if (best == ~0ull) break;  // every list is exhausted (warp-uniform)
        const uint32_t br = static_cast<uint32_t>(best);
        if (static_cast<uint32_t>(tk[0]) == br) {
            // a row probed twice (a repeated probe slot) leaves every list at once
#pragma unroll
            for (int j = 0; j < KF - 1; ++j) tk[j] = tk[j + 1];
            tk[KF - 1] = ~0ull;
        }
        if (rnd == lane) mine = br;
    }
    // 4. exact score of this lane's merged row
    constexpr bool largest = METRIC != RDB_METRIC_L2;
    float sc = largest ? -INFINITY : INFINITY;
    if (mine != kNoRow) {
        if (METRIC == RDB_METRIC_L2) {
            const T* xp = rows + static_cast<int64_t>(mine) * ldx;
            float acc = 0.f;
            for (int t = 0; t < d; ++t) {
                const float df = tof(qp[t]) - tof(xp[t]);
                acc = fmaf(df, df, acc);
            }
            sc = acc;
        } else {
            const float dot = exact_dot(mine);
            sc = METRIC == RDB_METRIC_COSINE ? final_score(METRIC, cos_small, dot, qvq, xv[mine]) : dot;
        }
    }
    // 5. the best k by exact score: k rounds of a warp arg-best
    uint32_t rw = mine;
    for (int i = 0; i < k; ++i) {
        float bv = rw == kNoRow ? (largest ? -INFINITY : INFINITY) : sc;
        uint32_t br = rw;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t orr = __shfl_xor_sync(0xffffffffu, br, o);
            const bool take =
                orr != kNoRow && (br == kNoRow || (largest ? ov > bv : ov < bv) || (ov == bv && orr < br));
            if (take) {
                bv = ov;
                br = orr;
            }
        }
        if (rw == br) rw = kNoRow;
        if (lane == 0) {
            out_v[qi * k + i] = br == kNoRow ? (largest ? -INFINITY : INFINITY) : bv;
            out_i[qi * k + i] = br == kNoRow ? -1 : (ids ? ids[br] : static_cast<int64_t>(br));
        }
    }
}

constexpr int kProbeBlock = 1024;  // centroid rows per unit of the dense probe scan

// Coarse probe set-up for queries [e0, e1): the centroids in blocks of
// kProbeBlock rows (block b is "list" b), one unit per (block, TQ queries);
// zeroes the hand-out counter.
__global__ void probe_units_kernel(int64_t e0, int64_t e1, int nlist, int64_t* list_off, int2* units, int* nunits,
                                   int* ctr) {
    const int nb = (nlist + kProbeBlock - 1) / kProbeBlock;
    const int64_t nc = (e1 - e0 + TQ - 1) / TQ;
    for (int b = threadIdx.x; b <= nb; b += blockDim.x) list_off[b] = std::min<int64_t>(nlist, int64_t(b) * kProbeBlock);
    for (int64_t i = threadIdx.x; i < nc * nb; i += blockDim.x)
        units[i] = make_int2(static_cast<int>(i % nb), static_cast<int>(e0 + (i / nb) * TQ));
    if (threadIdx.x == 0) {
        *nunits = static_cast<int>(nc * nb);
        *ctr = 0;
    }
}

constexpr int kProbeSlots = 256;  // collected centroids per query before the all-centroid rescan
constexpr int kProbeTop = 128;    // nprobe + margin limit

// Exact squared L2 of query qp and U centroids cp[u] with the flat search's
// arithmetic: per centroid, lane-strided fused multiply-add chains, then a
// butterfly sum (every lane gets the total).  The U chains and butterflies
// are interleaved so that their latencies overlap; each centroid's value is
// the one a single chain would give.
template <int U>
__device__ __forceinline__ void flat_l2_multi(const float* qp, const float* const (&cp)[U], int d, int lane,
                                              float (&out)[U]) {
    float acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = 0.f;
    for (int t = lane; t < d; t += 32) {
        const float qv = qp[t];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const float df = qv - cp[u][t];
            acc[u] = fmaf(df, df, acc[u]);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < U; ++u) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
#pragma unroll
    for (int u = 0; u < U; ++u) out[u] = acc[u];
}

// One warp per query over its row of tensor-core values (|c|^2 - 2 q.c,
// ld a multiple of 32, padding +inf): the kp-th smallest of the row's group
// minima (8 groups per lane) bounds the kp-th smallest value; the centroids
// at or below it (about kp) are scored again with the flat search's exact L2
// and the best nprobe (ties to the lower list) written to probe [nq, nprobe].
// More than kProbeSlots collected (many equal values): every centroid is
// scored exactly instead, in chunks.
__global__ void __launch_bounds__(256) probe_select_kernel(const float* __restrict__ dense,
                                                           const float* __restrict__ gmin, int64_t ld, int64_t e0,
                                                           int64_t n, int nlist, int kp, const float* __restrict__ q,
                                                           int64_t ldq, int d, const float* __restrict__ cent,
                                                           int64_t ldc, int nprobe, int64_t* __restrict__ probe,
                                                           unsigned long long* nover) {
    __shared__ int s_idx[8][kProbeSlots];
    __shared__ float s_val[8][kProbeSlots];
    __shared__ int s_top_i[8][kProbeTop];
    __shared__ float s_top_v[8][kProbeTop];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + w;
    if (r >= n) return;
    const float* row = dense + r * ld;
    const int nper = static_cast<int>(ld / 32);
    // With at least 2 kp groups of 32 columns, the scan's group minima bound the
    // kp-th value and only groups at or below the bound are read again;
    // otherwise lane-local runs of the lane's columns form the groups.
    const bool by_groups = nper >= 2 * kp;
    const int gsz = by_groups ? (nper + 255) / 256 : (nper >= 8 ? (nper + 7) / 8 : 1);
    const float* grow = gmin + r * nper;
    float gm[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        gm[g] = INFINITY;
        if (by_groups) {
            // groups of gsz scan groups: lane L, slot g covers scan groups (g * 32 + L) * gsz ..
            const int i0 = (g * 32 + lane) * gsz, i1 = min(nper, i0 + gsz);
            for (int i = i0; i < i1; ++i) gm[g] = fminf(gm[g], grow[i]);
        } else {
            const int i1 = min(nper, (g + 1) * gsz);
            for (int i = g * gsz; i < i1; ++i) gm[g] = fminf(gm[g], row[i * 32 + lane]);
        }
    }
    // kp-th smallest group minimum, by bisection on the ordered keys
    uint32_t lo = 0, hi = 0xffffffffu;
    {
        int fin = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) fin += gm[g] < INFINITY ? 1 : 0;
        if (__reduce_add_sync(0xffffffffu, fin) < kp) lo = fkey(INFINITY);
    }
    if (lo == 0) {
        while (lo < hi) {
            const uint32_t mid = lo + (hi - lo) / 2;
            int c = 0;
#pragma unroll
            for (int g = 0; g < 8; ++g) c += fkey(gm[g]) <= mid ? 1 : 0;
            if (static_cast<int>(__reduce_add_sync(0xffffffffu, c)) >= kp)
                hi = mid;
            else
                lo = mid + 1;
        }
    }
    const uint32_t tk = lo;
    // collect the columns at or below it (by_groups: from the groups whose minimum is)
    int cnt = 0;
    for (int i0 = 0; i0 < nper; i0 += by_groups ? 32 : 1) {
        unsigned gb = 1u;  // groups of 32 columns to read, one bit per lane's group
        if (by_groups) {
            const int gi = i0 + lane;
            gb = __ballot_sync(0xffffffffu, gi < nper && fkey(grow[gi]) <= tk);
        }
        while (gb) {
            // up to four groups at a time: their loads in flight together
            int gi4[4];
            float v4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                gi4[u] = -1;
                if (gb) {
                    gi4[u] = i0 + __ffs(gb) - 1;
                    gb &= gb - 1;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int col = gi4[u] * 32 + lane;
                v4[u] = (gi4[u] >= 0 && col < nlist) ? row[col] : INFINITY;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (gi4[u] < 0) break;  // warp-uniform
                const int col = gi4[u] * 32 + lane;
                const bool take = col < nlist && fkey(v4[u]) <= tk;
                const unsigned b = __ballot_sync(0xffffffffu, take);
                const int pos = cnt + __popc(b & ((1u << lane) - 1));
                if (take && pos < kProbeSlots) s_idx[w][pos] = col;
                cnt += __popc(b);
            }
        }
    }
    const bool all = cnt > kProbeSlots;
    if (all && lane == 0) atomicAdd(nover, 1ull);
    const int total = all ? nlist : cnt;
    const float* qp = q + (e0 + r) * ldq;
    int ntop = 0;
    for (int c0 = 0; c0 < total; c0 += kProbeSlots) {
        const int nc = min(kProbeSlots, total - c0);
        __syncwarp();
        for (int c = 0; c < nc; c += 4) {
            // four centroids at a time (the last ones repeat centroid nc - 1, unused)
            int l4[4];
            const float* cp4[4];
            float dist4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int cc = min(c + u, nc - 1);
                l4[u] = all ? c0 + cc : s_idx[w][cc];
                cp4[u] = cent + static_cast<int64_t>(l4[u]) * ldc;
            }
            flat_l2_multi<4>(qp, cp4, d, lane, dist4);
            if (lane == 0) {
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (c + u < nc) {
                        s_val[w][c + u] = dist4[u];
                        if (all) s_idx[w][c + u] = l4[u];
                    }
            }
        }
        __syncwarp();
        if (!all) {
            // every candidate in this one chunk: each goes straight to the
            // position of its rank in (distance, list) order -- the order of
            // the selection below (a NaN distance counts as +inf)
            for (int c = lane; c < nc; c += 32) {
                const float v0 = s_val[w][c];
                const float v = v0 != v0 ? INFINITY : v0;
                const int id = s_idx[w][c];
                int rank = 0;
                for (int j = 0; j < nc; ++j) {
                    const float u0 = s_val[w][j];
                    const float u = u0 != u0 ? INFINITY : u0;
                    rank += (u < v || (u == v && s_idx[w][j] < id)) ? 1 : 0;
                }
                if (rank < nprobe) probe[(e0 + r) * nprobe + rank] = id;
            }
            for (int i = nc + lane; i < nprobe; i += 32) probe[(e0 + r) * nprobe + i] = -1;
            return;
        }
        // best nprobe of this chunk and the running list
        float cv[8];
        int ci[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = lane + 32 * j;
            cv[j] = c < nc ? s_val[w][c] : INFINITY;
            ci[j] = c < nc ? s_idx[w][c] : -1;
        }
        float tv[kProbeTop / 32];
        int ti[kProbeTop / 32];
#pragma unroll
        for (int j = 0; j < kProbeTop / 32; ++j) {
            const int c = lane + 32 * j;
            tv[j] = c < ntop ? s_top_v[w][c] : INFINITY;
            ti[j] = c < ntop ? s_top_i[w][c] : -1;
        }
        __syncwarp();
        const int want = min(nprobe, ntop + nc);
        for (int i = 0; i < want; ++i) {
            float bv = INFINITY;
            int bi = -1;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (ci[j] >= 0 && (bi < 0 || cv[j] < bv || (cv[j] == bv && ci[j] < bi))) {
                    bv = cv[j];
                    bi = ci[j];
                }
#pragma unroll
            for (int j = 0; j < kProbeTop / 32; ++j)
                if (ti[j] >= 0 && (bi < 0 || tv[j] < bv || (tv[j] == bv && ti[j] < bi))) {
                    bv = tv[j];
                    bi = ti[j];
                }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi >= 0 && (bi < 0 || ov < bv || (ov == bv && oi < bi))) {
                    bv = ov;
                    bi = oi;
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (ci[j] == bi) ci[j] = -1;
#pragma unroll
            for (int j = 0; j < kProbeTop / 32; ++j)
                if (ti[j] == bi) ti[j] = -1;
            if (lane == 0) {
                s_top_v[w][i] = bv;
                s_top_i[w][i] = bi;
            }
        }
        ntop = want;
    }
    __syncwarp();
    for (int i = lane; i < nprobe; i += 32) probe[(e0 + r) * nprobe + i] = i < ntop ? s_top_i[w][i] : -1;
}

inline size_t au(size_t v) { return (v + 255) / 256 * 256; }

// coarse probe: queries per chunk, so that the chunk's [rows, nlist] value
// matrix stays within 2^26 floats
int64_t probe_chunk(int64_t nq, int nlist) {
    const int64_t ld = (nlist + 31) / 32 * 32;
    const int64_t c = std::max<int64_t>(TQ, ((int64_t(1) << 26) / ld) / TQ * TQ);
    return std::min<int64_t>(nq, c);
}

struct ProbeWs {
    size_t off_qh, off_ql, off_qs, off_dense, off_gmin, off_loff, off_units, off_fv, off_n, bytes;
    int64_t dp, chunk, ld;
    int kp;
};

ProbeWs probe_ws(int64_t nq, int nlist, int d, int nprobe) {
    ProbeWs w;
    w.dp = (d + TK - 1) / TK * TK;
    w.chunk = std::max<int64_t>(1, probe_chunk(nq, nlist));
    w.ld = (nlist + 31) / 32 * 32;
    w.kp = std::min(nlist, nprobe + kL2Margin);
    const int64_t nqp = std::max<int64_t>(nq, 1);
    size_t off = 0;
    w.off_qh = off;
    off = au(off + sizeof(__half) * nqp * w.dp);
    w.off_ql = off;
    off = au(off + sizeof(__half) * nqp * w.dp);
    w.off_qs = off;
    off = au(off + sizeof(float) * nqp);
    w.off_dense = off;
    off = au(off + sizeof(float) * w.chunk * w.ld);
    w.off_gmin = off;
    off = au(off + sizeof(float) * w.chunk * (w.ld / 32));
    const int64_t nb = (nlist + kProbeBlock - 1) / kProbeBlock;
    w.off_loff = off;
    off = au(off + sizeof(int64_t) * (nb + 1));
    w.off_units = off;
    off = au(off + sizeof(int2) * ((w.chunk + TQ - 1) / TQ) * nb);
    w.off_fv = off;
    off = au(off + sizeof(float2) * nlist);
    w.off_n = off;
    off = au(off + 2 * sizeof(int));
    w.bytes = off;
    return w;
}

struct TcWs {
    IvfWs inv;
    size_t off_qh, off_ql, off_qs, off_cv, off_cr, off_cn, off_units, off_fv, off_n, bytes;
    int64_t E, dp, max_units;
    int kk;
};

// ranked rows per entry: k + 8 (the rescoring margin)
int tc_kk(int k) { return k + kL2Margin; }

TcWs tc_ws(int64_t nq, int nprobe, int nlist, int d, int k, int64_t nrows) {
    TcWs w;
    w.inv = ivf_ws(nq, nprobe, nlist);
    w.E = nq * nprobe;
    w.dp = (d + TK - 1) / TK * TK;
    w.kk = tc_kk(k);
    w.max_units = (w.E + TQ - 1) / TQ + nlist;
    const int64_t Ep = std::max<int64_t>(w.E, 1);
    size_t off = au(w.inv.bytes);
    w.off_qh = off;
    off = au(off + sizeof(__half) * Ep * w.dp);
    w.off_ql = off;
    off = au(off + sizeof(__half) * Ep * w.dp);
    w.off_qs = off;
    off = au(off + sizeof(float) * Ep);
    w.off_cv = off;
    off = au(off + sizeof(float) * Ep * 2 * kCap);
    w.off_cr = off;
    off = au(off + sizeof(uint32_t) * Ep * 2 * kCap);
    w.off_cn = off;
    off = au(off + sizeof(int) * Ep * 2);
    w.off_units = off;
    off = au(off + sizeof(int2) * w.max_units);
    w.off_fv = off;
    off = au(off + sizeof(float2) * std::max<int64_t>(nrows, 1));
    w.off_n = off;  // unit count, hand-out counter
    off = au(off + 2 * sizeof(int));
    w.bytes = off;
    return w;
}

int map_f16(CUtensorMap* m, const void* base, int64_t rows, int64_t dp, int box_rows, int dtype = RDB_F16,
            int64_t ld = 0) {
    return make_map(m, dtype, base, rows, static_cast<int>(dp), (ld ? ld : dp) * 2, TK, box_rows);
}

template <int METRIC, int GK, bool DENSE = false>
int launch_scan(const CUtensorMap& mqh, const CUtensorMap& mql, const CUtensorMap& mxh, const CUtensorMap& mxl,
                const IvfTcArgs& a, int grid, cudaStream_t s, uint32_t idesc = tc_idesc(false, TQ, TR)) {
    static bool attr[64] = {false};
    int dev = 0;
    RDB_CUDA_TRY(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        RDB_CUDA_TRY(cudaFuncSetAttribute(ivf_tc_scan_kernel<METRIC, GK, DENSE>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        attr[dev] = true;
    }
    ivf_tc_scan_kernel<METRIC, GK, DENSE><<<grid, NTHR, SMEM_BYTES, s>>>(mqh, mql, mxh, mxl, a, idesc,
                                                                         device_status_word());
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

struct FinishArgs {
    int dtype;  // of q and rows
    const void* q;
    int64_t nq, ldq;
    int d;
    const int64_t* probe;
    int nlist;
    const int64_t* list_off;
    const int64_t* list_end;
    const void* rows;
    int64_t ldx;
    const int64_t* ids;
    int k;
    float* out_v;
    int64_t* out_i;
};

template <int METRIC, int KF, typename T>
int launch_finish_t(const IvfTcArgs& a, const FinishArgs& f, cudaStream_t s) {
    ivf_tc_finish_kernel<METRIC, KF, T><<<(unsigned)((f.nq + 7) / 8), 256, 0, s>>>(
        a.cos_small, static_cast<const T*>(f.q), f.nq, f.ldq, f.d, a.nprobe, f.probe, f.nlist, f.list_off,
        f.list_end, static_cast<const T*>(f.rows), f.ldx, a.xv, a.qv, a.cand_v, a.cand_r, a.cand_n, f.ids, f.k,
        f.out_v, f.out_i);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

template <int METRIC, int KF>
int launch_finish(const IvfTcArgs& a, const FinishArgs& f, cudaStream_t s) {
    if (f.dtype == RDB_F16) return launch_finish_t<METRIC, KF, __half>(a, f, s);
    if (f.dtype == RDB_BF16) return launch_finish_t<METRIC, KF, __nv_bfloat16>(a, f, s);
    return launch_finish_t<METRIC, KF, float>(a, f, s);
}

// scan with group-minimum lists of GK >= kk, then the per-query finish
template <int METRIC, int GK>
int run_metric(const CUtensorMap& mqh, const CUtensorMap& mql, const CUtensorMap& mxh, const CUtensorMap& mxl,
               const IvfTcArgs& a, int grid, uint32_t idesc, const FinishArgs& f, cudaStream_t s) {
    cudaEvent_t stop_ev;
    RDB_TRY(timing_begin(TIMING_IVF_SCAN, s, &stop_ev));
    RDB_TRY((launch_scan<METRIC, GK>(mqh, mql, mxh, mxl, a, grid, s, idesc)));
    if (stop_ev) RDB_CUDA_TRY(cudaEventRecord(stop_ev, s));
    return launch_finish<METRIC, GK>(a, f, s);
}

template <int METRIC>
int run_kk(const CUtensorMap& mqh, const CUtensorMap& mql, const CUtensorMap& mxh, const CUtensorMap& mxl,
           const IvfTcArgs& a, int grid, uint32_t idesc, const FinishArgs& f, cudaStream_t s) {
    if (a.kk <= 16) return run_metric<METRIC, 16>(mqh, mql, mxh, mxl, a, grid, idesc, f, s);
    if (a.kk <= 24) return run_metric<METRIC, 24>(mqh, mql, mxh, mxl, a, grid, idesc, f, s);
    return run_metric<METRIC, 32>(mqh, mql, mxh, mxl, a, grid, idesc, f, s);
}

// One warp per entry: the entry's query, as stored (fp16 / bf16), gathered
// into entry order with zero columns d .. dp - 1, scale 1.
template <typename T>
__global__ void gather_half_kernel(const T* __restrict__ q, int64_t ldq, int d, const int64_t* __restrict__ eperm,
                                   int nprobe, int64_t E, T* __restrict__ out, int64_t dp, float* __restrict__ scale) {
    const int lane = threadIdx.x & 31;
    const int64_t e = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (e >= E) return;
    const T* p = q + (eperm[e] / nprobe) * ldq;
    for (int t = lane; t < (int)dp; t += 32) out[e * dp + t] = t < d ? p[t] : T(0.f);
    if (lane == 0) scale[e] = 1.f;
}

// The tensor-core IVF-Flat search over fp32 rows (split planes) or fp16 /
// bf16 rows (as stored, one product per element).
int search_tc_impl(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d, const int64_t* probe,
                   int nprobe, const void* rows, int64_t ldx, const float* xv, const void* rows_hi, const void* rows_lo,
                   const float* row_scale, int64_t ldp, int64_t nrows, const int64_t* list_off,
                   const int64_t* list_end, int nlist, const int64_t* ids, int k, float* out_v, int64_t* out_i,
                   void* ws, size_t ws_bytes, cudaStream_t s) {
    const bool split = dtype == RDB_F32;
    const TcWs w = tc_ws(nq, nprobe, nlist, d, k, nrows);
    if (split) RDB_CHECK_ARG(ldp == w.dp, "row planes must have a stride of %lld (d padded to 64)", (long long)w.dp);
    RDB_CHECK_ARG(w.E < (1LL << 31) - TQ && nrows < (1LL << 31) - TR, "too many entries or rows for one search");
    if (ws_bytes < w.bytes) return set_error(RDB_ERR_WORKSPACE, "workspace too small: %zu < %zu", ws_bytes, w.bytes);
    char* base = static_cast<char*>(ws);
    RDB_TRY(invert_probes(probe, nq, nprobe, nlist, w.inv, base, s));
    const int64_t* eperm = reinterpret_cast<const int64_t*>(base + w.inv.off_perm);
    const int64_t* eseg = reinterpret_cast<const int64_t*>(base + w.inv.off_seg);
    float* qv = reinterpret_cast<float*>(base + w.inv.off_qv);
    if (metric == RDB_METRIC_COSINE) {
        RDB_TRY(row_sqnorms_ld(dtype, q, nq, d, ldq, qv, s));
        RDB_TRY(rdb_vec_values(metric, d, qv, nq, qv, s));
    }
    __half* qh = reinterpret_cast<__half*>(base + w.off_qh);
    __half* ql = reinterpret_cast<__half*>(base + w.off_ql);
    float* qs = reinterpret_cast<float*>(base + w.off_qs);
    // the probing queries, entry by entry in list order
    const unsigned gblocks = (unsigned)((w.E + 7) / 8);
    if (split) {
        split_f16_kernel<<<gblocks, 256, 0, s>>>(static_cast<const float*>(q), w.E, ldq, d, qh, ql, w.dp, qs, eperm,
                                                 nprobe, nullptr);
    } else if (dtype == RDB_F16) {
        gather_half_kernel<__half><<<gblocks, 256, 0, s>>>(static_cast<const __half*>(q), ldq, d, eperm, nprobe, w.E,
                                                           qh, w.dp, qs);
    } else {
        gather_half_kernel<__nv_bfloat16><<<gblocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(q), ldq, d,
                                                                  eperm, nprobe, w.E,
                                                                  reinterpret_cast<__nv_bfloat16*>(qh), w.dp, qs);
    }
    RDB_LAUNCH_CHECK();
    int2* units = reinterpret_cast<int2*>(base + w.off_units);
    int* counters = reinterpret_cast<int*>(base + w.off_n);
    ivf_tc_units_kernel<<<1, 1024, 0, s>>>(eseg, nlist, units, counters, counters + 1);
    RDB_LAUNCH_CHECK();
    float2* colfv = reinterpret_cast<float2*>(base + w.off_fv);
    if (nrows > 0) {
        col_factors_kernel<<<(unsigned)((nrows + 255) / 256), 256, 0, s>>>(metric, row_scale, xv, nrows, colfv);
        RDB_LAUNCH_CHECK();
    }
    const int mdt = split ? RDB_F16 : dtype;  // element type the MMA reads
    CUtensorMap mqh, mql, mxh, mxl;
    RDB_TRY(map_f16(&mqh, qh, w.E, w.dp, TQ, mdt));
    RDB_TRY(map_f16(&mql, ql, w.E, w.dp, TQ, mdt));
    if (split) {
        RDB_TRY(map_f16(&mxh, rows_hi, std::max<int64_t>(nrows, 1), w.dp, TR));
        RDB_TRY(map_f16(&mxl, rows_lo, std::max<int64_t>(nrows, 1), w.dp, TR));
    } else {
        // the stored rows themselves: ldx columns (zero past d), K blocks past them read as zero
        RDB_TRY(map_f16(&mxh, rows, std::max<int64_t>(nrows, 1), ldx, TR, mdt, ldx));
        mxl = mxh;
    }
    IvfTcArgs a = {};
    a.metric = metric;
    a.cos_small = d <= 128 ? 1 : 0;
    a.nkb = static_cast<int>(w.dp / TK);
    a.planes = split ? 2 : 1;
    a.kk = w.kk;
    a.units = units;
    a.nunits = counters;
    a.unit_ctr = counters + 1;
    a.eseg = eseg;
    a.eperm = eperm;
    a.nprobe = nprobe;
    a.list_off = list_off;
    a.list_end = list_end;
    a.xv = xv;
    a.row_scale = row_scale;
    a.colfv = colfv;
    a.qv = qv;
    a.ent_scale = qs;
    a.cand_v = reinterpret_cast<float*>(base + w.off_cv);
    a.cand_r = reinterpret_cast<uint32_t*>(base + w.off_cr);
    a.cand_n = reinterpret_cast<int*>(base + w.off_cn);
    FinishArgs f = {dtype, q, nq, ldq, d, probe, nlist, list_off, list_end, rows, ldx, ids, k, out_v, out_i};
    const int grid = static_cast<int>(std::min<int64_t>(w.max_units, num_sms()));
    const uint32_t idesc = tc_idesc(mdt == RDB_BF16, TQ, TR);
    switch (metric) {
        case RDB_METRIC_L2: return run_kk<RDB_METRIC_L2>(mqh, mql, mxh, mxl, a, grid, idesc, f, s);
        case RDB_METRIC_COSINE: return run_kk<RDB_METRIC_COSINE>(mqh, mql, mxh, mxl, a, grid, idesc, f, s);
        default: return run_kk<RDB_METRIC_DOT>(mqh, mql, mxh, mxl, a, grid, idesc, f, s);
    }
}

}  // namespace
}  // namespace rdb

using namespace rdb;

extern "C" {

int rdb_f16_split(const float* x, int64_t n, int64_t ldx, int d, void* hi, void* lo, int64_t ldp, float* scale,
                  unsigned* flag, void* stream) {
    RDB_CHECK_ARG(n >= 0 && d >= 1 && ldx >= d && ldp >= d && ldp % 8 == 0, "bad shape");
    if (n == 0) return RDB_OK;
    RDB_CHECK_ARG(x && hi && lo && scale, "NULL pointer");
    split_f16_kernel<<<(unsigned)((n + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, n, ldx, d, static_cast<__half*>(hi), static_cast<__half*>(lo), ldp, scale, nullptr, 1, flag);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

int rdb_ivf_tc_overflows(unsigned long long* out_host, int reset) {
    RDB_CHECK_ARG(out_host, "NULL pointer");
    RDB_CUDA_TRY(cudaDeviceSynchronize());
    RDB_CUDA_TRY(cudaMemcpyFromSymbol(out_host, g_tc_overflows, sizeof(unsigned long long)));
    RDB_CUDA_TRY(cudaMemcpyFromSymbol(out_host + 1, g_probe_rescans, sizeof(unsigned long long)));
    if (reset) {
        const unsigned long long zero = 0;
        RDB_CUDA_TRY(cudaMemcpyToSymbol(g_tc_overflows, &zero, sizeof(zero)));
        RDB_CUDA_TRY(cudaMemcpyToSymbol(g_probe_rescans, &zero, sizeof(zero)));
    }
    return RDB_OK;
}

int rdb_ivf_flat_search_tc_supported(int d, int k) {
    return d >= 1 && d <= kMaxDp && k >= 1 && tc_kk(k) <= kMaxKK ? 1 : 0;
}

size_t rdb_ivf_flat_search_tc_workspace(int64_t nq, int nprobe, int nlist, int d, int k, int64_t nrows) {
    if (nq <= 0 || nprobe <= 0 || nlist <= 0 || d <= 0 || k <= 0) return 256;
    return tc_ws(nq, nprobe, nlist, d, k, nrows).bytes;
}

int rdb_ivf_flat_search_tc(int metric, const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe,
                           int nprobe, const float* rows, int64_t ldx, const float* xv, const void* rows_hi,
                           const void* rows_lo, const float* row_scale, int64_t ldp, int64_t nrows,
                           const int64_t* list_off, const int64_t* list_end, int nlist, const int64_t* ids, int k,
                           float* out_v, int64_t* out_i, void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(metric >= 0 && metric <= 2, "unknown metric %d", metric);
    RDB_CHECK_ARG(nq >= 0 && nprobe >= 1 && nlist >= 1 && nlist <= kMaxLabels, "bad shape");
    RDB_CHECK_ARG(rdb_ivf_flat_search_tc_supported(d, k), "tensor-core IVF search: d must be in [1, %d], k in [1, %d]",
                  kMaxDp, kMaxKK - kL2Margin);
    if (nq == 0) return RDB_OK;
    RDB_CHECK_ARG(q && probe && rows && rows_hi && rows_lo && row_scale && list_off && out_v && out_i && ws,
                  "NULL pointer");
    RDB_CHECK_ARG(metric == RDB_METRIC_DOT || xv, "cosine / L2 need per-row values");
    RDB_CHECK_ARG((reinterpret_cast<uintptr_t>(rows_hi) & 15) == 0 && (reinterpret_cast<uintptr_t>(rows_lo) & 15) == 0,
                  "row planes must be 16-byte aligned");
    return search_tc_impl(metric, RDB_F32, q, nq, ldq, d, probe, nprobe, rows, ldx, xv, rows_hi, rows_lo, row_scale,
                          ldp, nrows, list_off, list_end, nlist, ids, k, out_v, out_i, ws, ws_bytes,
                          static_cast<cudaStream_t>(stream));
}

int rdb_ivf_flat_search_tc_half(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d,
                                const int64_t* probe, int nprobe, const void* rows, int64_t ldx, const float* xv,
                                int64_t nrows, const int64_t* list_off, const int64_t* list_end, int nlist,
                                const int64_t* ids, int k, float* out_v, int64_t* out_i, void* ws, size_t ws_bytes,
                                void* stream) {
    RDB_CHECK_ARG(metric >= 0 && metric <= 2, "unknown metric %d", metric);
    RDB_CHECK_ARG(dtype == RDB_F16 || dtype == RDB_BF16, "rows must be fp16 or bf16");
    RDB_CHECK_ARG(nq >= 0 && nprobe >= 1 && nlist >= 1 && nlist <= kMaxLabels, "bad shape");
    RDB_CHECK_ARG(rdb_ivf_flat_search_tc_supported(d, k), "tensor-core IVF search: d must be in [1, %d], k in [1, %d]",
                  kMaxDp, kMaxKK - kL2Margin);
    RDB_CHECK_ARG(ldx >= d && ldx % 8 == 0, "row stride must be a multiple of 8 elements (16 bytes)");
    if (nq == 0) return RDB_OK;
    RDB_CHECK_ARG(q && probe && rows && list_off && out_v && out_i && ws, "NULL pointer");
    RDB_CHECK_ARG(metric == RDB_METRIC_DOT || xv, "cosine / L2 need per-row values");
    RDB_CHECK_ARG((reinterpret_cast<uintptr_t>(rows) & 15) == 0, "rows must be 16-byte aligned");
    return search_tc_impl(metric, dtype, q, nq, ldq, d, probe, nprobe, rows, ldx, xv, nullptr, nullptr, nullptr, 0,
                          nrows, list_off, list_end, nlist, ids, k, out_v, out_i, ws, ws_bytes,
                          static_cast<cudaStream_t>(stream));
}

int rdb_ivf_probe_tc_supported(int d, int nlist, int nprobe) {
    return d >= 1 && d <= kMaxDp && nlist >= 1 && nprobe >= 1 && nprobe <= nlist &&
                   std::min(nlist, nprobe + kL2Margin) <= kProbeTop
               ? 1
               : 0;
}

size_t rdb_ivf_probe_tc_workspace(int64_t nq, int nlist, int d, int nprobe) {
    if (nq <= 0 || nlist <= 0 || d <= 0 || nprobe <= 0) return 256;
    return probe_ws(nq, nlist, d, nprobe).bytes;
}

int rdb_ivf_probe_tc(const float* q, int64_t nq, int64_t ldq, int d, const float* cent, int64_t ldc,
                     const float* cent_sq, const void* cent_hi, const void* cent_lo, const float* cent_scale,
                     int64_t ldp, int nlist, int nprobe, int64_t* probe, void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(nq >= 0 && ldq >= d && ldc >= d, "bad shape");
    RDB_CHECK_ARG(rdb_ivf_probe_tc_supported(d, nlist, nprobe),
                  "tensor-core probe: d in [1, %d], nprobe in [1, nlist], min(nlist, nprobe + %d) <= %d", kMaxDp,
                  kL2Margin, kProbeTop);
    if (nq == 0) return RDB_OK;
    RDB_CHECK_ARG(q && cent && cent_sq && cent_hi && cent_lo && cent_scale && probe && ws, "NULL pointer");
    const ProbeWs w = probe_ws(nq, nlist, d, nprobe);
    RDB_CHECK_ARG(ldp == w.dp, "centroid planes must have a stride of %lld (d padded to 64)", (long long)w.dp);
    RDB_CHECK_ARG(nq < (1LL << 31) - TQ, "too many queries for one probe");
    RDB_CHECK_ARG((reinterpret_cast<uintptr_t>(cent_hi) & 15) == 0 && (reinterpret_cast<uintptr_t>(cent_lo) & 15) == 0,
                  "centroid planes must be 16-byte aligned");
    if (ws_bytes < w.bytes) return set_error(RDB_ERR_WORKSPACE, "workspace too small: %zu < %zu", ws_bytes, w.bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* base = static_cast<char*>(ws);
    __half* qh = reinterpret_cast<__half*>(base + w.off_qh);
    __half* ql = reinterpret_cast<__half*>(base + w.off_ql);
    float* qs = reinterpret_cast<float*>(base + w.off_qs);
    split_f16_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(q, nq, ldq, d, qh, ql, w.dp, qs, nullptr, 1, nullptr);
    RDB_LAUNCH_CHECK();
    CUtensorMap mqh, mql, mxh, mxl;
    RDB_TRY(map_f16(&mqh, qh, nq, w.dp, TQ));
    RDB_TRY(map_f16(&mql, ql, nq, w.dp, TQ));
    RDB_TRY(map_f16(&mxh, cent_hi, nlist, w.dp, TR));
    RDB_TRY(map_f16(&mxl, cent_lo, nlist, w.dp, TR));
    int64_t* loff = reinterpret_cast<int64_t*>(base + w.off_loff);
    int2* units = reinterpret_cast<int2*>(base + w.off_units);
    int* counters = reinterpret_cast<int*>(base + w.off_n);
    float* dense = reinterpret_cast<float*>(base + w.off_dense);
    float* gmins = reinterpret_cast<float*>(base + w.off_gmin);
    IvfTcArgs a = {};
    a.metric = RDB_METRIC_L2;
    a.cos_small = 1;
    a.nkb = static_cast<int>(w.dp / TK);
    a.planes = 2;
    a.kk = 1;
    a.units = units;
    a.nunits = counters;
    a.unit_ctr = counters + 1;
    a.nprobe = 1;
    a.list_off = loff;
    a.list_end = nullptr;
    a.xv = cent_sq;
    a.row_scale = cent_scale;
    float2* cfv = reinterpret_cast<float2*>(base + w.off_fv);
    col_factors_kernel<<<(unsigned)((nlist + 255) / 256), 256, 0, s>>>(RDB_METRIC_L2, cent_scale, cent_sq, nlist, cfv);
    RDB_LAUNCH_CHECK();
    a.colfv = cfv;
    a.ent_scale = qs;
    a.dense = dense;
    a.dense_gmin = gmins;
    a.dense_ld = w.ld;
    for (int64_t e0 = 0; e0 < nq; e0 += w.chunk) {
        const int64_t e1 = std::min(nq, e0 + w.chunk);
        probe_units_kernel<<<1, 256, 0, s>>>(e0, e1, nlist, loff, units, counters, counters + 1);
        RDB_LAUNCH_CHECK();
        a.dense_e0 = e0;
        a.dense_e1 = e1;
        const int64_t nunits = (e1 - e0 + TQ - 1) / TQ * ((nlist + kProbeBlock - 1) / kProbeBlock);
        const int grid = static_cast<int>(std::min<int64_t>(nunits, num_sms()));
        RDB_TRY((launch_scan<RDB_METRIC_L2, 16, true>(mqh, mql, mxh, mxl, a, grid, s)));
        unsigned long long* nover = nullptr;
        RDB_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void**>(&nover), g_probe_rescans));
        probe_select_kernel<<<(unsigned)((e1 - e0 + 7) / 8), 256, 0, s>>>(dense, gmins, w.ld, e0, e1 - e0, nlist,
                                                                          w.kp, q, ldq, d, cent, ldc, nprobe, probe,
                                                                          nover);
        RDB_LAUNCH_CHECK();
    }
    return RDB_OK;
}

}  // extern "C"
