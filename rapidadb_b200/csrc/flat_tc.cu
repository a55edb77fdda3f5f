// tcgen05 fused scan for fp16 / bf16 rows (sm_100a).
//
// One CTA = 128 queries x a contiguous split of rows, walked in tiles of 256
// rows (UMMA N = 256); with more than 128 queries two CTAs pair up (UMMA
// M = 256, see TcCfg).  Warp roles:
//   warp 0      TMA producer: per K block of 64 (one 128-byte swizzle atom)
//               loads the query tile and the row tile into a shared-memory
//               ring (SWIZZLE_128B, K-major).
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32 accumulators);
//               one lane (of the leader CTA) issues tcgen05.mma kind::f16
//               (K = 16 per instruction) and commits stage releases /
//               accumulator-ready barriers.
//   warps 2..9  epilogue, two warps per TMEM lane quadrant: each thread owns
//               one query row (one TMEM lane) and half of the tile's columns,
//               reads 32 accumulator columns per tcgen05.ld and keeps only the
//               rows whose dot product passes the query's threshold
//               (dot >= A * xv[row] + B, see filter_coef), appending
//               (score, row) to the query's candidate list.  Nothing else of
//               the [queries, rows] score tile leaves the SM.
// While the epilogue drains one accumulator the MMA fills the other.
//
// Every mbarrier wait is bounded (kWaitLimitNs): a role that gives up sets the
// CTA abort flag and a bit in the device status word, waits (bounded) for its
// own in-flight TMA loads / MMAs, and the CTA frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "scan.cuh"
#include "tc_common.cuh"

namespace rdb {
namespace {

constexpr int BM = kTcQueries;  // 128
constexpr int BN = kTcRows;     // 256
constexpr int BK = 64;
constexpr int UK = 16;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = 512;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quadrant
constexpr int EPI_THREADS = EPI_WARPS * 32;
constexpr int NUM_THREADS = 64 + EPI_THREADS;
constexpr int BAR_BYTES = 256;
constexpr int XV_BYTES = 2 * BN * 4;
// per-query candidate counters / arg-best hand-over, then per 32-row block the
// largest 1 / xv of the row values' two buffers (cosine group maxima)
constexpr int EPI_SHARED_BYTES = 2 * BM * 4 + 2 * (BN / 32) * 4;
static_assert(EPI_THREADS == BN, "one epilogue thread per row of a tile (row values)");

static_assert(NUM_ACC * BN <= TMEM_COLS, "accumulators exceed TMEM allocation");

// Named barrier among the epilogue warps (id 1; id 0 is __syncthreads).
__device__ __forceinline__ void epi_bar_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(EPI_THREADS) : "memory");
}

// Same barrier with an AND-reduction: every epilogue thread learns whether all
// of them succeeded, so they leave the tile loop together.
__device__ __forceinline__ bool epi_bar_and(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pin, pout;\n\t"
        "setp.ne.u32 pin, %1, 0;\n\t"
        "bar.red.and.pred pout, 1, %2, pin;\n\t"
        "selp.u32 %0, 1, 0, pout;\n\t}"
        : "=r"(r)
        : "r"(ok ? 1u : 0u), "n"(EPI_THREADS)
        : "memory");
    return r != 0;
}


// ------------------------------------------------------------------ kernel --
//
// Two launch shapes share one body:
//   single CTA  (PAIR = false): UMMA M = 128, the CTA loads its 128 queries and
//               all 256 rows of each tile; 4 stages of 48 KB.
//   CTA pair    (PAIR = true, cluster of 2, tcgen05 cta_group::2): UMMA
//               M = 256 across the pair.  CTA r loads its own 128 queries and
//               rows [128 r, 128 r + 128) of each 256-row tile, so a pair reads
//               every row tile once for 256 queries (a third less L2 traffic
//               per SM than the single-CTA shape); 6 stages of 32 KB.  Only
//               the leader (rank 0) issues MMAs; both CTAs' TMA loads complete
//               on the leader's stage barrier; stage / accumulator releases
//               are committed to both CTAs; both epilogues arrive on the
//               leader's accumulator-empty barrier.  No TMA load uses
//               multicast.

template <bool PAIR>
struct TcCfg {
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // rows of B loaded per CTA
    static constexpr int A_B = BM * BK * 2;
    static constexpr int B_B = B_ROWS * BK * 2;
    static constexpr int STAGE_B = A_B + B_B;
    static constexpr int NSTAGE = PAIR ? 6 : 4;
    static constexpr int UMMA_M = PAIR ? 2 * BM : BM;
    static constexpr int SMEM = NSTAGE * STAGE_B + 1024 + BAR_BYTES + XV_BYTES + EPI_SHARED_BYTES;
};
static_assert(TcCfg<false>::SMEM <= 232448 && TcCfg<true>::SMEM <= 232448, "shared memory over 227 KB");

template <int MODE, bool PAIR>
__device__ __forceinline__ void tc_scan_body(uint8_t* smem_raw, const CUtensorMap& tmap_q, const CUtensorMap& tmap_x,
                                             const ScanArgs& a, const uint32_t idesc, unsigned* status) {
    using Cfg = TcCfg<PAIR>;
    constexpr int NST = Cfg::NSTAGE;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * Cfg::STAGE_B);
    uint64_t* empty = full + NST;
    uint64_t* tfull = empty + NST;
    uint64_t* tempty = tfull + NUM_ACC;
    uint64_t* mma_done = tempty + NUM_ACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* xv_s = reinterpret_cast<float*>(smem + NST * Cfg::STAGE_B + BAR_BYTES);
    uint32_t* cnt_s = reinterpret_cast<uint32_t*>(xv_s + 2 * BN);  // [BM]
    float* best_s = reinterpret_cast<float*>(cnt_s + BM);            // [BM]
    float* rxm_s = best_s + BM;                                      // [2][BN / 32]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    const bool leader = rank == 0;
    const int split = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    // query blocks run along y, continuing in z past the 65535 limit of y; both
    // CTAs of a pair share y and z, so they leave together
    const int64_t qblk = static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y;
    if ((PAIR ? 2 * qblk : qblk) * BM >= a.nq) return;
    const int64_t q0 = (PAIR ? (2 * qblk + rank) : qblk) * BM;
    const int64_t r_begin = static_cast<int64_t>(split) * a.rows_per_split;
    const int64_t r_end = min(a.n, r_begin + a.rows_per_split);
    const int ntiles = r_end > r_begin ? static_cast<int>((r_end - r_begin + BN - 1) / BN) : 0;
    const int nk = (a.d + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int c = 0; c < NUM_ACC; ++c) {
            mbar_init(&tfull[c], 1);
            mbar_init(&tempty[c], PAIR ? 2 * EPI_WARPS : EPI_WARPS);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_x);
    }
    if (warp == 1) {
        tmem_alloc_t<PAIR>(tmem_slot, TMEM_COLS);
        tmem_relinquish_t<PAIR>();
    }
    tc_fence_before();
    if (PAIR)
        cluster_sync_all();  // both CTAs' barriers initialised before any remote use
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // the leader's barriers as shared::cluster addresses (own barriers without a pair)
    uint32_t full_lead0 = PAIR ? map_to_rank(&full[0], 0) : smem_u32(&full[0]);
    uint32_t tempty_lead[NUM_ACC];
#pragma unroll
    for (int c = 0; c < NUM_ACC; ++c) tempty_lead[c] = PAIR ? map_to_rank(&tempty[c], 0) : smem_u32(&tempty[c]);

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool ok = true;
            for (int t = 0; t < ntiles && ok; ++t) {
                const int row0 = static_cast<int>(r_begin + static_cast<int64_t>(t) * BN) +
                                 static_cast<int>(rank) * Cfg::B_ROWS;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + stage * Cfg::STAGE_B;
                    if (PAIR) {
                        if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_B);
                        const uint32_t bar = full_lead0 + static_cast<uint32_t>(stage * sizeof(uint64_t));
                        tma_load_2d_pair(&tmap_q, bar, sa, kb * BK, static_cast<int>(q0));
                        tma_load_2d_pair(&tmap_x, bar, sa + Cfg::A_B, kb * BK, row0);
                    } else {
                        mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_B);
                        tma_load_2d(&tmap_q, &full[stage], sa, kb * BK, static_cast<int>(q0));
                        tma_load_2d(&tmap_x, &full[stage], sa + Cfg::A_B, kb * BK, row0);
                    }
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == NST) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                if (status) atomicOr(status, DEV_TIMEOUT_PRODUCER);
                // let the loads tracked by this CTA's barriers land before its
                // shared memory is released
                if (!PAIR || leader)
                    for (int s = 0; s < NST; ++s)
                        if (issued_mask & (1u << s)) {
                            const uint64_t t0 = globaltimer_ns();
                            while (!mbar_try_wait(&full[s], (issued_phase >> s) & 1) &&
                                   globaltimer_ns() - t0 < kWaitLimitNs) {
                            }
                        }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------------------------------------- MMA issuer
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true, any = false;
            for (int t = 0; t < ntiles && ok; ++t) {
                const int acc = t & 1;
                const uint32_t acc_phase = (t >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * Cfg::STAGE_B);
                    const uint64_t adesc = make_sdesc(a_addr);
                    const uint64_t bdesc = make_sdesc(a_addr + Cfg::A_B);
#pragma unroll
                    for (int k = 0; k < BK / UK; ++k) {
                        if (PAIR)
                            umma_f16_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                        else
                            umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    any = true;
                    if (PAIR)
                        umma_commit_pair_both(&empty[stage]);
                    else
                        umma_commit(&empty[stage]);
                    if (++stage == NST) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (ok) {
                    if (PAIR)
                        umma_commit_pair_both(&tfull[acc]);
                    else
                        umma_commit(&tfull[acc]);
                }
            }
            if (!ok) {
                *abort_flag = 1;
                if (status) atomicOr(status, DEV_TIMEOUT_MMA);
            }
            if (any) {
                // wait for every MMA this thread issued before TMEM is freed
                if (PAIR)
                    umma_commit_pair_self(mma_done);
                else
                    umma_commit(mma_done);
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(mma_done, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
                }
            }
        }
    } else {
        // -------------------------------------------------- epilogue
        // Eight warps, two per TMEM lane quadrant: thread = one query row =
        // one TMEM lane; warp half h drains columns [128 h, 128 h + 128) of
        // each 256-row tile.  Per tile the 256 per-row values xv[] sit in
        // shared memory (loaded one tile ahead, one row per thread); per
        // 32-column chunk the pass test is branch-free (FFMA + FSETP + OR per
        // column, four independent OR chains), and a lane with hits reserves
        // slots in its query's list with one shared-memory atomic and picks
        // each hit out of its registers with a select network.
        const int ew = warp - 2;          // 0..7
        const int quad = warp & 3;        // TMEM lanes this warp may read
        const int half = ew >> 2;         // which 128 columns of each tile
        const int etid = ew * 32 + lane;  // 0..255
        const int qrow = quad * 32 + lane;
        const int64_t q = q0 + qrow;
        const bool qvalid = q < a.nq;
        const float qv = (qvalid && a.qv) ? a.qv[q] : 0.f;
        FilterCoef fc = {0.f, -INFINITY};
        if (MODE == SCAN_FILTER) {
            const float thr = (qvalid && a.thr) ? a.thr[q] : __int_as_float(0x7fc00000);
            fc = filter_coef(a.metric, a.cos_small, thr, qv);
        }
        const float nA = -fc.A;
        uint2* cbase = (MODE == SCAN_FILTER && qvalid)
                           ? a.cand + (static_cast<int64_t>(split) * a.nq + q) * a.cap
                           : nullptr;
        const uint32_t cap = static_cast<uint32_t>(min(a.cap, static_cast<int64_t>(0xffffffffu)));
        if (MODE == SCAN_FILTER && half == 0) cnt_s[qrow] = 0u;
        float best = -INFINITY;
        uint32_t best_r = 0;
        float gb = -INFINITY;  // running group maximum (groups of 64 / 128 rows)
        const float* __restrict__ xvp = a.xv;
        const int64_t step = a.row_step;
        // cosine group maxima rank by t = dot / xv: the tile holds 1 / xv
        // (0 for a zero row, whose dot is 0), one division per row and tile
        const bool cos_recip = MODE == SCAN_GROUPMAX && a.metric == RDB_METRIC_COSINE;
        auto load_xv = [&](int t) -> float {
            const int64_t r = r_begin + static_cast<int64_t>(t) * BN + etid;
            const float x = (xvp && r < r_end) ? __ldg(xvp + r * step) : 0.f;
            return cos_recip ? (x > 0.f ? 1.f / x : 0.f) : x;
        };
        float xv_next = 0.f;
        // the row values of a tile into buffer b; cosine group maxima also
        // keep each 32-row block's largest 1 / xv (a warp holds 32 rows)
        auto put_xv = [&](int b, float x) {
            xv_s[b * BN + etid] = x;
            if (cos_recip) {
                const unsigned m = __reduce_max_sync(0xffffffffu, __float_as_uint(x));  // x >= 0
                if (lane == 0) rxm_s[b * (BN / 32) + etid / 32] = __uint_as_float(m);
            }
        };
        if (ntiles > 0) put_xv(0, load_xv(0));
        epi_bar_sync();
        for (int t = 0; t < ntiles; ++t) {
            const int acc = t & 1;
            const uint32_t acc_phase = (t >> 1) & 1;
            if (t + 1 < ntiles) xv_next = load_xv(t + 1);
            // all eight epilogue warps leave together if any wait gave up
            if (!epi_bar_and(mbar_wait(&tfull[acc], acc_phase, abort_flag))) {
                *abort_flag = 1;
                if (status) atomicOr(status, DEV_TIMEOUT_EPILOGUE);
                break;
            }
            tc_fence_after();
            const int64_t row0 = r_begin + static_cast<int64_t>(t) * BN;
            const float* xs_tile = xv_s + acc * BN;
            // 32-column chunk c (0..7 within the tile) of this tile: the
            // accumulator values are in r
            auto process_chunk = [&](const uint32_t (&r)[32], const int c) {
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                const int64_t col0 = row0 + c * 32;
                const int64_t nv64 = r_end - col0;
                const uint32_t valid = nv64 >= 32 ? 0xffffffffu : (nv64 > 0 ? ((1u << nv64) - 1u) : 0u);
                const float4* xs4 = reinterpret_cast<const float4*>(xs_tile + c * 32);
                if (MODE == SCAN_FILTER) {
                    uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        const float4 x4 = xs4[j4];
                        const int j = 4 * j4;
                        m0 |= fmaf(nA, x4.x, v[j]) >= fc.B ? 1u << j : 0u;
                        m1 |= fmaf(nA, x4.y, v[j + 1]) >= fc.B ? 2u << j : 0u;
                        m2 |= fmaf(nA, x4.z, v[j + 2]) >= fc.B ? 4u << j : 0u;
                        m3 |= fmaf(nA, x4.w, v[j + 3]) >= fc.B ? 8u << j : 0u;
                    }
                    uint32_t m = (m0 | m1) | (m2 | m3);
                    m &= valid;
                    if (!qvalid) m = 0;
                    if (m) {
                        uint32_t slot = atomicAdd(&cnt_s[qrow], static_cast<uint32_t>(__popc(m)));
                        do {
                            const int j = __ffs(m) - 1;
                            m &= m - 1;
                            if (slot < cap) {
                                const float sc = final_score(a.metric, a.cos_small, pick32(v, j), qv,
                                                             xs_tile[c * 32 + j]);
                                cbase[slot] = make_uint2(__float_as_uint(sc), static_cast<uint32_t>(col0 + j));
                            }
                            ++slot;
                        } while (m);
                    }
                } else if (MODE == SCAN_ARGMIN) {
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        const float4 x4 = xs4[j4];
                        const float xx[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int j = 4 * j4 + u;
                            const float tt = fmaf(-0.5f, xx[u], v[j]);
                            if (((valid >> j) & 1u) && tt > best) {
                                best = tt;
                                best_r = static_cast<uint32_t>(col0 + j);
                            }
                        }
                    }
                } else if (MODE == SCAN_GROUPMAX) {
                    // ranking values, larger = better: L2 in the order-reversed
                    // space dot - xv / 2; cosine t = dot / xv (the tile holds
                    // 1 / xv), turned into a score bound per group below; dot
                    // as is
                    const bool cos_eps = a.metric == RDB_METRIC_COSINE && !a.cos_small;
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4) {
                        const float4 x4 = xs4[j4];
                        const float xx[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int j = 4 * j4 + u;
                            float sc;
                            if (a.metric == RDB_METRIC_L2)
                                sc = fmaf(-0.5f, xx[u], v[j]);
                            else if (a.metric == RDB_METRIC_COSINE)
                                sc = v[j] * xx[u];
                            else
                                sc = v[j];
                            v[j] = ((valid >> j) & 1u) ? sc : -INFINITY;
                        }
                    }
                    const int g = a.group;
                    const float* rxm = rxm_s + acc * (BN / 32);  // this tile's 32-row block maxima of 1 / xv
                    // group maximum -> the value written: for cosine a lower
                    // bound on the score of the row with the largest t, which
                    // is dot / (qv xv + 1e-8) = t / (qv + 1e-8 / xv) (d > 128;
                    // t / qv for d <= 128, whose values carry the epsilon under
                    // the square roots): t / (qv + 1e-8 wmax) for t > 0 with
                    // wmax at least the group's largest 1 / xv (the maximum
                    // over the 32-row blocks it lies in), t / qv otherwise, so
                    // the k-th best of the group bounds is still at most the
                    // k-th best score (rounding: a few ulps, within the
                    // threshold's 2^-16 slack).  Blocks [b0, b1] of the tile.
                    auto emit = [&](float* p, float mx, int b0, int b1) {
                        float out = mx;
                        if (a.metric == RDB_METRIC_L2) {
                            out = fmaxf(qv - 2.f * mx, 0.f);
                        } else if (a.metric == RDB_METRIC_COSINE) {
                            float wmax = 0.f;
                            if (cos_eps)
                                for (int b = b0; b <= b1; ++b) wmax = fmaxf(wmax, rxm[b]);
                            out = mx > 0.f ? mx / (cos_eps ? fmaf(1e-8f, wmax, qv) : qv)
                                           : (mx < 0.f ? mx / qv : mx);
                        }
                        *p = out;
                    };
                    if (qvalid) {
                        float* gout = a.group_out + q * a.ngroups;
                        if (g > 32) {
                            // groups of 64 / 128 span two / four chunks of this warp
                            float m0 = v[0], m1 = v[1];
#pragma unroll
                            for (int j = 2; j < 32; j += 2) {
                                m0 = fmaxf(m0, v[j]);
                                m1 = fmaxf(m1, v[j + 1]);
                            }
                            gb = fmaxf(gb, fmaxf(m0, m1));
                            if (((c + 1) * 32) % g == 0) {
                                const int64_t gs = (col0 + 32) - g;  // first row of the group
                                if (gs < r_end) emit(gout + gs / g, gb, c + 1 - g / 32, c);
                                gb = -INFINITY;
                            }
                        } else if (g == 16) {
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                float m0 = v[16 * h];
#pragma unroll
                                for (int j = 1; j < 16; ++j) m0 = fmaxf(m0, v[16 * h + j]);
                                if ((valid >> (16 * h)) & 1u) emit(gout + col0 / 16 + h, m0, c, c);
                            }
                        } else {
                            float gm = -INFINITY;
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                gm = fmaxf(gm, v[j]);
                                if (((j + 1) & (g - 1)) == 0) {
                                    if ((valid >> (j + 1 - g)) & 1u) emit(gout + (col0 + j) / g, gm, c, c);
                                    gm = -INFINITY;
                                }
                            }
                        }
                    }
                } else {  // SCAN_DENSE
                    if (qvalid) {
                        float* orow = a.dense_out + q * a.ld_out + col0;
#pragma unroll
                        for (int j4 = 0; j4 < 8; ++j4) {
                            const float4 x4 = xs4[j4];
                            const float xx[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const int j = 4 * j4 + u;
                                if ((valid >> j) & 1u) orow[j] = final_score(a.metric, a.cos_small, v[j], qv, xx[u]);
                            }
                        }
                    }
                }
            };
            // TMEM loads double-buffered: chunk c + 1 is in flight while chunk c
            // is processed
            constexpr int NCH = BN / 2 / 32;  // chunks per warp half
            const int c0 = half * NCH;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN + c0 * 32);
            uint32_t ra[32], rb[32];
            tmem_ld32_async(tbase, ra);
            tmem_ld_wait(ra);
#pragma unroll 1
            for (int c = 0; c < NCH; c += 2) {
                tmem_ld32_async(tbase + static_cast<uint32_t>((c + 1) * 32), rb);
                process_chunk(ra, c0 + c);
                tmem_ld_wait(rb);
                if (c + 2 < NCH) tmem_ld32_async(tbase + static_cast<uint32_t>((c + 2) * 32), ra);
                process_chunk(rb, c0 + c + 1);
                if (c + 2 < NCH) tmem_ld_wait(ra);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(tempty_lead[acc]);
            // publish the next tile's row values (its buffer was last read in
            // tile t - 1, which every epilogue thread has finished)
            if (t + 1 < ntiles) put_xv((t + 1) & 1, xv_next);
            epi_bar_sync();
        }
        // the second warp of each quadrant hands its arg-best to the first
        if (MODE == SCAN_ARGMIN && half == 1) {
            best_s[qrow] = best;
            cnt_s[qrow] = best_r;
        }
        epi_bar_sync();
        if (qvalid && half == 0) {
            if (MODE == SCAN_FILTER)
                a.counts[static_cast<int64_t>(split) * a.nq + q] = static_cast<int>(min(cnt_s[qrow], 0x7fffffffu));
            if (MODE == SCAN_ARGMIN) {
                // larger wins, the lower row on ties (each half kept its first)
                const float b1 = best_s[qrow];
                const uint32_t r1 = cnt_s[qrow];
                if (b1 > best || (b1 == best && r1 < best_r)) {
                    best = b1;
                    best_r = r1;
                }
                const float dist = fmaxf(qv - 2.f * best, 0.f);
                a.best[static_cast<int64_t>(split) * a.nq + q] =
                    (ntiles > 0 && best > -INFINITY)
                        ? ((static_cast<unsigned long long>(float_asc_key(dist)) << 32) | best_r)
                        : ~0ull;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync_all();  // neither CTA leaves while its partner may still signal it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_t<PAIR>(tmem_base, TMEM_COLS);
    }
}

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_scan_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_x,
                   const ScanArgs a, const uint32_t idesc, unsigned* status) {
    extern __shared__ uint8_t smem_raw[];
    tc_scan_body<MODE, false>(smem_raw, tmap_q, tmap_x, a, idesc, status);
}

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    tc_scan_pair_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_x,
                        const ScanArgs a, const uint32_t idesc, unsigned* status) {
    extern __shared__ uint8_t smem_raw[];
    tc_scan_body<MODE, true>(smem_raw, tmap_q, tmap_x, a, idesc, status);
}

// --------------------------------------------------------------- host side --

template <int MODE, bool PAIR>
int launch_mode(const CUtensorMap& mq, const CUtensorMap& mx, const ScanArgs& a, uint32_t idesc,
                dim3 grid, cudaStream_t s) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    constexpr int smem = TcCfg<PAIR>::SMEM;
    if (dev < 64 && !attr[dev]) {
        if (PAIR)
            RDB_CUDA_TRY(cudaFuncSetAttribute(tc_scan_pair_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              smem));
        else
            RDB_CUDA_TRY(cudaFuncSetAttribute(tc_scan_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr[dev] = true;
    }
    if (PAIR)
        tc_scan_pair_kernel<MODE><<<grid, NUM_THREADS, smem, s>>>(mq, mx, a, idesc, device_status_word());
    else
        tc_scan_kernel<MODE><<<grid, NUM_THREADS, smem, s>>>(mq, mx, a, idesc, device_status_word());
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

template <bool PAIR>
int launch_shape(const ScanArgs& a, int mode, cudaStream_t s) {
    const int qunit = PAIR ? 2 * BM : BM;
    const int64_t gq = (a.nq + qunit - 1) / qunit;
    const int64_t gy = std::min<int64_t>(gq, 65535), gz = (gq + gy - 1) / gy;
    RDB_CHECK_ARG(gz <= 65535, "too many queries for one launch");
    CUtensorMap mq, mx;
    RDB_TRY(make_map(&mq, a.dtype, a.q, a.nq, a.d, a.ldq * 2, BK, BM));
    RDB_TRY(make_map(&mx, a.dtype, a.x, a.n, a.d, a.ldx * 2 * a.row_step, BK, TcCfg<PAIR>::B_ROWS));
    const uint32_t idesc = tc_idesc(a.dtype == RDB_BF16, TcCfg<PAIR>::UMMA_M, BN);
    dim3 grid(PAIR ? 2 * a.nsplit : a.nsplit, static_cast<unsigned>(gy), static_cast<unsigned>(gz));
    if (mode == SCAN_FILTER) return launch_mode<SCAN_FILTER, PAIR>(mq, mx, a, idesc, grid, s);
    if (mode == SCAN_ARGMIN) return launch_mode<SCAN_ARGMIN, PAIR>(mq, mx, a, idesc, grid, s);
    if (mode == SCAN_GROUPMAX) return launch_mode<SCAN_GROUPMAX, PAIR>(mq, mx, a, idesc, grid, s);
    return launch_mode<SCAN_DENSE, PAIR>(mq, mx, a, idesc, grid, s);
}

// Bounded-wait probe: one thread waits on an mbarrier of its own CTA that
// no thread ever arrives at, through the same mbar_wait as the scan roles,
// with a caller-given limit.  Nothing else is in flight (no TMA load, no
// MMA), so giving up leaves nothing behind; the timeout is recorded in the
// device status word exactly as a scan role records it.
__global__ void wait_probe_kernel(uint64_t limit_ns, unsigned* status, unsigned* out_waited_out) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool ok = mbar_wait(&bar, 0, &abort_flag, limit_ns);
        if (!ok && status) atomicOr(status, (unsigned)DEV_TIMEOUT_PROBE);
        *out_waited_out = ok ? 0u : 1u;
    }
}

}  // namespace

int launch_wait_probe(uint64_t limit_ns, unsigned* out_waited_out, cudaStream_t s) {
    wait_probe_kernel<<<1, 32, 0, s>>>(limit_ns, device_status_word(), out_waited_out);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

bool tc_use_pair(int64_t nq) { return nq > kTcQueries; }

int launch_scan_tc(const ScanArgs& a, int mode, cudaStream_t s) {
    if (a.nq <= 0 || a.n <= 0) return RDB_OK;
    RDB_CHECK_ARG(a.dtype == RDB_F16 || a.dtype == RDB_BF16, "tensor-core scan needs fp16/bf16");
    RDB_CHECK_ARG(a.rows_per_split % BN == 0, "rows_per_split must be a multiple of %d", BN);
    RDB_CHECK_ARG(a.n < (1LL << 31), "scan rows must be < 2^31 per launch");
    RDB_CHECK_ARG(((a.ldq * 2) % 16) == 0 && ((a.ldx * 2 * a.row_step) % 16) == 0,
                  "row strides must be multiples of 16 bytes");
    RDB_CHECK_ARG((reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0,
                  "base pointers must be 16-byte aligned");
    if (mode == SCAN_GROUPMAX)
        RDB_CHECK_ARG(a.group >= 1 && a.group <= BN / 2 && (a.group & (a.group - 1)) == 0 && a.n % a.group == 0,
                      "group must be a power of two <= %d dividing n", BN / 2);
    return tc_use_pair(a.nq) ? launch_shape<true>(a, mode, s) : launch_shape<false>(a, mode, s);
}

}  // namespace rdb
