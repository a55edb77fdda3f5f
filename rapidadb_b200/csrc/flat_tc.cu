// tcgen05 fused scan for fp16 / bf16 rows (sm_100a).
//
// One CTA = 128 queries (UMMA M) x a contiguous split of rows, walked in tiles
// of 256 rows (UMMA N).  Warp roles:
//   warp 0      TMA producer: per K block of 64 (one 128-byte swizzle atom)
//               loads the 128 x 64 query tile and the 256 x 64 row tile into a
//               4-stage shared-memory ring (SWIZZLE_128B, K-major).
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32 accumulators);
//               one lane issues tcgen05.mma kind::f16 (K = 16 per instruction)
//               and commits stage releases / accumulator-ready barriers.
//   warps 2..5  epilogue: each thread owns one query row (one TMEM lane),
//               reads 32 accumulator columns per tcgen05.ld and keeps only the
//               rows whose dot product passes the query's threshold
//               (dot >= A * xv[row] + B, see filter_coef), appending
//               (dot, row) to the query's private candidate list.  Nothing
//               else of the [queries, rows] score tile leaves the SM.
// While the epilogue drains one accumulator the MMA fills the other.
//
// Every mbarrier wait is bounded (kWaitLimitNs): a role that gives up sets the
// CTA abort flag and a bit in the device status word, waits (bounded) for its
// own in-flight TMA loads / MMAs, and the CTA frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "scan.cuh"

namespace rdb {
namespace {

constexpr int BM = kTcQueries;  // 128
constexpr int BN = kTcRows;     // 256
constexpr int BK = 64;
constexpr int UK = 16;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = 512;
constexpr int NUM_THREADS = 192;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;

static_assert(NUM_ACC * BN <= TMEM_COLS, "accumulators exceed TMEM allocation");

// ------------------------------------------------------------ PTX wrappers --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase of `parity`; false when it gave up (time limit or
// another role raised the abort flag).
__device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int x,
                                            int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row core groups
// 1024 bytes apart (SBO), leading offset unused for swizzled K-major (1),
// descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr) {
    uint64_t desc = 0;
    desc |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    desc |= static_cast<uint64_t>(1) << 16;
    desc |= static_cast<uint64_t>(1024 >> 4) << 32;
    desc |= static_cast<uint64_t>(1) << 46;
    desc |= static_cast<uint64_t>(2) << 61;
    return desc;
}

// Instruction descriptor, kind::f16: D fp32, A/B fp16 (0) or bf16 (1),
// both K-major, N = BN, M = BM.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
           (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

// ------------------------------------------------------------------ kernel --

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_scan_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_x,
                   const ScanArgs a, const uint32_t idesc, unsigned* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + NUM_ACC;
    uint64_t* mma_done = tempty + NUM_ACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x;
    const int64_t q0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t r_begin = static_cast<int64_t>(split) * a.rows_per_split;
    const int64_t r_end = min(a.n, r_begin + a.rows_per_split);
    const int ntiles = r_end > r_begin ? static_cast<int>((r_end - r_begin + BN - 1) / BN) : 0;
    const int nk = (a.d + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int c = 0; c < NUM_ACC; ++c) {
            mbar_init(&tfull[c], 1);
            mbar_init(&tempty[c], 4);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_x);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool ok = true;
            for (int t = 0; t < ntiles && ok; ++t) {
                const int row0 = static_cast<int>(r_begin + static_cast<int64_t>(t) * BN);
                for (int kb = 0; kb < nk; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                    uint8_t* sa = smem + stage * STAGE_BYTES;
                    tma_load_2d(&tmap_q, &full[stage], sa, kb * BK, static_cast<int>(q0));
                    tma_load_2d(&tmap_x, &full[stage], sa + A_BYTES, kb * BK, row0);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                if (status) atomicOr(status, DEV_TIMEOUT_PRODUCER);
                // let this thread's loads land before the CTA's shared memory is released
                for (int s = 0; s < STAGES; ++s)
                    if (issued_mask & (1u << s)) {
                        const uint64_t t0 = globaltimer_ns();
                        while (!mbar_try_wait(&full[s], (issued_phase >> s) & 1) &&
                               globaltimer_ns() - t0 < kWaitLimitNs) {
                        }
                    }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
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
                    const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
                    const uint64_t adesc = make_sdesc(a_addr);
                    const uint64_t bdesc = make_sdesc(a_addr + A_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / UK; ++k)
                        umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc,
                                 (kb > 0 || k > 0) ? 1u : 0u);
                    any = true;
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (ok) umma_commit(&tfull[acc]);
            }
            if (!ok) {
                *abort_flag = 1;
                if (status) atomicOr(status, DEV_TIMEOUT_MMA);
            }
            if (any) {
                // wait for every MMA this thread issued before TMEM is freed
                umma_commit(mma_done);
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(mma_done, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
                }
            }
        }
    } else {
        // -------------------------------------------------- epilogue
        const int quad = warp & 3;  // TMEM lanes this warp may read
        const int qrow = quad * 32 + lane;
        const int64_t q = q0 + qrow;
        const bool qvalid = q < a.nq;
        const float qv = (qvalid && a.qv) ? a.qv[q] : 0.f;
        FilterCoef fc = {0.f, -INFINITY};
        if (MODE == SCAN_FILTER) {
            const float thr = (qvalid && a.thr) ? a.thr[q] : __int_as_float(0x7fc00000);
            fc = filter_coef(a.metric, a.cos_small, thr, qv);
        }
        uint2* cbase = (MODE == SCAN_FILTER && qvalid)
                           ? a.cand + (static_cast<int64_t>(split) * a.nq + q) * a.cap
                           : nullptr;
        int64_t cnt = 0;
        float best = -INFINITY;
        uint32_t best_r = 0;
        const float* __restrict__ xvp = a.xv;
        const int64_t step = a.row_step;
        for (int t = 0; t < ntiles; ++t) {
            const int acc = t & 1;
            const uint32_t acc_phase = (t >> 1) & 1;
            if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) {
                *abort_flag = 1;
                if (status) atomicOr(status, DEV_TIMEOUT_EPILOGUE);
                break;
            }
            tc_fence_after();
            const int64_t row0 = r_begin + static_cast<int64_t>(t) * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                float v[32];
                tmem_ld32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                              static_cast<uint32_t>(acc * BN + c * 32),
                          v);
                const int64_t col0 = row0 + c * 32;
                const int nvalid = static_cast<int>(min(static_cast<int64_t>(32), r_end - col0));
                float xv[32];
                if (step == 1 && nvalid == 32 && xvp) {
                    const float4* p4 = reinterpret_cast<const float4*>(xvp + col0);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float4 f = __ldg(p4 + j);
                        xv[4 * j] = f.x;
                        xv[4 * j + 1] = f.y;
                        xv[4 * j + 2] = f.z;
                        xv[4 * j + 3] = f.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        xv[j] = (j < nvalid && xvp) ? __ldg(xvp + (col0 + j) * step) : 0.f;
                }
                if (MODE == SCAN_FILTER) {
                    if (qvalid) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (j < nvalid && v[j] >= fmaf(fc.A, xv[j], fc.B)) {
                                if (cnt < a.cap)
                                    cbase[cnt] = make_uint2(__float_as_uint(v[j]),
                                                            static_cast<uint32_t>(col0 + j));
                                ++cnt;
                            }
                        }
                    }
                } else if (MODE == SCAN_ARGMIN) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float tt = fmaf(-0.5f, xv[j], v[j]);
                        if (j < nvalid && tt > best) {
                            best = tt;
                            best_r = static_cast<uint32_t>(col0 + j);
                        }
                    }
                } else {  // SCAN_DENSE
                    if (qvalid)
                        for (int j = 0; j < nvalid; ++j)
                            a.dense_out[q * a.ld_out + col0 + j] =
                                final_score(a.metric, a.cos_small, v[j], qv, xv[j]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        if (qvalid) {
            if (MODE == SCAN_FILTER)
                a.counts[static_cast<int64_t>(split) * a.nq + q] =
                    static_cast<int>(min(cnt, static_cast<int64_t>(0x7fffffff)));
            if (MODE == SCAN_ARGMIN) {
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
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// --------------------------------------------------------------- host side --

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult qres;
        void* p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &qres) == cudaSuccess &&
            qres == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

int make_map(CUtensorMap* m, int dtype, const void* base, int64_t rows, int d, int64_t ld_bytes,
             int box_rows) {
    auto fn = encode_fn();
    if (!fn) return set_error(RDB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_bytes)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, dtype == RDB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(RDB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return RDB_OK;
}

template <int MODE>
int launch_mode(const CUtensorMap& mq, const CUtensorMap& mx, const ScanArgs& a, uint32_t idesc,
                dim3 grid, cudaStream_t s) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        RDB_CUDA_TRY(cudaFuncSetAttribute(tc_scan_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          SMEM_BYTES));
        attr[dev] = true;
    }
    tc_scan_kernel<MODE><<<grid, NUM_THREADS, SMEM_BYTES, s>>>(mq, mx, a, idesc, device_status_word());
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // namespace

int launch_scan_tc(const ScanArgs& a, int mode, cudaStream_t s) {
    if (a.nq <= 0 || a.n <= 0) return RDB_OK;
    RDB_CHECK_ARG(a.dtype == RDB_F16 || a.dtype == RDB_BF16, "tensor-core scan needs fp16/bf16");
    RDB_CHECK_ARG(a.rows_per_split % BN == 0, "rows_per_split must be a multiple of %d", BN);
    RDB_CHECK_ARG(a.n < (1LL << 31), "scan rows must be < 2^31 per launch");
    RDB_CHECK_ARG(((a.ldq * 2) % 16) == 0 && ((a.ldx * 2 * a.row_step) % 16) == 0,
                  "row strides must be multiples of 16 bytes");
    RDB_CHECK_ARG((reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0,
                  "base pointers must be 16-byte aligned");
    int64_t gy = (a.nq + BM - 1) / BM;
    RDB_CHECK_ARG(gy <= 65535, "too many queries for one launch");
    CUtensorMap mq, mx;
    RDB_TRY(make_map(&mq, a.dtype, a.q, a.nq, a.d, a.ldq * 2, BM));
    RDB_TRY(make_map(&mx, a.dtype, a.x, a.n, a.d, a.ldx * 2 * a.row_step, BN));
    const uint32_t idesc = make_idesc(a.dtype == RDB_BF16);
    dim3 grid(a.nsplit, static_cast<unsigned>(gy));
    if (mode == SCAN_FILTER) return launch_mode<SCAN_FILTER>(mq, mx, a, idesc, grid, s);
    if (mode == SCAN_ARGMIN) return launch_mode<SCAN_ARGMIN>(mq, mx, a, idesc, grid, s);
    return launch_mode<SCAN_DENSE>(mq, mx, a, idesc, grid, s);
}

}  // namespace rdb
