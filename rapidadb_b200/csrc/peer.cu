// Peer exchange over NVLink for the row-sharded search: every rank owns one
// exchange arena (cudaMalloc, shared with the other ranks of the node as a
// CUDA IPC handle), and one kernel per exchange signals that this rank's
// source rows are ready, waits (bounded) until every other rank has signalled
// the same epoch, then reads the rows it needs straight out of the other
// ranks' arenas with plain peer loads (no multicast, no copy engine, no
// collective library).
//
// The reference is single-GPU (README.md:14 only names multi-GPU); the rows
// exchanged are those of the sharded search's three exchange steps (sample
// maxima to the owner of each query, thresholds back to every rank, per-rank
// result lists to the owner).
//
// Arena layout: bytes [0, RDB_PEER_FLAG_BYTES) hold the flags, one 64-byte
// line per slot, word p of a line written by rank p (an epoch number).  A
// rank signals slot s by storing the epoch into word `rank` of line s of
// EVERY rank's arena (release at system scope, after its own source rows were
// written by earlier work on its stream), and waits by reading its own
// arena's line s (acquire at system scope) until every word is at least the
// epoch, so all polling is local.
//
// Reuse without a second buffer: in the sharded search every exchange depends
// on all ranks, so a rank cannot overwrite a source row of epoch e before
// every other rank has signalled an exchange of epoch e + 1, which each does
// only after it has finished reading the rows of epoch e.
#include <algorithm>

#include "common.cuh"

namespace rdb {
namespace {

constexpr int PG_THREADS = 256;
constexpr int PG_UNROLL = 4;

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long* flag_word(void* base, int slot, int rank) {
    return reinterpret_cast<unsigned long long*>(static_cast<char*>(base) + 64 * slot) + rank;
}

// Units of U bytes (16 or 4): unit u of rank p's share is row u / upr, column
// u % upr of that rank's rows.  Loads are issued PG_UNROLL at a time before
// the stores, so several peer reads are in flight per thread.
template <typename U>
__device__ __forceinline__ void copy_units(const RdbPeerGather& a, int64_t total, const int64_t* first) {
    const int64_t upr = a.row_bytes / static_cast<int64_t>(sizeof(U));
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t u0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u0 < total;
         u0 += stride * PG_UNROLL) {
        U v[PG_UNROLL];
        U* dst[PG_UNROLL];
#pragma unroll
        for (int j = 0; j < PG_UNROLL; ++j) {
            const int64_t u = u0 + j * stride;
            dst[j] = nullptr;
            if (u >= total) continue;
            int p = 0;
            while (p + 1 < a.world && first[p + 1] <= u) ++p;
            const int64_t w = u - first[p], row = w / upr, col = w - row * upr;
            const char* src = static_cast<const char*>(a.base[p]) + a.src_off + (a.row0[p] + row) * a.src_row_stride;
            v[j] = __ldcg(reinterpret_cast<const U*>(src) + col);
            dst[j] = reinterpret_cast<U*>(static_cast<char*>(a.dst) + a.dst_off[p] + row * a.dst_row_stride) + col;
        }
#pragma unroll
        for (int j = 0; j < PG_UNROLL; ++j)
            if (dst[j]) *dst[j] = v[j];
    }
}

__global__ void __launch_bounds__(PG_THREADS) peer_gather_kernel(RdbPeerGather a, int vec16, uint64_t limit_ns,
                                                                 unsigned* status, unsigned* mirror) {
    __shared__ int ok;
    __shared__ int64_t first[RDB_PEER_MAX_RANKS + 1];
    if (threadIdx.x == 0) {
        // signal: this rank's source rows (written by earlier work on this
        // stream, complete before this kernel started) are ready
        if (blockIdx.x == 0)
            for (int p = 0; p < a.world; ++p) st_release_sys(flag_word(a.base[p], a.slot, a.rank), a.epoch);
        // wait until every rank has signalled this epoch (bounded)
        int good = 1;
        const uint64_t t0 = globaltimer_ns();
        for (int p = 0; p < a.world && good; ++p) {
            const unsigned long long* f = flag_word(a.base[a.rank], a.slot, p);
            while (ld_acquire_sys(f) < a.epoch) {
                if (globaltimer_ns() - t0 > limit_ns) {
                    good = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        if (!good) {
            if (status) atomicOr(status, static_cast<unsigned>(DEV_TIMEOUT_PEER));
            if (mirror) atomicOr_system(mirror, static_cast<unsigned>(DEV_TIMEOUT_PEER));
        }
        ok = good;
        const int64_t unit = vec16 ? 16 : 4;
        int64_t acc = 0;
        for (int p = 0; p < a.world; ++p) {
            first[p] = acc;
            acc += a.nrows[p] * (a.row_bytes / unit);
        }
        first[a.world] = acc;
    }
    __syncthreads();
    if (!ok) return;
    if (vec16)
        copy_units<uint4>(a, first[a.world], first);
    else
        copy_units<unsigned>(a, first[a.world], first);
}

}  // namespace
}  // namespace rdb

static bool aligned16(int64_t v) { return (v & 15) == 0; }

extern "C" {

int rdb_peer_arena_alloc(size_t bytes, void** ptr, unsigned char* handle) {
    RDB_CHECK_ARG(ptr && handle, "NULL pointer");
    RDB_CHECK_ARG(bytes >= RDB_PEER_FLAG_BYTES, "an arena holds at least its %d flag bytes", RDB_PEER_FLAG_BYTES);
    void* p = nullptr;
    RDB_CUDA_TRY(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return rdb::set_error(RDB_ERR_CUDA, "peer arena: %s", cudaGetErrorString(e));
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == RDB_PEER_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return RDB_OK;
}

int rdb_peer_arena_free(void* ptr) {
    if (ptr) RDB_CUDA_TRY(cudaFree(ptr));
    return RDB_OK;
}

int rdb_peer_arena_open(const unsigned char* handle, void** ptr) {
    RDB_CHECK_ARG(ptr && handle, "NULL pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    RDB_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = p;
    return RDB_OK;
}

int rdb_peer_arena_close(void* ptr) {
    if (ptr) RDB_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return RDB_OK;
}

int rdb_peer_gather(const RdbPeerGather* args, unsigned long long limit_ns, void* stream) {
    RDB_CHECK_ARG(args != nullptr, "NULL pointer");
    const RdbPeerGather& a = *args;
    RDB_CHECK_ARG(a.world >= 1 && a.world <= RDB_PEER_MAX_RANKS, "world must be in [1, %d]", RDB_PEER_MAX_RANKS);
    RDB_CHECK_ARG(a.rank >= 0 && a.rank < a.world, "rank out of range");
    RDB_CHECK_ARG(a.slot >= 0 && a.slot < RDB_PEER_SLOTS, "slot must be in [0, %d)", RDB_PEER_SLOTS);
    RDB_CHECK_ARG(a.epoch > 0, "epoch must be positive");
    RDB_CHECK_ARG(a.row_bytes >= 0 && a.row_bytes % 4 == 0, "row_bytes must be a multiple of 4");
    RDB_CHECK_ARG(a.src_off >= RDB_PEER_FLAG_BYTES && a.src_off % 4 == 0,
                  "src_off must lie past the flags and be a multiple of 4");
    RDB_CHECK_ARG(a.src_row_stride % 4 == 0 && a.dst_row_stride % 4 == 0, "row strides must be multiples of 4");
    RDB_CHECK_ARG(a.dst != nullptr || a.row_bytes == 0, "dst is NULL");
    RDB_CHECK_ARG(limit_ns >= 1000ull && limit_ns <= 10000000000ull, "limit_ns must be in [1 us, 10 s]");
    bool vec16 = aligned16(a.row_bytes) && aligned16(a.src_off) && aligned16(a.src_row_stride) &&
                 aligned16(a.dst_row_stride) && aligned16(reinterpret_cast<uintptr_t>(a.dst));
    int64_t units = 0;
    for (int p = 0; p < a.world; ++p) {
        RDB_CHECK_ARG(a.base[p] != nullptr, "base[%d] is NULL", p);
        RDB_CHECK_ARG(a.row0[p] >= 0 && a.nrows[p] >= 0, "negative rows for rank %d", p);
        RDB_CHECK_ARG(a.dst_off[p] % 4 == 0, "dst_off[%d] must be a multiple of 4", p);
        RDB_CHECK_ARG(a.nrows[p] == 0 || a.src_off + (a.row0[p] + a.nrows[p] - 1) * a.src_row_stride + a.row_bytes <=
                                             a.arena_bytes,
                      "rows of rank %d run past the end of its arena", p);
        vec16 = vec16 && aligned16(a.dst_off[p]) && aligned16(reinterpret_cast<uintptr_t>(a.base[p]));
        units += a.nrows[p] * (a.row_bytes / 4);
    }
    if (vec16) units /= 4;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t per_block = static_cast<int64_t>(rdb::PG_THREADS) * rdb::PG_UNROLL;
    const int blocks = static_cast<int>(std::max<int64_t>(
        1, std::min<int64_t>((units + per_block - 1) / per_block, 2 * static_cast<int64_t>(rdb::num_sms()))));
    rdb::peer_gather_kernel<<<blocks, rdb::PG_THREADS, 0, s>>>(a, vec16 ? 1 : 0, limit_ns,
                                                                rdb::device_status_word(),
                                                                rdb::status_mirror_device());
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // extern "C"
