// IVF-Flat list scan for callers that cannot allocate GPU memory.
//
// Some hosts embed this library where device allocation is off limits while
// they run: a caller that has already carved all device memory into its own
// pool, a real-time serving thread that must never block in the allocator, or
// a plug-in whose host runtime owns the CUDA context and forbids allocations
// from guest code.  rdb_ivf_flat_scan needs a scratch workspace from its
// caller; rdb_ivf_flat_scan_noalloc runs the same scan with its scratch taken
// from a fixed array compiled into this library, so after set-up
// (rdb_noalloc_init) the call allocates nothing.
//
// Costs and rules:
//   - every context that is set up (rdb_noalloc_init, or a first scan) holds
//     kNoAllocScratchBytes (8 MiB) of device memory for this array until the
//     context ends;
//   - all calls on a device share the one array: calls that overlap on the
//     GPU (on different streams, or from different host threads) race and
//     corrupt each other's results -- serialise them;
//   - the array is device memory of this library's module, which the CUDA
//     runtime loads into a context lazily (CUDA_MODULE_LOADING=LAZY is the
//     default): rdb_noalloc_init() looks the array up with
//     cudaGetSymbolAddress, which loads the module and so allocates the 8 MiB
//     at set-up time, and loads the kernels the scan launches (each kernel is
//     also loaded lazily, on first use).  Call it once per device and
//     context, with that device current, before the first scan and before
//     any stream capture.  A scan
//     whose context has not been set up this way does the lookup itself, and
//     that first call then allocates;
//   - every call looks the address up again for the context current at the
//     time (a cheap query once the module is loaded), so the address is never
//     stale after cudaDeviceReset or in a context that the host made current
//     itself;
//   - the array keeps the previous call's contents, but nothing in it needs to
//     start at zero: every scratch byte the scan reads is written earlier in
//     the same call.
#include "common.cuh"

namespace rdb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array in the current context.  The host-side
// name g_noalloc_scratch is only a stand-in for the symbol; the address that
// kernels may use comes from cudaGetSymbolAddress.
int scratch_address(void** out) {
    void* p = nullptr;
    RDB_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    *out = p;
    return RDB_OK;
}

}  // namespace
}  // namespace rdb

using namespace rdb;

extern "C" {

size_t rdb_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int rdb_noalloc_init(void) {
    void* p = nullptr;
    RDB_TRY(scratch_address(&p));
    return ivf_flat_scan_preload();
}

int rdb_ivf_flat_scan_noalloc(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d,
                              const int64_t* probe, int nprobe, const void* rows, int64_t ldx, const float* xv,
                              const int64_t* list_off, const int64_t* list_end, int nlist, const int64_t* ids,
                              int k, float* out_v,
                              int64_t* out_i, void* stream) {
    RDB_CHECK_ARG(nq >= 0 && nprobe >= 1 && nlist >= 1, "bad shape");
    const size_t need = rdb_ivf_scan_workspace(nq, nprobe, nlist);
    if (need > kNoAllocScratchBytes)
        return set_error(RDB_ERR_UNSUPPORTED,
                         "rdb_ivf_flat_scan_noalloc: nq=%lld x nprobe=%d over nlist=%d needs %zu bytes of scratch, "
                         "more than the %zu-byte static array; use rdb_ivf_flat_scan with a workspace or split the "
                         "queries",
                         (long long)nq, nprobe, nlist, need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    RDB_TRY(scratch_address(&scratch));
    return rdb_ivf_flat_scan(metric, dtype, q, nq, ldq, d, probe, nprobe, rows, ldx, xv, list_off, list_end, nlist, ids,
                             k,
                             out_v, out_i, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
