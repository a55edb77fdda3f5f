// Stable counting sort of ids by label: per-block label histograms ->
// per-(block, label) offsets -> a per-block stable scatter that ranks equal
// labels inside each 1024-element tile with a shared-memory bitonic sort of
// (label, position) keys.  Integer atomics only touch shared-memory
// histograms, and the output order is deterministic.  Used by the k-means
// update (points by centroid), by IVF list building (rows by list) and by the
// list-major IVF scans (probe entries by list).
#include <algorithm>

#include "sort.cuh"

namespace rdb {
namespace {

constexpr int kSortTile = 1024;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__global__ void label_hist_kernel(const int32_t* __restrict__ labels, int64_t n, int K, int64_t per_block,
                                  int* __restrict__ blockhist) {
    extern __shared__ int h[];
    for (int c = threadIdx.x; c < K; c += blockDim.x) h[c] = 0;
    __syncthreads();
    const int64_t lo = (int64_t)blockIdx.x * per_block, hi = min(n, lo + per_block);
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) atomicAdd(&h[labels[i]], 1);
    __syncthreads();
    for (int c = threadIdx.x; c < K; c += blockDim.x) blockhist[(int64_t)blockIdx.x * K + c] = h[c];
}

// per centroid: running start of each block's run, total count
__global__ void label_offsets_kernel(int nblk, int K, const int* __restrict__ blockhist, int* __restrict__ boff,
                                     int64_t* __restrict__ counts) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= K) return;
    int run = 0;
    for (int b = 0; b < nblk; ++b) {
        boff[(int64_t)b * K + c] = run;
        run += blockhist[(int64_t)b * K + c];
    }
    counts[c] = run;
}

// exclusive scan of counts -> seg_start[0..K] (one block)
__global__ void seg_scan_kernel(const int64_t* __restrict__ counts, int K, int64_t* __restrict__ seg_start) {
    __shared__ int64_t part[1024];
    const int per = (K + blockDim.x - 1) / blockDim.x;
    const int c0 = threadIdx.x * per, c1 = min(K, c0 + per);
    int64_t s = 0;
    for (int c = c0; c < c1; ++c) s += counts[c];
    part[threadIdx.x] = s;
    __syncthreads();
    for (int o = 1; o < (int)blockDim.x; o <<= 1) {
        int64_t v = threadIdx.x >= (unsigned)o ? part[threadIdx.x - o] : 0;
        __syncthreads();
        part[threadIdx.x] += v;
        __syncthreads();
    }
    int64_t run = part[threadIdx.x] - s;
    for (int c = c0; c < c1; ++c) {
        seg_start[c] = run;
        run += counts[c];
    }
    if (threadIdx.x == blockDim.x - 1) seg_start[K] = part[threadIdx.x];
}

// stable scatter of point ids into label order
__global__ void __launch_bounds__(kSortTile) label_scatter_kernel(const int32_t* __restrict__ labels, int64_t n,
                                                                   int K, int64_t per_block,
                                                                   const int* __restrict__ boff,
                                                                   const int64_t* __restrict__ seg_start,
                                                                   int64_t* __restrict__ perm) {
    extern __shared__ unsigned long long sm[];
    unsigned long long* keys = sm;                                  // kSortTile
    long long* cursor = reinterpret_cast<long long*>(sm + kSortTile);  // K
    for (int c = threadIdx.x; c < K; c += blockDim.x)
        cursor[c] = seg_start[c] + boff[(int64_t)blockIdx.x * K + c];
    const int64_t lo = (int64_t)blockIdx.x * per_block, hi = min(n, lo + per_block);
    for (int64_t base = lo; base < hi; base += kSortTile) {
        __syncthreads();
        const int64_t i = base + threadIdx.x;
        keys[threadIdx.x] = i < hi ? (((unsigned long long)(uint32_t)labels[i] << 32) | threadIdx.x) : ~0ull;
        __syncthreads();
        for (int size = 2; size <= kSortTile; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                int p = threadIdx.x;
                int q = p ^ stride;
                if (q > p) {
                    bool up = (p & size) == 0;
                    unsigned long long x = keys[p], y = keys[q];
                    if ((x > y) == up) {
                        keys[p] = y;
                        keys[q] = x;
                    }
                }
                __syncthreads();
            }
        const int p = threadIdx.x;
        const unsigned long long key = keys[p];
        const bool valid = key != ~0ull;
        const uint32_t lab = (uint32_t)(key >> 32);
        // first sorted position holding this label
        int lo_p = 0, hi_p = p;
        while (lo_p < hi_p) {
            int mid = (lo_p + hi_p) >> 1;
            if ((uint32_t)(keys[mid] >> 32) < lab) lo_p = mid + 1; else hi_p = mid;
        }
        const int rank = p - lo_p;
        const bool last = p == kSortTile - 1 || (uint32_t)(keys[p + 1] >> 32) != lab;
        long long slot = 0;
        if (valid) slot = cursor[lab] + rank;
        __syncthreads();
        if (valid) {
            perm[slot] = base + (int64_t)(uint32_t)key;
            if (last) cursor[lab] += rank + 1;
        }
    }
}

struct SortWs {
    int nblk;
    int64_t per_block;
    size_t off_hist, off_boff, off_counts, bytes;
};

SortWs sort_ws(int64_t n, int K) {
    SortWs w;
    // about two 1024-element tiles per block, as many blocks as keep the
    // per-(block, label) histograms and offsets within 2 MB, at most 2 per SM
    const int64_t by_mem = std::max<int64_t>(1, (int64_t(1) << 18) / std::max(K, 1));
    w.nblk = (int)std::max<int64_t>(1, std::min<int64_t>({(n + 2047) / 2048, by_mem, 296}));
    w.per_block = (n + w.nblk - 1) / w.nblk;
    size_t off = 0;
    w.off_hist = off;
    off = align_up(off + sizeof(int) * (size_t)w.nblk * K, 256);
    w.off_boff = off;
    off = align_up(off + sizeof(int) * (size_t)w.nblk * K, 256);
    w.off_counts = off;
    off = align_up(off + sizeof(int64_t) * K, 256);
    w.bytes = off;
    return w;
}

}  // namespace

size_t label_sort_workspace(int64_t n, int K) { return sort_ws(n, K).bytes; }

int label_sort_preload() {
    cudaFuncAttributes fa;
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, label_hist_kernel));
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, label_offsets_kernel));
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, seg_scan_kernel));
    RDB_CUDA_TRY(cudaFuncGetAttributes(&fa, label_scatter_kernel));
    return RDB_OK;
}

int label_sort(const int32_t* labels, int64_t n, int K, int64_t* seg_start, int64_t* perm, int64_t* counts,
               void* ws, size_t ws_bytes, cudaStream_t s) {
    RDB_CHECK_ARG(K >= 1 && K <= kMaxLabels, "label count must be in [1, %d]", kMaxLabels);
    SortWs w = sort_ws(n, K);
    if (ws_bytes < w.bytes) return set_error(RDB_ERR_WORKSPACE, "workspace too small: %zu < %zu", ws_bytes, w.bytes);
    char* base = static_cast<char*>(ws);
    int* hist = reinterpret_cast<int*>(base + w.off_hist);
    int* boff = reinterpret_cast<int*>(base + w.off_boff);
    if (!counts) counts = reinterpret_cast<int64_t*>(base + w.off_counts);
    if (n == 0) {
        RDB_CUDA_TRY(cudaMemsetAsync(seg_start, 0, sizeof(int64_t) * (K + 1), s));
        RDB_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int64_t) * K, s));
        return RDB_OK;
    }
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        RDB_CUDA_TRY(cudaFuncSetAttribute(label_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)(sizeof(int) * kMaxLabels)));
        RDB_CUDA_TRY(cudaFuncSetAttribute(label_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)(sizeof(unsigned long long) * kSortTile + sizeof(long long) * kMaxLabels)));
        attr[dev] = true;
    }
    label_hist_kernel<<<w.nblk, 1024, sizeof(int) * K, s>>>(labels, n, K, w.per_block, hist);
    RDB_LAUNCH_CHECK();
    label_offsets_kernel<<<(K + 255) / 256, 256, 0, s>>>(w.nblk, K, hist, boff, counts);
    RDB_LAUNCH_CHECK();
    seg_scan_kernel<<<1, 1024, 0, s>>>(counts, K, seg_start);
    RDB_LAUNCH_CHECK();
    label_scatter_kernel<<<w.nblk, kSortTile, sizeof(unsigned long long) * kSortTile + sizeof(long long) * K, s>>>(
        labels, n, K, w.per_block, boff, seg_start, perm);
    RDB_LAUNCH_CHECK();
    return RDB_OK;
}

}  // namespace rdb

using namespace rdb;

extern "C" {

size_t rdb_label_sort_workspace(int64_t n, int K) { return label_sort_workspace(n, K); }

int rdb_label_sort(const int32_t* labels, int64_t n, int K, int64_t* seg_start, int64_t* perm, int64_t* counts,
                   void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(n >= 0, "bad shape");
    RDB_CHECK_ARG(seg_start && (n == 0 || (labels && perm)) && ws, "NULL pointer");
    return label_sort(labels, n, K, seg_start, perm, counts, ws, ws_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
