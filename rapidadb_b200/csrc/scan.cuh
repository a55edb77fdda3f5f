// Shared description of a "scan": score a block of queries against a range of
// stored rows and either keep the rows that pass a per-query threshold
// (candidate lists for the selection kernel), write the dense score matrix,
// or keep the best row per query (argmin, for k-means / list assignment).
#pragma once

#include "common.cuh"

namespace rdb {

enum ScanMode : int {
    SCAN_FILTER = 0,  // append (final score, row) pairs whose score reaches thr[q]
    SCAN_DENSE = 1,   // write final scores to dense_out[q, row]
    SCAN_ARGMIN = 2,  // best row per (split, query) by squared L2
    SCAN_GROUPMAX = 3,  // best score of every `group` consecutive logical rows
    SCAN_ARGMIN_EXACT = 4,  // CUDA cores: argmin of sum (q - x)^2, one FMA per element in order
    SCAN_PARTIAL = 5,  // fp32 TMA scan: dense_out[q, row] += dot over the K share of blockIdx.x % ksplit
};

struct ScanArgs {
    int metric;
    int cos_small;
    int dtype;

    const void* q;  // [nq, d] (row stride ldq elements)
    int64_t nq;
    int64_t ldq;

    const void* x;     // stored rows; logical row j is physical row j * row_step
    int64_t n;         // logical rows
    int64_t ldx;
    int64_t row_step;
    int d;

    const float* qv;   // [nq] per-query metric value
    const float* xv;   // per physical row metric value
    // rows stored as SQ8 codes (int8) with a per-physical-row fp32 scale:
    // the row value is fl(x_scale[row] * code); queries stay fp32 (dtype)
    int x_i8;
    const float* x_scale;
    const float* thr;  // [nq] thresholds in final-score units (NULL: accept all)

    // SCAN_FILTER: candidate lists [nsplit][nq][cap] + counts [nsplit][nq]
    uint2* cand;
    int* counts;
    int64_t cap;

    int nsplit;
    int64_t rows_per_split;  // multiple of the kernel's row tile

    // SCAN_PARTIAL: grid.x = nsplit * ksplit, dense_out zeroed by the caller
    int ksplit;

    // SCAN_DENSE (and SCAN_PARTIAL)
    float* dense_out;
    int64_t ld_out;

    // SCAN_ARGMIN: [nsplit][nq] best (score key, row) pairs
    unsigned long long* best;

    // SCAN_GROUPMAX: group_out[q][row / group] = best final score (approximate
    // to a few ulps) over logical rows [g * group, (g + 1) * group); group is a
    // power of two <= 128 and n a multiple of it.
    float* group_out;
    int group;
    int64_t ngroups;
};

// CUDA-core scan (any dtype).  Grid = (nsplit, ceil(nq / 32)).
int launch_scan_simt(const ScanArgs& a, int mode, cudaStream_t stream);
// true when launch_scan_simt runs `mode` on the TMA-fed fp32 kernel (the only
// one with SCAN_PARTIAL)
bool simt_tma_ok(const ScanArgs& a, int mode);
// dense_out[q, row] = final score of the dot product it holds (qv, xv per
// query / logical row), in place
int launch_partial_finalize(const ScanArgs& a, cudaStream_t stream);

// tcgen05 scan for fp16 / bf16 (sm_100a).  Grid = (nsplit, ceil(nq / 128)), or
// with more than 128 queries CTA pairs: (2 nsplit, ceil(nq / 256)).
int launch_scan_tc(const ScanArgs& a, int mode, cudaStream_t stream);
bool tc_use_pair(int64_t nq);

// Row tiles of the two kernels (rows_per_split must be a multiple).
constexpr int kSimtRows = 256;
constexpr int kSimtQueries = 32;
constexpr int kTcRows = 256;
constexpr int kTcQueries = 128;

}  // namespace rdb
