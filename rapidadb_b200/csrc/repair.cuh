// Device-side completion of flat search (internal interface): per-query
// values, and the exact repair of candidate lists that overflowed.
#pragma once

#include "common.cuh"

namespace rdb {

struct RepairArgs {
    int metric;
    int cos_small;
    int dtype;
    const void* q;  // [nq, d], row stride ldq
    int64_t nq;
    int64_t ldq;
    const void* x;  // [n, d] stored rows, row stride ldx
    int64_t n;
    int64_t ldx;
    int d;
    int k;
    int x_i8;                 // rows are SQ8 codes: value = fl(x_scale[row] * code)
    const float* x_scale;
    const float* qv;  // [nq] per-query values (cosine)
    const float* xv;  // [n] per-row values (cosine)
    const unsigned* flag;    // nonzero when some list of this chunk overflowed
    const unsigned* mark_q;  // [nq] 1 for the queries to repair
    uint2* cand;             // [nsplit][nq][cap] candidate lists, rewritten for marked queries
    int* counts;             // [nsplit][nq]
    int64_t cap;
    int nsplit;
    int64_t rows_per_split;
    int buf_keys;  // repair_buffer_keys(k, cap)
    const unsigned* status;   // device status word (NULL: not forwarded)
    unsigned* status_mirror;  // host-mapped word receiving a nonzero status
};

// qv[q] = vec_value(metric, |q|^2) for nq queries of stride ldq; clears
// *flag (may be NULL) in the same launch.
int launch_query_prep(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d, float* qv,
                      unsigned* flag, cudaStream_t s);
// Shared-memory keys the repair kernel needs for k results per list of cap.
int repair_buffer_keys(int k, int64_t cap);
int launch_flat_repair(const RepairArgs& a, cudaStream_t s);

}  // namespace rdb
