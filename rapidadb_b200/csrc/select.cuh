// Per-query top-k selection over candidate lists (internal interface).
#pragma once

#include "common.cuh"

namespace rdb {

enum SelectInput : int {
    SEL_CANDIDATES = 0,  // segmented (final score bits, row) pairs from a scan kernel
    SEL_DENSE = 1,       // one row of a dense [B, N] fp32 score matrix
    SEL_MERGE = 2,       // G sorted lists of (score, int64 id)
};

enum SelectOutput : int {
    SEL_OUT_TOPK = 0,       // sorted best-k scores + ids
    SEL_OUT_THRESHOLD = 1,  // only the k-th best score
};

struct SelectArgs {
    int input;
    int output;
    int64_t nq;  // number of queries (rows)
    int k;       // results per query
    int largest;

    // SEL_CANDIDATES
    const uint2* cand;   // [nsplit][nq][cap]
    const int* counts;   // [nsplit][nq] (may exceed cap: overflow)
    int64_t cap;
    int nsplit;
    int metric;
    int cos_small;
    const float* qv;     // [nq]
    const float* xv;     // per physical row
    int64_t row_step;    // candidate row r is physical row r * row_step

    // SEL_DENSE
    const float* dense;  // [nq][dense_n]
    int64_t dense_n;

    // SEL_MERGE
    const float* merge_v;  // [G][nq][kin]; element (g, q, t) at merge_v[g * gstride_v + q * ldv + t]
    const int64_t* merge_i;  // same shape; element (g, q, t) at merge_i[g * gstride_i + q * ldi + t]
    int64_t gstride_v;       // 0: nq * ldv
    int64_t gstride_i;       // 0: nq * ldi
    int64_t ldv;             // row (query) stride of the scores, 0: kin
    int64_t ldi;             // row stride of the ids, 0: kin
    int G;
    int kin;

    // outputs
    float* out_v;         // [nq][k]
    int64_t* out_i;       // [nq][k]
    float* out_thr;       // [nq]
    const int64_t* ids;   // physical row -> user id (NULL: row + id_offset)
    int64_t id_offset;
    unsigned* overflow;   // set to 1 when any count exceeded cap
    unsigned* mark_q;     // [nq] (SEL_CANDIDATES): 1 where the query's lists overflowed, else 0
    const unsigned* only_q;  // [nq]: process only queries marked nonzero (NULL: all)
    const unsigned* gate;    // nothing to do while *gate == 0 (NULL: always run)
    int force_cta;           // one CTA per query (select_kernel), grid of at most one CTA per SM
    int64_t expect;       // expected elements per query (0: unknown); picks the kernel
    int cache_keys;       // set by launch_select: keys per query the CTA kernel holds in shared memory

    // exact L2 rescoring of the selected rows (SEL_CANDIDATES, metric L2)
    int rescore_margin;  // extra rows selected before rescoring (0 = off)
    int dtype;
    const void* qdata;
    int64_t ldq;
    const void* xdata;
    int64_t ldx;
    int d;
    int x_i8;              // rows are SQ8 codes: value = fl(x_scale[row] * code)
    const float* x_scale;
};

// Largest k supported by the in-shared-memory final sort.
constexpr int kMaxK = 4096;

int launch_select(const SelectArgs& a, cudaStream_t stream);

}  // namespace rdb
