/*
 * rapidadb_b200.h -- C ABI of the B200 (sm_100a) kernels behind RapidaDB's
 * search path.
 *
 * Plain C: pointers, sizes and integer codes only.  Every function
 *   - takes DEVICE pointers (all on the current CUDA device) unless a
 *     parameter says "host",
 *   - enqueues its work on `stream` (a cudaStream_t passed as void*; NULL is
 *     the legacy default stream) and returns without synchronising unless its
 *     comment says otherwise,
 *   - returns RDB_OK (0) or an RDB_ERR_* code; rdb_last_error() then holds a
 *     message for the calling thread.  No C++ exception crosses this ABI.
 *
 * Scratch memory is the caller's: functions that need it take (ws, ws_bytes)
 * and have a *_workspace() companion returning the bytes required.
 *
 * Each declaration names the reference interface it replaces
 * (VARUN3WARE/RAPIDADB, path:line).
 */
#ifndef RAPIDADB_B200_H
#define RAPIDADB_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define RDB_OK 0
#define RDB_ERR_INVALID 1     /* bad argument (message says which)            */
#define RDB_ERR_CUDA 2        /* CUDA runtime / launch error                  */
#define RDB_ERR_TIMEOUT 3     /* a kernel gave up on a bounded device wait    */
#define RDB_ERR_UNSUPPORTED 4 /* valid request outside the supported range    */
#define RDB_ERR_OVERFLOW 5    /* candidate buffer overflowed; retry exhaustive */
#define RDB_ERR_WORKSPACE 6   /* ws_bytes smaller than *_workspace() asked    */

/* ---- metrics: order of rapidadb::Metric, csrc/include/rapidadb/core/types.h:17-21 */
#define RDB_METRIC_COSINE 0
#define RDB_METRIC_L2 1
#define RDB_METRIC_DOT 2

/* ---- element types: rapidadb::Precision, types.h:9-14 (INT8 not stored) */
#define RDB_F32 0
#define RDB_F16 1
#define RDB_BF16 2

/* ---- flat-search flags -------------------------------------------------- */
#define RDB_SEARCH_EXHAUSTIVE 1 /* no sampled threshold: every row is a candidate */

/* Message of the last failed call on this thread ("" if none). */
const char* rdb_last_error(void);
/* ABI version (major * 100 + minor). */
int rdb_version(void);
/* Reads (and with clear != 0 resets) the current device's status word, where
 * kernels record bounded waits that ran out (bit 0 producer, 1 MMA issuer,
 * 2 epilogue).  Synchronises the device. */
int rdb_device_status(unsigned* out_host, int clear);

/* Dense [nq, nx] score matrix with the reference formulas.
 * Replaces cosine_similarity_cuda / l2_distance_cuda / dot_product_cuda,
 * csrc/kernels/distance.cu:471-610 (bound as _C.cosine_similarity /
 * l2_distance / dot_product, csrc/bindings/torch_extension.cpp:34-44).
 * q [nq, d] and x [nx, d] row-major in `dtype`; out [nq, nx] fp32.
 * L2 is summed directly as sum (q - x)^2; cosine uses the d <= 128 or d > 128
 * epsilon placement of the reference (distance.cu:175 vs :332, :367). */
int rdb_distance(int metric, int dtype, const void* q, int64_t nq, const void* x, int64_t nx,
                 int d, float* out, void* stream);

/* Squared L2 norm of each row of x [n, d] (fp32 accumulation). */
int rdb_row_sqnorms(int dtype, const void* x, int64_t n, int d, float* out, void* stream);

/* Per-row metric value from squared norms: |x|^2 (L2), sqrt|x|^2 or
 * sqrt(|x|^2 + 1e-8) (cosine, d > 128 / d <= 128), 0 (dot).  out may alias sq. */
int rdb_vec_values(int metric, int d, const float* sq, int64_t n, float* out, void* stream);

/* Sorted top-k of each row of a dense [B, N] fp32 matrix, ties to the lower
 * column.  Replaces topk_thrust (csrc/kernels/topk.cu:14-28) and the two
 * entry points routed to it, topk_warp_heap / topk_auto
 * (csrc/kernels/topk_warp.cu:80-110). */
size_t rdb_topk_workspace(int64_t B, int64_t N, int k);
int rdb_topk(const float* dist, int64_t B, int64_t N, int k, int largest, float* out_v,
             int64_t* out_i, void* ws, size_t ws_bytes, void* stream);

/* Exact flat search: scores of nq queries against n stored rows, sorted
 * top-k, local row -> user id.  Replaces FlatIndex::search
 * (csrc/index/flat_index.cpp:49-86: distance kernel -> topk_thrust ->
 * ids_.index_select) with one fused scan that never writes the [nq, n]
 * matrix.
 *   x [n, d] rows in `dtype` (row stride ldx elements, ldx * elem_size a
 *   multiple of 16 bytes), xv [n] per-row values (rdb_vec_values),
 *   q [nq, d] queries in the same dtype (stride ldq, same alignment rule),
 *   ids [n] user ids or NULL for (row + id_offset).
 *   out_d [nq, k] scores (L2 ascending, cosine / dot descending), out_i ids.
 * fp16 / bf16 run on the tcgen05 tensor cores; fp32 on CUDA cores.
 * Synchronises `stream` once to read its overflow flag; returns
 * RDB_ERR_OVERFLOW if a query's candidates overflowed, in which case the
 * caller repeats the call with flags = RDB_SEARCH_EXHAUSTIVE (whose
 * workspace is sized by the same flag). */
size_t rdb_flat_search_workspace(int metric, int dtype, int64_t nq, int64_t n, int d, int k,
                                 int flags);
int rdb_flat_search(int metric, int dtype, const void* q, int64_t nq, int64_t ldq,
                    const void* x, int64_t n, int64_t ldx, const float* xv, int d, int k,
                    const int64_t* ids, int64_t id_offset, int flags, float* out_d,
                    int64_t* out_i, void* ws, size_t ws_bytes, void* stream);

/* Merge G per-shard sorted lists [G, nq, kin] (scores + int64 ids) into the
 * best k per query, ties to the lower id: the final step after the NCCL
 * all-gather of row-sharded search (the reference is single-GPU). */
int rdb_topk_merge(int largest, const float* in_v, const int64_t* in_i, int G, int64_t nq,
                   int kin, int k, float* out_v, int64_t* out_i, void* stream);

/* Profiling hook (no reference counterpart; the reference times whole calls,
 * benchmarks/src/bench_compare.py:56-59): when enabled, CUDA events are
 * recorded on the launching stream around every main-pass scan launch of
 * rdb_flat_search; rdb_timing_read synchronises them and returns the summed
 * device time and the number of timed launches. */
int rdb_timing_enable(int enable);
int rdb_timing_read(double* total_ms, int* launches, int reset);

#ifdef __cplusplus
}
#endif
#endif /* RAPIDADB_B200_H */
