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
#define RDB_ERR_OVERFLOW 5    /* reserved: overflows are repaired on the device */
#define RDB_ERR_WORKSPACE 6   /* ws_bytes smaller than *_workspace() asked    */

/* ---- metrics: order of rapidadb::Metric, csrc/include/rapidadb/core/types.h:17-21 */
#define RDB_METRIC_COSINE 0
#define RDB_METRIC_L2 1
#define RDB_METRIC_DOT 2

/* ---- element types: rapidadb::Precision, types.h:9-14 (INT8: the SQ8 entry points below) */
#define RDB_F32 0
#define RDB_F16 1
#define RDB_BF16 2

/* ---- flat-search flags -------------------------------------------------- */
#define RDB_SEARCH_EXHAUSTIVE 1 /* no sampled threshold: every row is a candidate */
#define RDB_SEARCH_SYNC 2       /* wait for the call; RDB_ERR_TIMEOUT if a kernel gave up on a wait */

/* Message of the last failed call on this thread ("" if none). */
const char* rdb_last_error(void);
/* ABI version (major * 100 + minor). */
int rdb_version(void);
/* Reads (and with clear != 0 resets) the current device's status word, where
 * kernels record bounded waits that ran out (tensor-core scan: bit 0 producer,
 * 1 MMA issuer, 2 epilogue; bit 4 the TMA-fed CUDA-core scan; bit 5
 * rdb_probe_bounded_wait; bit 6 rdb_peer_gather).  Synchronises the device. */
int rdb_device_status(unsigned* out_host, int clear);
/* The status word as last forwarded by a completed rdb_flat_search on the
 * current device, read from mapped host memory without synchronising (0: no
 * kernel has reported a timeout).  Asynchronous error reporting in the manner
 * of CUDA's own: a search returns before its kernels finish, and a timeout
 * shows up here (and in rdb_device_status) once they have.  Cleared by
 * rdb_device_status(.., 1).  No reference counterpart (the reference checks
 * launch errors only, csrc/include/rapidadb/core/cuda_utils.h:12-30). */
int rdb_pending_status(unsigned* out_host);
/* Test hook of the bounded device waits (no reference counterpart): one
 * thread waits on an mbarrier that nothing arrives at, through the same wait
 * routine as the tensor-core scan's roles, for limit_ns (1 us .. 1 s); no TMA
 * load or MMA is in flight.  The wait runs out, sets bit 5 of the status
 * word, and the call (which synchronises `stream`) returns RDB_ERR_TIMEOUT. */
int rdb_probe_bounded_wait(unsigned long long limit_ns, void* stream);

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
 * Returns without waiting for the device.  A query whose candidate list
 * overflows its sampled-threshold capacity is rescanned exactly on the
 * device within the same call (the answer never depends on the threshold).
 * flags: RDB_SEARCH_EXHAUSTIVE (no sampled threshold; its own workspace
 * size), RDB_SEARCH_SYNC (wait; report a device-wait timeout). */
size_t rdb_flat_search_workspace(int metric, int dtype, int64_t nq, int64_t n, int d, int k,
                                 int flags);
/* The plan rdb_flat_search follows for these sizes (16-byte aligned layouts;
 * no reference counterpart, for tests and tuning): out[0] sampled rows (0: no
 * sample pass), out[1] rows per group maximum of the tensor-core sample pass,
 * out[2] row splits of the main pass, out[3] candidate capacity per (split,
 * query), out[4] rows per split, out[5] 1 when the tensor cores run the scan,
 * out[6] queries per chunk. */
int rdb_flat_search_plan(int metric, int dtype, int64_t nq, int64_t n, int d, int k, int flags, int64_t* out);
int rdb_flat_search(int metric, int dtype, const void* q, int64_t nq, int64_t ldq,
                    const void* x, int64_t n, int64_t ldx, const float* xv, int d, int k,
                    const int64_t* ids, int64_t id_offset, int flags, float* out_d,
                    int64_t* out_i, void* ws, size_t ws_bytes, void* stream);

/* INT8 storage: per-row symmetric scalar quantisation (SQ8).  The reference
 * names INT8 among its precisions (csrc/include/rapidadb/core/types.h:9-14,
 * python/rapidadb/config.py:21-26) without defining it; here a row x is
 * stored as scale = max_i |x_i| / 127 (fp32 division; 0 for a zero row) and
 * codes c_i = rint(x_i / scale) clamped to [-127, 127] (ties to even), and
 * stands for the dequantised row x^_i = fl(scale * c_i).
 *   rdb_sq8_encode        x [n, d] (dtype, stride ldx) -> codes [n, ldc] int8
 *                         (columns d .. ldc - 1 zero), scales [n]
 *   rdb_sq8_row_values    per-row metric values of x^ (as rdb_vec_values)
 *   rdb_flat_search_sq8   rdb_flat_search over SQ8 rows with fp32 queries: the
 *                         exact search over x^ (reference formulas, L2 summed
 *                         directly for the returned rows), CUDA cores, one
 *                         byte per stored element; ldx (bytes) a multiple of 4 */
int rdb_sq8_encode(int dtype, const void* x, int64_t n, int64_t ldx, int d, int8_t* codes, int64_t ldc, float* scales,
                   void* stream);
int rdb_sq8_row_values(int metric, const int8_t* codes, const float* scales, int64_t n, int64_t ldc, int d,
                       float* out, void* stream);
size_t rdb_flat_search_sq8_workspace(int metric, int64_t nq, int64_t n, int d, int k, int flags);
int rdb_flat_search_sq8(int metric, const float* q, int64_t nq, int64_t ldq, const int8_t* codes, const float* scales,
                        int64_t n, int64_t ldx, const float* xv, int d, int k, const int64_t* ids, int64_t id_offset,
                        int flags, float* out_d, int64_t* out_i, void* ws, size_t ws_bytes, void* stream);

/* Row-sharded flat search with one threshold for all shards (no reference
 * counterpart: the reference is single-GPU).  Each shard computes the group
 * maxima of a strided sample of its rows, the maxima of every shard are
 * gathered (one all-gather), the k-th best of them is a lower bound on the
 * global k-th best score (k distinct rows reach it), and each shard keeps
 * only rows reaching it:
 *   rdb_flat_sample_maxima  out [nq, sample_rows / group]: best final score
 *                           of each group of `group` (power of two <= 128)
 *                           consecutive sampled rows; the sample is rows
 *                           0, s, 2 s, ... (s = n / sample_rows) of x.
 *                           fp16 / bf16 rows on the tensor cores only
 *                           (RDB_ERR_UNSUPPORTED otherwise); the scores are
 *                           exact up to a few ulps.  ws: rdb_flat_sample_workspace.
 *   rdb_select_threshold    out_thr[q] = k-th best of scores[q, 0..G) (L2
 *                           smallest, cosine / dot largest; +-inf if G < k).
 *   rdb_flat_search_thr     rdb_flat_search with caller thresholds thr [nq]
 *                           (final-score units; must not be better than the
 *                           true k-th best) and `expect` candidates per query
 *                           expected over the n rows (sizes the candidate
 *                           lists); overflowed queries are repaired as in
 *                           rdb_flat_search. */
size_t rdb_flat_sample_workspace(int64_t nq);
int rdb_flat_sample_maxima(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, const void* x, int64_t n,
                           int64_t ldx, const float* xv, int d, int64_t sample_rows, int group, float* out, void* ws,
                           size_t ws_bytes, void* stream);
int rdb_select_threshold(int largest, const float* scores, int64_t nq, int64_t G, int k, float* out_thr,
                         void* stream);
size_t rdb_flat_search_thr_workspace(int metric, int dtype, int64_t nq, int64_t n, int d, int k, int64_t expect);
int rdb_flat_search_thr(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, const void* x, int64_t n,
                        int64_t ldx, const float* xv, int d, int k, const int64_t* ids, int64_t id_offset,
                        const float* thr, int64_t expect, float* out_d, int64_t* out_i, void* ws, size_t ws_bytes,
                        void* stream);

/* Merge G per-shard sorted lists [G, nq, kin] (scores + int64 ids) into the
 * best k per query, ties to the lower id: the final step after the NCCL
 * all-gather of row-sharded search (the reference is single-GPU). */
int rdb_topk_merge(int largest, const float* in_v, const int64_t* in_i, int G, int64_t nq,
                   int kin, int k, float* out_v, int64_t* out_i, void* stream);
/* Same with list g at in_v + g * gstride_v and in_i + g * gstride_i (0: nq *
 * kin), e.g. the per-rank blocks of an all-gather buffer, read in place. */
int rdb_topk_merge_strided(int largest, const float* in_v, int64_t gstride_v, const int64_t* in_i,
                           int64_t gstride_i, int G, int64_t nq, int kin, int k, float* out_v, int64_t* out_i,
                           void* stream);
/* Same with row strides: element (g, q, t) of the scores at in_v[g *
 * gstride_v + q * ldv + t], of the ids at in_i[g * gstride_i + q * ldi + t]
 * (ldv / ldi 0: kin), e.g. scores and ids interleaved by row in one packed
 * exchange buffer. */
int rdb_topk_merge_ld(int largest, const float* in_v, int64_t gstride_v, int64_t ldv, const int64_t* in_i,
                      int64_t gstride_i, int64_t ldi, int G, int64_t nq, int kin, int k, float* out_v, int64_t* out_i,
                      void* stream);

/* ---- peer exchange over NVLink (no reference counterpart: the reference is
 * single-GPU, README.md:14) --------------------------------------------- */

#define RDB_PEER_MAX_RANKS 8
#define RDB_PEER_SLOTS 8
#define RDB_PEER_FLAG_BYTES 512 /* the flags at the start of every arena */
#define RDB_PEER_HANDLE_BYTES 64

/* One exchange arena per rank: `bytes` of device memory on the current
 * device, zeroed, and its 64-byte CUDA IPC handle for the other processes of
 * the node.  Bytes [0, RDB_PEER_FLAG_BYTES) hold the exchange flags (64 bytes
 * per slot, word p written by rank p); the data sections follow. */
int rdb_peer_arena_alloc(size_t bytes, void** ptr, unsigned char* handle);
int rdb_peer_arena_free(void* ptr);
/* Maps another process's arena into this one (peer access enabled). */
int rdb_peer_arena_open(const unsigned char* handle, void** ptr);
int rdb_peer_arena_close(void* ptr);

/* One exchange step.  Rank p's source rows are rows row0[p] ..
 * row0[p] + nrows[p] - 1 of the array at byte src_off of rank p's arena
 * (rows src_row_stride bytes apart, row_bytes bytes each); they land at
 * dst + dst_off[p] + i * dst_row_stride in this rank's memory. */
typedef struct RdbPeerGather {
    int world, rank;          /* ranks of the exchange (<= RDB_PEER_MAX_RANKS), this rank */
    int slot, pad;            /* flag slot, < RDB_PEER_SLOTS */
    unsigned long long epoch; /* above every earlier epoch of the slot; the same on every rank */
    void* base[RDB_PEER_MAX_RANKS]; /* every rank's arena as mapped here (own included) */
    long long arena_bytes;          /* size of every arena: every source row lies inside it */
    long long src_off, src_row_stride, row_bytes;
    long long row0[RDB_PEER_MAX_RANKS], nrows[RDB_PEER_MAX_RANKS];
    void* dst;
    long long dst_off[RDB_PEER_MAX_RANKS], dst_row_stride;
} RdbPeerGather;

/* Launches one kernel on `stream` that (1) signals slot `slot` at `epoch` in
 * every rank's arena: this rank's source rows, written by earlier work on
 * the stream, are ready; (2) waits until every rank has signalled the slot
 * at `epoch` or later, for at most limit_ns (1 us .. 10 s); (3) copies the
 * rows with peer loads.  A wait that runs out sets bit 6 (64) of the device
 * status word (rdb_device_status, rdb_pending_status) and copies nothing.
 * Multicast is not used.  All sizes, offsets and strides are multiples of 4
 * bytes; 16-byte alignment throughout selects 16-byte copies. */
int rdb_peer_gather(const RdbPeerGather* args, unsigned long long limit_ns, void* stream);

/* ---- k-means --------------------------------------------------------- */

/* Lloyd assign step: label[i] = argmin_c |x_i - c|^2 (ties to the lower
 * centroid) and its squared distance.  Replaces assign_clusters_kernel
 * (csrc/kernels/kmeans.cu:11-45; the reference writes sqrt of the minimum and
 * has no launcher).  fp16 / bf16 points and centroids run as a tcgen05 GEMM
 * with the argmin fused into the epilogue (|c|^2 - 2 x.c), fp32 on CUDA cores.
 * x [n, d] (stride ldx), centroids [K, d] (stride ldc, same dtype),
 * c_sqnorms [K] = |c|^2 of the centroids as stored. */
size_t rdb_kmeans_assign_workspace(int dtype, int64_t n, int K, int d);
int rdb_kmeans_assign(int dtype, const void* x, int64_t n, int64_t ldx, int d, const void* centroids, int K,
                      int64_t ldc, const float* c_sqnorms, int32_t* labels, float* sqdist, void* ws,
                      size_t ws_bytes, void* stream);

/* Lloyd update step, atomic-free: per-centroid sums [K, d] (fp32) and counts
 * [K] of the points with each label, summed in ascending point order.
 * Replaces update_centroids_kernel (csrc/kernels/kmeans.cu:48-94, float
 * atomics).  Multi-GPU callers all-reduce sums and counts, then finalize. */
size_t rdb_kmeans_update_workspace(int64_t n, int K);
int rdb_kmeans_update(int dtype, const void* x, int64_t n, int64_t ldx, int d, const int32_t* labels, int K,
                      float* sums, int64_t* counts, void* ws, size_t ws_bytes, void* stream);

/* centroid = sums / count; a centroid with count 0 keeps its value (the
 * reference leaves it unwritten, csrc/kernels/kmeans.cu:88-93). */
int rdb_kmeans_finalize(const float* sums, const int64_t* counts, int K, int d, float* centroids, void* stream);

/* Exact list assignment for IVF indices: argmin over centroids of the
 * sequential sum of (x - c)^2 with one fused multiply-add per element, the
 * reference assign arithmetic (csrc/kernels/kmeans.cu:31-35) bit for bit;
 * fp32 only. */
size_t rdb_assign_exact_workspace(int64_t n, int K, int d);
int rdb_assign_exact(const float* x, int64_t n, int64_t ldx, int d, const float* centroids, int K, int64_t ldc,
                     int32_t* labels, float* sqdist, void* ws, size_t ws_bytes, void* stream);

/* Stable counting sort by label (no reference counterpart; the building block
 * of the atomic-free k-means update and of the IVF list layouts):
 * perm[seg_start[c] .. seg_start[c + 1]) = the ids i with labels[i] == c in
 * ascending order, counts[c] the segment sizes (counts may be NULL).
 * Labels must lie in [0, K), K <= 16384. */
size_t rdb_label_sort_workspace(int64_t n, int K);
int rdb_label_sort(const int32_t* labels, int64_t n, int K, int64_t* seg_start, int64_t* perm, int64_t* counts,
                   void* ws, size_t ws_bytes, void* stream);

/* ---- IVF-Flat / IVF-PQ (no reference implementation: the reference only
 * names them, python/rapidadb/config.py:14-18, :50-56; index.py:64-69) ---- */

/* List-major scan of an IVF index whose rows are stored list by list:
 * list l is rows list_off[l] .. list_end[l] - 1, inside its capacity
 * list_off[l] .. list_off[l + 1] - 1 (list_end NULL: the whole capacity, no
 * free slots; free slots let rows be appended without moving the others, see
 * rdb_pq_scatter_codes).  probe [nq, nprobe]
 * holds each query's lists (from a coarse rdb_flat_search over the
 * centroids).  For every (query, probe slot) the best k rows of that list,
 * scored with the flat formula of `metric` (L2 summed directly), go to
 * out_v / out_i [nprobe, nq, k] (ids[row], or -1 padding when a list has
 * fewer than k rows); rdb_topk_merge then keeps the best k per query.
 * q and rows share `dtype`; xv [n] per-row values (rdb_row_sqnorms then
 * rdb_vec_values: required for cosine; for L2 with k <= 24, |x|^2 lets the
 * scan rank by |q|^2 + |x|^2 - 2 q.x and rescore k + 8 rows per list
 * directly; NULL keeps the direct L2 scan); k <= 32. */
size_t rdb_ivf_scan_workspace(int64_t nq, int nprobe, int nlist);
int rdb_ivf_flat_scan(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d, const int64_t* probe,
                      int nprobe, const void* rows, int64_t ldx, const float* xv, const int64_t* list_off,
                      const int64_t* list_end, int nlist, const int64_t* ids, int k, float* out_v, int64_t* out_i,
                      void* ws, size_t ws_bytes, void* stream);

/* rdb_ivf_flat_scan over SQ8 rows (codes [.., ldx] int8 with per-row scales,
 * see rdb_sq8_encode) and fp32 queries: the exact scan of the dequantised
 * rows; ldx (bytes) a multiple of 4. */
int rdb_ivf_flat_scan_sq8(int metric, const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe,
                          int nprobe, const int8_t* codes, int64_t ldx, const float* scales, const float* xv,
                          const int64_t* list_off, const int64_t* list_end, int nlist, const int64_t* ids, int k,
                          float* out_v, int64_t* out_i, void* ws, size_t ws_bytes, void* stream);

/* fp32 rows as two fp16 planes for the tensor-core IVF search: per row a
 * power-of-two scale 2^e (largest |x_t| 2^-e in [2^13, 2^14); 1 for a zero
 * row), hi = fp16(x 2^-e), lo = fp16(x 2^-e - hi); hi / lo [n, ldp] fp16,
 * columns d .. ldp - 1 zero; scale [n].  *flag (may be NULL) gets bit 0 when a
 * value is not finite (such rows must be searched with rdb_ivf_flat_scan).
 * ldp a multiple of 8. */
int rdb_f16_split(const float* x, int64_t n, int64_t ldx, int d, void* hi, void* lo, int64_t ldp, float* scale,
                  unsigned* flag, void* stream);

/* IVF-Flat search of fp32 rows on the tensor cores (no counterpart in the
 * reference, whose IVF search ranks with CUDA-core distances): the list scan
 * of rdb_ivf_flat_scan as a tcgen05 contraction of each list's probing
 * queries with its rows (the rows' rdb_f16_split planes, three fp16 products
 * per element into fp32), ranking the best k + 8 rows per (query, probe
 * slot); per query the best k + 8 of those are scored again with
 * rdb_ivf_flat_scan's arithmetic on the fp32 rows, so scores equal the
 * CUDA-core scan's.  Output out_v / out_i [nq, k]: the merged answer (best
 * first, ties to the lower stored row, ids[row] or -1 padding), no
 * rdb_topk_merge step.  rows / xv / list_off / list_end / ids as
 * rdb_ivf_flat_scan (xv required for L2 and cosine: |x|^2, resp. the norm);
 * rows_hi / rows_lo [nrows, ldp] and row_scale [nrows] from rdb_f16_split of
 * the same rows, ldp = d rounded up to a multiple of 64, 16-byte aligned.
 * Supported for d <= 128 and k <= 24 (rdb_ivf_flat_search_tc_supported). */
/* The same search over fp16 / bf16 rows (dtype RDB_F16 / RDB_BF16) and
 * queries of the same type, as rdb_ivf_flat_scan takes them: the MMA reads
 * the stored rows directly (stride ldx elements, a multiple of 8; one exact
 * fp16 / bf16 product per element into fp32), no planes; the best k + 8
 * rows per query are rescored with rdb_ivf_flat_scan's arithmetic, so scores
 * equal its scores.  Workspace rdb_ivf_flat_search_tc_workspace. */
int rdb_ivf_flat_search_tc_half(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d,
                                const int64_t* probe, int nprobe, const void* rows, int64_t ldx, const float* xv,
                                int64_t nrows, const int64_t* list_off, const int64_t* list_end, int nlist,
                                const int64_t* ids, int k, float* out_v, int64_t* out_i, void* ws, size_t ws_bytes,
                                void* stream);
int rdb_ivf_flat_search_tc_supported(int d, int k);
/* Counts on the current device since the last reset (host out[2]): out[0]
 * (query, probe slot) entries whose collected rows overflowed the per-entry
 * buffer so that their list was rescanned exactly; out[1] queries of
 * rdb_ivf_probe_tc whose collected centroids overflowed so that every
 * centroid was scored exactly.  Both keep results correct and cost time;
 * expected only for many rows (centroids) of equal value.  Synchronises the
 * device. */
int rdb_ivf_tc_overflows(unsigned long long* out_host, int reset);
size_t rdb_ivf_flat_search_tc_workspace(int64_t nq, int nprobe, int nlist, int d, int k, int64_t nrows);
int rdb_ivf_flat_search_tc(int metric, const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe,
                           int nprobe, const float* rows, int64_t ldx, const float* xv, const void* rows_hi,
                           const void* rows_lo, const float* row_scale, int64_t ldp, int64_t nrows,
                           const int64_t* list_off, const int64_t* list_end, int nlist, const int64_t* ids, int k,
                           float* out_v, int64_t* out_i, void* ws, size_t ws_bytes, void* stream);

/* Coarse probe on the tensor cores (replaces the CUDA-core flat search over
 * the centroids; no reference counterpart): the nprobe nearest centroids of
 * each query by squared L2, ascending, ties to the lower list -- probe
 * [nq, nprobe].  Every (query, centroid) value |c|^2 - 2 q.c comes from the
 * three-product fp16 split contraction (centroid planes from rdb_f16_split,
 * stride ldp = d rounded up to 64), the best nprobe + 8 of each query are
 * scored again as sum (q - c)^2 with rdb_flat_search's exact L2 arithmetic,
 * so the lists equal those of a flat L2 search over the centroids.  cent
 * [nlist, ldc] fp32 centroids, cent_sq [nlist] their |c|^2.  Supported for
 * d <= 128 and min(nlist, nprobe + 8) <= 128 (rdb_ivf_probe_tc_supported). */
int rdb_ivf_probe_tc_supported(int d, int nlist, int nprobe);
size_t rdb_ivf_probe_tc_workspace(int64_t nq, int nlist, int d, int nprobe);
int rdb_ivf_probe_tc(const float* q, int64_t nq, int64_t ldq, int d, const float* cent, int64_t ldc,
                     const float* cent_sq, const void* cent_hi, const void* cent_lo, const float* cent_scale,
                     int64_t ldp, int nlist, int nprobe, int64_t* probe, void* ws, size_t ws_bytes, void* stream);

/* rdb_ivf_flat_scan for callers that may not allocate GPU memory (no
 * counterpart in the reference): the same list-major scan and the same
 * results, with its scratch taken from an 8 MiB array compiled into the
 * library (rdb_noalloc_scratch_bytes) instead of a caller workspace, for
 * hosts that pool all device memory themselves, serving threads that must
 * not block in an allocator, or plug-ins whose host runtime forbids guest
 * allocations.  Returns RDB_ERR_UNSUPPORTED when rdb_ivf_scan_workspace(nq,
 * nprobe, nlist) exceeds the array.  Set-up: call rdb_noalloc_init() once per
 * device (and per context the host makes current), with that device
 * current, before the first scan and before any stream capture; it loads the
 * library's device module, which is when the 8 MiB is allocated (CUDA loads
 * modules lazily by default).  After it, a scan allocates nothing; without
 * it the first scan in a context does the lookup and allocates.  The array
 * stays allocated until the context ends; all calls on a device share it, so
 * calls that overlap on the GPU race -- serialise them. */
size_t rdb_noalloc_scratch_bytes(void);
int rdb_noalloc_init(void);
int rdb_ivf_flat_scan_noalloc(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, int d,
                              const int64_t* probe, int nprobe, const void* rows, int64_t ldx, const float* xv,
                              const int64_t* list_off, const int64_t* list_end, int nlist, const int64_t* ids, int k,
                              float* out_v, int64_t* out_i, void* stream);

/* Residual product-quantisation codes: for row i in list labels[i], residual
 * r = x_i - centroid; code m = argmin over the ksub codewords of subspace m
 * (codebooks [M, ksub, d / M]) of the sequential fused-FMA squared distance,
 * ties to the lower codeword.  codes [n, M] uint8.  fp32 inputs. */
int rdb_pq_encode(const float* x, int64_t n, int64_t ldx, int d, const int32_t* labels, const float* centroids,
                  const float* codebooks, int M, int ksub, uint8_t* codes, void* stream);

/* List-major IVF-PQ asymmetric-distance scan (squared L2): per (query,
 * probed list) a table LUT[m][j] = |(q - centroid)_m - codeword_mj|^2 is built
 * in shared memory and each stored code scores sum_m LUT[m][code_m]; output
 * layout as rdb_ivf_flat_scan.  Codes stored list by list in the slot ranges
 * of rdb_ivf_flat_scan (list_off / list_end); k <= 32. */
int rdb_ivfpq_scan(const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe, int nprobe,
                   const float* centroids, int nlist, const float* codebooks, int M, int ksub, const uint8_t* codes,
                   const int64_t* list_off, const int64_t* list_end, const int64_t* ids, int k, float* out_v,
                   int64_t* out_i, void* ws, size_t ws_bytes, void* stream);

/* Query-major IVF-PQ search (squared L2; replaces rdb_ivfpq_scan + the merge
 * when rdb_pq_fast_layout(M) is 1, i.e. M in {4, 8, 16, 32, 64, 96}).
 * The residual ADC distance is regrouped as
 *   |q - c_l|^2 + row_terms[row] + sum_m QT[m][code_m],  QT[m][j] = -2 <q_m, cb[m][j]>,
 * so one lookup table per query serves all of its probed lists.
 *   rdb_pq_row_terms     row_terms[i] = sum_m |cb[m][c_m]|^2 + 2 <(c_{labels[i]})_m, cb[m][c_m]>
 *                        for unrotated codes [n, M] (once per added row);
 *   rdb_pq_rotate_codes  in place: within each group of G = min(M, 32) code
 *                        bytes, row i (list order) is rotated by i mod G
 *                        (stored byte s = code[(i + s) mod G]); inverse != 0
 *                        undoes it.  rdb_ivfpq_search reads rotated codes;
 *   rdb_ivfpq_search     probe [nq, nprobe] list ids; codes / row_terms /
 *                        ids in list order (slot ranges list_off [nlist + 1]
 *                        / list_end [nlist] as rdb_ivf_flat_scan); writes the
 *                        best k (k <= 32) per query, ascending, ties to the
 *                        lower stored row, to out_v / out_i [nq, k] (ids[row],
 *                        or -1 padding).  nprobe <= 4096, nlist <= 16384,
 *                        fewer than 2^32 stored rows.
 * No reference counterpart (the reference declares IVF-PQ parameters only,
 * python/rapidadb/config.py:50-56). */
int rdb_pq_fast_layout(int M);
int rdb_pq_row_terms(const uint8_t* codes, int64_t n, int M, const int32_t* labels, const float* centroids, int d,
                     const float* codebooks, int ksub, float* out_terms, void* stream);
int rdb_pq_rotate_codes(uint8_t* codes, int64_t n, int M, int inverse, void* stream);
/* Appends into free list slots (no reference counterpart): dst row dest[i] =
 * src row i for i < n (rows of M code bytes, dest distinct), stored as
 * rdb_pq_rotate_codes lays out row dest[i] when `rotated` != 0 (M as
 * rdb_pq_fast_layout).  src holds unrotated codes. */
int rdb_pq_scatter_codes(const uint8_t* src, int64_t n, int M, const int64_t* dest, uint8_t* dst, int rotated,
                         void* stream);
size_t rdb_ivfpq_search_workspace(int64_t nq, int nlist);
int rdb_ivfpq_search(const float* q, int64_t nq, int64_t ldq, int d, const int64_t* probe, int nprobe,
                     const float* centroids, int nlist, const float* codebooks, int M, int ksub, const uint8_t* codes,
                     const float* row_terms, const int64_t* list_off, const int64_t* list_end, const int64_t* ids,
                     int k, float* out_v, int64_t* out_i, void* ws, size_t ws_bytes, void* stream);

/* Profiling hook (no reference counterpart; the reference times whole calls,
 * benchmarks/src/bench_compare.py:56-59): `mask` selects launches to time
 * with CUDA events recorded on their launching stream -- 1 the main scan of
 * rdb_flat_search, 2 the rdb_ivf_flat_scan list scan, 4 the rdb_ivfpq_scan
 * list scan or the rdb_ivfpq_search kernel, 8 the rdb_kmeans_assign scan, 16
 * the rdb_kmeans_update segment sums, and the phases of rdb_flat_search: 32
 * per-query values, 64 sample pass + threshold select, 128 candidate
 * select, 256 overflow repair (0 turns timing off).  rdb_timing_read
 * synchronises the recorded events and returns the summed device time and
 * the number of timed launches; rdb_timing_read_tags does the same for the
 * launches whose tag is in `mask`, without resetting. */
int rdb_timing_enable(int mask);
int rdb_timing_read(double* total_ms, int* launches, int reset);
int rdb_timing_read_tags(int mask, double* total_ms, int* launches);

/* Kernels this library has launched so far in the process, all devices and
 * threads (no reference counterpart): read it before and after a region. */
unsigned long long rdb_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* RAPIDADB_B200_H */
