/*
 * CPU oracle for the RapidaDB search hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  The parity tests compare against this file: it
 * is loaded by the tests, by __graft_entry__.smoke() and by bench.py's
 * CPU-baseline leg, never by the product path (rapidadb_b200/), which fails
 * loudly when its CUDA library is missing instead of falling back to anything
 * here.
 *
 * Every function restates the reference's algorithm in plain C (+ OpenMP) and
 * cites the reference file:line it follows (paths are relative to the
 * VARUN3WARE/RAPIDADB source tree).  Where the reference has no
 * implementation (IVF-Flat, IVF-PQ, the k-means driver), the oracle *defines*
 * the semantics and says so: parity for those parts is pinned only by the
 * oracle itself, not by reference outputs.
 *
 * Numerics:
 *   - Flat distances accumulate in double ("exact" mode, acc64 = 1) or in
 *     fp32 with eight interleaved accumulators (acc64 = 0, the timed CPU
 *     baseline, close to the reference's multi-accumulator fp32 kernels).
 *   - k-means / IVF assignment and PQ encoding use the reference's assign
 *     arithmetic bit for bit: diff = p - c; dist = fmaf(diff, diff, dist),
 *     summed sequentially over the dimension (csrc/kernels/kmeans.cu:31-35,
 *     built with -fmad=true so `dist += diff * diff` is one fused FMA).  The
 *     GPU product uses the same arithmetic for list assignment and PQ codes,
 *     which is why codes can be compared for equality.
 *   - This file is compiled with -ffp-contract=off so the compiler never
 *     fuses anything that is not written as fmaf().
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_COSINE 0
#define ORC_L2 1
#define ORC_DOT 2

/* Reference kernel dispatch threshold: dim <= TILE_DIM (128) uses the
 * shared-memory "optimized" kernels, larger dims the register-tiled ones
 * (csrc/kernels/distance.cu:16, :493-511, :540-559, :591-606). */
#define ORC_TILE_DIM 128

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------ */
/* dot products / squared norms                                        */
/* ------------------------------------------------------------------ */

static double dot64(const float* a, const float* b, int d) {
    double s = 0.0;
    for (int i = 0; i < d; ++i) s += (double)a[i] * (double)b[i];
    return s;
}

static double l2sq64(const float* a, const float* b, int d) {
    double s = 0.0;
    for (int i = 0; i < d; ++i) {
        double t = (double)a[i] - (double)b[i];
        s += t * t;
    }
    return s;
}

/* fp32, eight interleaved accumulators (vectorisable without fast-math). */
static float dot32(const float* a, const float* b, int d) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= d; i += 8)
        for (int j = 0; j < 8; ++j) acc[j] += a[i + j] * b[i + j];
    float s = 0.f;
    for (int j = 0; j < 8; ++j) s += acc[j];
    for (; i < d; ++i) s += a[i] * b[i];
    return s;
}

static float l2sq32(const float* a, const float* b, int d) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= d; i += 8)
        for (int j = 0; j < 8; ++j) {
            float t = a[i + j] - b[i + j];
            acc[j] += t * t;
        }
    float s = 0.f;
    for (int j = 0; j < 8; ++j) s += acc[j];
    for (; i < d; ++i) {
        float t = a[i] - b[i];
        s += t * t;
    }
    return s;
}

/* Sequential fused-FMA squared distance, the reference assign arithmetic
 * (csrc/kernels/kmeans.cu:31-35). */
static float l2sq_fma_seq(const float* a, const float* b, int d) {
    float s = 0.f;
    for (int i = 0; i < d; ++i) {
        float t = a[i] - b[i];
        s = fmaf(t, t, s);
    }
    return s;
}

/* Final score of one (query, row) pair, following the reference formulas:
 *   L2      : sum (q_i - x_i)^2                        distance.cu:414-438
 *   DOT     : sum q_i x_i                              distance.cu:443-466
 *   COSINE  : d >  128: dot / (sqrt(|q|^2) sqrt(|x|^2) + 1e-8)   distance.cu:175
 *             d <= 128: dot / (sqrt(|q|^2 + 1e-8) sqrt(|x|^2 + 1e-8))
 *                                                       distance.cu:332, :367
 * qsq / xsq are the squared norms (only used by COSINE). */
static float score_pair(int metric, const float* q, const float* x, int d,
                        double qsq, double xsq, int acc64) {
    if (metric == ORC_L2) return acc64 ? (float)l2sq64(q, x, d) : l2sq32(q, x, d);
    if (acc64) {
        double dot = dot64(q, x, d);
        if (metric == ORC_DOT) return (float)dot;
        if (d > ORC_TILE_DIM) return (float)(dot / (sqrt(qsq) * sqrt(xsq) + 1e-8));
        return (float)(dot / (sqrt(qsq + 1e-8) * sqrt(xsq + 1e-8)));
    } else {
        float dot = dot32(q, x, d);
        if (metric == ORC_DOT) return dot;
        if (d > ORC_TILE_DIM) return dot / (sqrtf((float)qsq) * sqrtf((float)xsq) + 1e-8f);
        return dot / (sqrtf((float)qsq + 1e-8f) * sqrtf((float)xsq + 1e-8f));
    }
}

static void row_sqnorms(const float* x, int64_t n, int d, double* out, int acc64) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i)
        out[i] = acc64 ? dot64(x + i * d, x + i * d, d) : (double)dot32(x + i * d, x + i * d, d);
}

/* Dense distance matrix, the reference raw ops
 * (_C.cosine_similarity / l2_distance / dot_product,
 *  csrc/bindings/torch_extension.cpp:34-44 -> distance.cu:471-610).
 * Note: the reference's register-tiled kernels (d > 128) drop the d % 4 tail
 * (distance.cu:45, :99, :147); the oracle sums every element. */
void orc_distance(int metric, const float* q, int64_t Q, const float* x, int64_t N,
                  int d, float* out, int acc64, int nthreads) {
    set_threads(nthreads);
    double* qsq = (double*)malloc(sizeof(double) * (Q > 0 ? Q : 1));
    double* xsq = (double*)malloc(sizeof(double) * (N > 0 ? N : 1));
    row_sqnorms(q, Q, d, qsq, acc64);
    row_sqnorms(x, N, d, xsq, acc64);
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t i = 0; i < Q; ++i)
        for (int64_t j = 0; j < N; ++j)
            out[i * N + j] = score_pair(metric, q + i * d, x + j * d, d, qsq[i], xsq[j], acc64);
    free(qsq);
    free(xsq);
}

/* ------------------------------------------------------------------ */
/* top-k                                                               */
/* ------------------------------------------------------------------ */

/* "a ranks before b": the order torch::topk(sorted=true) produces
 * (csrc/kernels/topk.cu:25), with ties broken by the lower index (torch
 * leaves the tie order unspecified; the oracle fixes it). */
static inline int better(float va, int64_t ia, float vb, int64_t ib, int largest) {
    if (va != vb) return largest ? (va > vb) : (va < vb);
    return ia < ib;
}

/* Bounded heap whose root is the worst kept element. */
typedef struct {
    float* v;
    int64_t* i;
    int n, cap, largest;
} heap_t;

static void heap_sift_down(heap_t* h, int p) {
    for (;;) {
        int l = 2 * p + 1, r = l + 1, w = p;
        /* root must be the WORST element: child replaces parent when the
         * child ranks after (is worse than) the parent */
        if (l < h->n && better(h->v[w], h->i[w], h->v[l], h->i[l], h->largest)) w = l;
        if (r < h->n && better(h->v[w], h->i[w], h->v[r], h->i[r], h->largest)) w = r;
        if (w == p) return;
        float tv = h->v[p]; h->v[p] = h->v[w]; h->v[w] = tv;
        int64_t ti = h->i[p]; h->i[p] = h->i[w]; h->i[w] = ti;
        p = w;
    }
}

static void heap_sift_up(heap_t* h, int c) {
    while (c > 0) {
        int p = (c - 1) / 2;
        if (better(h->v[p], h->i[p], h->v[c], h->i[c], h->largest)) {
            float tv = h->v[p]; h->v[p] = h->v[c]; h->v[c] = tv;
            int64_t ti = h->i[p]; h->i[p] = h->i[c]; h->i[c] = ti;
            c = p;
        } else {
            return;
        }
    }
}

static void heap_push(heap_t* h, float v, int64_t i) {
    if (h->n < h->cap) {
        h->v[h->n] = v;
        h->i[h->n] = i;
        heap_sift_up(h, h->n);
        h->n++;
    } else if (better(v, i, h->v[0], h->i[0], h->largest)) {
        h->v[0] = v;
        h->i[0] = i;
        heap_sift_down(h, 0);
    }
}

/* Pop everything, writing best-first into out. */
static void heap_drain_sorted(heap_t* h, float* ov, int64_t* oi) {
    int n = h->n;
    for (int pos = n - 1; pos >= 0; --pos) {
        ov[pos] = h->v[0];
        oi[pos] = h->i[0];
        h->n--;
        if (h->n > 0) {
            h->v[0] = h->v[h->n];
            h->i[0] = h->i[h->n];
            heap_sift_down(h, 0);
        }
    }
}

/* Top-k along rows of a dense [B, N] matrix (_C.topk / topk_thrust,
 * csrc/kernels/topk.cu:14-28; topk_warp.cu:80-110 route to the same). */
void orc_topk(const float* dist, int64_t B, int64_t N, int k, int largest,
              float* out_v, int64_t* out_i, int nthreads) {
    set_threads(nthreads);
#pragma omp parallel
    {
        float* hv = (float*)malloc(sizeof(float) * k);
        int64_t* hi = (int64_t*)malloc(sizeof(int64_t) * k);
#pragma omp for schedule(dynamic, 1)
        for (int64_t b = 0; b < B; ++b) {
            heap_t h = {hv, hi, 0, k, largest};
            for (int64_t j = 0; j < N; ++j) heap_push(&h, dist[b * N + j], j);
            heap_drain_sorted(&h, out_v + b * k, out_i + b * k);
        }
        free(hv);
        free(hi);
    }
}

/* Exact flat search: FlatIndex::search (csrc/index/flat_index.cpp:49-86) =
 * distance kernel -> topk_thrust -> ids_.index_select.  Streams rows per
 * query so the [Q, N] matrix is never held.  ids may be NULL (row index).
 * L2 sorts ascending, cosine / dot descending (flat_index.cpp:61-76). */
void orc_flat_search(int metric, const float* q, int64_t Q, const float* x, int64_t N,
                     int d, int k, const int64_t* ids, float* out_d, int64_t* out_i,
                     int acc64, int nthreads) {
    set_threads(nthreads);
    int largest = metric != ORC_L2;
    double* xsq = NULL;
    if (metric == ORC_COSINE) {
        xsq = (double*)malloc(sizeof(double) * (N > 0 ? N : 1));
        row_sqnorms(x, N, d, xsq, acc64);
    }
#pragma omp parallel
    {
        float* hv = (float*)malloc(sizeof(float) * k);
        int64_t* hi = (int64_t*)malloc(sizeof(int64_t) * k);
#pragma omp for schedule(dynamic, 1)
        for (int64_t b = 0; b < Q; ++b) {
            const float* qb = q + b * d;
            double qsq = 0.0;
            if (metric == ORC_COSINE) qsq = acc64 ? dot64(qb, qb, d) : (double)dot32(qb, qb, d);
            heap_t h = {hv, hi, 0, k, largest};
            for (int64_t j = 0; j < N; ++j) {
                float s = score_pair(metric, qb, x + j * d, d, qsq, xsq ? xsq[j] : 0.0, acc64);
                heap_push(&h, s, j);
            }
            heap_drain_sorted(&h, out_d + b * k, out_i + b * k);
            if (ids)
                for (int t = 0; t < k; ++t) out_i[b * k + t] = ids[out_i[b * k + t]];
        }
        free(hv);
        free(hi);
    }
    free(xsq);
}

/* Merge G per-shard top-k lists [G, Q, kin] into [Q, k] (the row-sharded
 * multi-GPU merge; the reference is single-GPU, so this defines it). */
void orc_topk_merge(int largest, const float* in_v, const int64_t* in_i, int G, int64_t Q,
                    int kin, int k, float* out_v, int64_t* out_i) {
    float* hv = (float*)malloc(sizeof(float) * k);
    int64_t* hi = (int64_t*)malloc(sizeof(int64_t) * k);
    for (int64_t b = 0; b < Q; ++b) {
        heap_t h = {hv, hi, 0, k, largest};
        for (int g = 0; g < G; ++g)
            for (int t = 0; t < kin; ++t) {
                int64_t o = ((int64_t)g * Q + b) * kin + t;
                heap_push(&h, in_v[o], in_i[o]);
            }
        heap_drain_sorted(&h, out_v + b * k, out_i + b * k);
    }
    free(hv);
    free(hi);
}

/* ------------------------------------------------------------------ */
/* k-means                                                             */
/* ------------------------------------------------------------------ */

/* Lloyd assign step, assign_clusters_kernel (csrc/kernels/kmeans.cu:11-45):
 * argmin over centroids of the sequential fused-FMA squared distance, strict
 * '<' so ties go to the lowest centroid index; dist_out gets sqrtf(min)
 * (kmeans.cu:43) when non-NULL, sqdist_out the squared minimum. */
void orc_kmeans_assign(const float* x, int64_t N, int d, const float* c, int K,
                       int32_t* labels, float* dist_out, float* sqdist_out, int nthreads) {
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < N; ++i) {
        const float* p = x + i * d;
        float best = INFINITY;
        int bi = 0;
        for (int j = 0; j < K; ++j) {
            float s = l2sq_fma_seq(p, c + (int64_t)j * d, d);
            if (s < best) {
                best = s;
                bi = j;
            }
        }
        labels[i] = bi;
        if (dist_out) dist_out[i] = sqrtf(best);
        if (sqdist_out) sqdist_out[i] = best;
    }
}

/* Lloyd update step, update_centroids_kernel (csrc/kernels/kmeans.cu:48-94):
 * centroid = mean of its points; a centroid with no points is left as it was
 * (the reference never writes it, kmeans.cu:88-93).  Sums in double here;
 * counts_out (may be NULL) receives the per-centroid counts. */
void orc_kmeans_update(const float* x, int64_t N, int d, const int32_t* labels, int K,
                       float* centroids, int64_t* counts_out) {
    double* sums = (double*)calloc((size_t)K * d, sizeof(double));
    int64_t* cnt = (int64_t*)calloc((size_t)K, sizeof(int64_t));
    for (int64_t i = 0; i < N; ++i) {
        int c = labels[i];
        cnt[c]++;
        const float* p = x + i * d;
        double* s = sums + (int64_t)c * d;
        for (int t = 0; t < d; ++t) s[t] += p[t];
    }
    for (int c = 0; c < K; ++c) {
        if (cnt[c] > 0)
            for (int t = 0; t < d; ++t)
                centroids[(int64_t)c * d + t] = (float)(sums[(int64_t)c * d + t] / (double)cnt[c]);
        if (counts_out) counts_out[c] = cnt[c];
    }
    free(sums);
    free(cnt);
}

/* Lloyd iterations from given initial centroids (kmeans_cuda's declared
 * contract, csrc/include/rapidadb/clustering/kmeans.h:9-24; the reference
 * never implements it).  Convergence: stop after an iteration whose summed
 * squared centroid shift is <= tol * (sum of squared centroid norms); tol <= 0
 * runs exactly max_iters iterations.  Returns the iterations run; *inertia is
 * the sum of squared distances of the final assignment. */
int orc_kmeans(const float* x, int64_t N, int d, int K, int max_iters, float tol,
               float* centroids, int32_t* labels, double* inertia, int nthreads) {
    float* sq = (float*)malloc(sizeof(float) * (N > 0 ? N : 1));
    float* prev = (float*)malloc(sizeof(float) * (size_t)K * d);
    int it = 0;
    for (it = 0; it < max_iters; ++it) {
        orc_kmeans_assign(x, N, d, centroids, K, labels, NULL, sq, nthreads);
        memcpy(prev, centroids, sizeof(float) * (size_t)K * d);
        orc_kmeans_update(x, N, d, labels, K, centroids, NULL);
        if (tol > 0) {
            double sh = 0, nn = 0;
            for (int64_t t = 0; t < (int64_t)K * d; ++t) {
                double dd = (double)centroids[t] - prev[t];
                sh += dd * dd;
                nn += (double)prev[t] * prev[t];
            }
            if (sh <= tol * nn) {
                ++it;
                break;
            }
        }
    }
    orc_kmeans_assign(x, N, d, centroids, K, labels, NULL, sq, nthreads);
    double s = 0;
    for (int64_t i = 0; i < N; ++i) s += sq[i];
    *inertia = s;
    free(sq);
    free(prev);
    return it;
}

/* ------------------------------------------------------------------ */
/* IVF-Flat (no reference implementation: semantics defined here)      */
/* ------------------------------------------------------------------ */

/* Coarse probe: the nprobe lists whose centroids are nearest in squared L2
 * (ascending, ties by lower list id).  Scores use the exact double formula. */
static void coarse_probe(const float* qv, const float* cent, int nlist, int d, int nprobe,
                         int64_t* probe, float* hv, int64_t* hi) {
    heap_t h = {hv, hi, 0, nprobe, 0};
    for (int l = 0; l < nlist; ++l) heap_push(&h, (float)l2sq64(qv, cent + (int64_t)l * d, d), l);
    float* tv = (float*)malloc(sizeof(float) * nprobe);
    heap_drain_sorted(&h, tv, probe);
    free(tv);
}

/* IVF-Flat search over an index stored list-contiguously: list l holds rows
 * list_off[l] .. list_off[l+1]-1 of x (row-major [n, d]), row_ids maps a
 * stored row to its user id.  Probes nprobe lists per query (coarse L2) and
 * scores every row of those lists with the flat formula of `metric`; output
 * ids sorted best-first, ties by lower user id. */
void orc_ivf_flat_search(int metric, const float* q, int64_t Q, int d,
                         const float* centroids, int nlist, const int64_t* list_off,
                         const float* x, const int64_t* row_ids, int nprobe, int k,
                         float* out_d, int64_t* out_i, int nthreads) {
    set_threads(nthreads);
    int largest = metric != ORC_L2;
#pragma omp parallel
    {
        float* hv = (float*)malloc(sizeof(float) * k);
        int64_t* hi = (int64_t*)malloc(sizeof(int64_t) * k);
        float* pv = (float*)malloc(sizeof(float) * nprobe);
        int64_t* pi = (int64_t*)malloc(sizeof(int64_t) * nprobe);
        int64_t* probe = (int64_t*)malloc(sizeof(int64_t) * nprobe);
#pragma omp for schedule(dynamic, 1)
        for (int64_t b = 0; b < Q; ++b) {
            const float* qb = q + b * d;
            coarse_probe(qb, centroids, nlist, d, nprobe, probe, pv, pi);
            double qsq = metric == ORC_COSINE ? dot64(qb, qb, d) : 0.0;
            heap_t h = {hv, hi, 0, k, largest};
            for (int p = 0; p < nprobe; ++p) {
                int64_t l = probe[p];
                for (int64_t r = list_off[l]; r < list_off[l + 1]; ++r) {
                    const float* xr = x + r * d;
                    double xsq = metric == ORC_COSINE ? dot64(xr, xr, d) : 0.0;
                    heap_push(&h, score_pair(metric, qb, xr, d, qsq, xsq, 1), row_ids[r]);
                }
            }
            /* fewer than k rows probed: pad with the worst value, id -1 */
            int got = h.n;
            heap_drain_sorted(&h, out_d + b * k, out_i + b * k);
            for (int t = got; t < k; ++t) {
                out_d[b * k + t] = largest ? -INFINITY : INFINITY;
                out_i[b * k + t] = -1;
            }
        }
        free(hv);
        free(hi);
        free(pv);
        free(pi);
        free(probe);
    }
}

/* ------------------------------------------------------------------ */
/* Product quantisation (no reference implementation: defined here)    */
/* ------------------------------------------------------------------ */

/* Residual PQ encoding.  Row i belongs to list labels[i]; its residual
 * r = x_i - centroid[labels[i]] (one fp32 subtraction per element) is split
 * into M sub-vectors of dsub = d / M dims; code m is the argmin over the ksub
 * codewords of the sequential fused-FMA squared distance (the assign
 * arithmetic above), ties to the lower codeword.  codebooks: [M, ksub, dsub]. */
void orc_pq_encode(const float* x, int64_t N, int d, const int32_t* labels,
                   const float* centroids, const float* codebooks, int M, int ksub,
                   uint8_t* codes, int nthreads) {
    set_threads(nthreads);
    int dsub = d / M;
#pragma omp parallel
    {
        float* r = (float*)malloc(sizeof(float) * d);
#pragma omp for schedule(static)
        for (int64_t i = 0; i < N; ++i) {
            const float* c = centroids + (int64_t)labels[i] * d;
            for (int t = 0; t < d; ++t) r[t] = x[i * d + t] - c[t];
            for (int m = 0; m < M; ++m) {
                const float* cb = codebooks + (int64_t)m * ksub * dsub;
                float best = INFINITY;
                int bj = 0;
                for (int j = 0; j < ksub; ++j) {
                    float s = l2sq_fma_seq(r + m * dsub, cb + (int64_t)j * dsub, dsub);
                    if (s < best) {
                        best = s;
                        bj = j;
                    }
                }
                codes[i * M + m] = (uint8_t)bj;
            }
        }
        free(r);
    }
}

/* IVF-PQ asymmetric-distance search (L2).  For each probed list l the query
 * residual r = q - centroid[l] gives a table LUT[m][j] = |r_m - codeword_mj|^2
 * (double); the distance of a stored row is sum_m LUT[m][code_m].  Lists are
 * stored contiguously as in orc_ivf_flat_search; codes [n, M]. */
void orc_ivfpq_search(const float* q, int64_t Q, int d, const float* centroids, int nlist,
                      const int64_t* list_off, const uint8_t* codes, const int64_t* row_ids,
                      const float* codebooks, int M, int ksub, int nprobe, int k,
                      float* out_d, int64_t* out_i, int nthreads) {
    set_threads(nthreads);
    int dsub = d / M;
#pragma omp parallel
    {
        float* hv = (float*)malloc(sizeof(float) * k);
        int64_t* hi = (int64_t*)malloc(sizeof(int64_t) * k);
        float* pv = (float*)malloc(sizeof(float) * nprobe);
        int64_t* pi = (int64_t*)malloc(sizeof(int64_t) * nprobe);
        int64_t* probe = (int64_t*)malloc(sizeof(int64_t) * nprobe);
        double* lut = (double*)malloc(sizeof(double) * M * ksub);
        float* r = (float*)malloc(sizeof(float) * d);
#pragma omp for schedule(dynamic, 1)
        for (int64_t b = 0; b < Q; ++b) {
            const float* qb = q + b * d;
            coarse_probe(qb, centroids, nlist, d, nprobe, probe, pv, pi);
            heap_t h = {hv, hi, 0, k, 0};
            for (int p = 0; p < nprobe; ++p) {
                int64_t l = probe[p];
                const float* c = centroids + l * d;
                for (int t = 0; t < d; ++t) r[t] = qb[t] - c[t];
                for (int m = 0; m < M; ++m)
                    for (int j = 0; j < ksub; ++j)
                        lut[m * ksub + j] =
                            l2sq64(r + m * dsub, codebooks + ((int64_t)m * ksub + j) * dsub, dsub);
                for (int64_t row = list_off[l]; row < list_off[l + 1]; ++row) {
                    const uint8_t* cd = codes + row * M;
                    double s = 0.0;
                    for (int m = 0; m < M; ++m) s += lut[m * ksub + cd[m]];
                    heap_push(&h, (float)s, row_ids[row]);
                }
            }
            int got = h.n;
            heap_drain_sorted(&h, out_d + b * k, out_i + b * k);
            for (int t = got; t < k; ++t) {
                out_d[b * k + t] = INFINITY;
                out_i[b * k + t] = -1;
            }
        }
        free(hv);
        free(hi);
        free(pv);
        free(pi);
        free(probe);
        free(lut);
        free(r);
    }
}
