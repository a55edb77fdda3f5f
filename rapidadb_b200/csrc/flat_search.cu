// Exact flat search (the replacement of FlatIndex::search,
// csrc/index/flat_index.cpp:49-86) and dense top-k (topk_thrust,
// csrc/kernels/topk.cu:14-28).
//
// Flat search never materialises the [nq, n] score matrix:
//   1. sample pass   - scan a strided sample of S rows with no threshold; the
//                      selection kernel returns each query's k-th best sample
//                      score thr[q].  The k sample winners are real rows, so
//                      the true k-th best score over all n rows is at least as
//                      good as thr[q]: rows scoring worse can never be in the
//                      answer.
//   2. main pass     - the fused scan (tcgen05 for fp16/bf16, CUDA cores for
//                      fp32) scores every row and appends only rows reaching
//                      thr[q] (about n k / S per query) to per-(split, query)
//                      candidate lists.
//   3. select        - per query: exact top-k of its candidates, sorted, ties to
//                      the lower row, rows -> user ids; L2 winners are
//                      re-scored as sum (q - x)^2.
//   4. repair        - a query whose candidate list overflowed its capacity
//                      (adversarial data, e.g. many identical rows) is marked
//                      by the select; the repair kernel rescans its splits
//                      exactly and a second select answers it (repair.cu).
//                      Both launches return at once when nothing overflowed.
// Everything stays on the stream: the call returns without waiting for the
// device (RDB_SEARCH_SYNC waits and reports a bounded-wait timeout).
#include <math.h>

#include <algorithm>
#include <utility>
#include <vector>

#include "repair.cuh"
#include "scan.cuh"
#include "select.cuh"

namespace rdb {
namespace {

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct PassPlan {
    int64_t rows;  // logical rows scanned
    int64_t row_step;
    int nsplit;
    int64_t rps;   // rows per split
    int64_t cap;   // candidates per (split, query)
};

struct FlatPlan {
    bool tc;
    int qtile, rtile;
    int64_t nq;  // queries in one chunk
    bool sample;
    bool given;       // thresholds supplied by the caller
    int64_t expect;   // candidates per query expected under given thresholds
    int group;        // tensor-core sample pass: rows per group maximum
    int64_t ngroups;  // sample rows / group
    PassPlan s, m;
    size_t ws_bytes;
    size_t off_qv, off_thr, off_cand, off_counts, off_flag, off_mark;
};

// target: (split x query-block) units to launch, about one per SM for the
// tensor-core scan (a CTA pair per two SMs when queries come in 256s), two per
// SM for the CUDA-core scan
PassPlan plan_pass(int64_t rows, int64_t row_step, int64_t nq, int qtile, int rtile, int64_t target) {
    PassPlan p;
    p.rows = rows;
    p.row_step = row_step;
    int64_t nqb = (nq + qtile - 1) / qtile;
    int64_t ntiles = (rows + rtile - 1) / rtile;
    int64_t nsplit = std::max<int64_t>(1, target / std::max<int64_t>(nqb, 1));
    nsplit = std::min<int64_t>(nsplit, std::max<int64_t>(ntiles, 1));
    nsplit = std::min<int64_t>(nsplit, 1024);
    // (query block, split) units run in waves of `target`; a CTA's time is
    // about (its tiles + 1) per wave.  When the one-wave split leaves many
    // SMs idle (nqb not dividing target), more splits over several waves can
    // balance better: take the split count with the least modelled time if
    // it gains more than 3 %
    {
        auto cost = [&](int64_t ns) {
            const int64_t waves = (nqb * ns + target - 1) / target;
            return (double)waves * (double)((ntiles + ns - 1) / ns + 1);
        };
        int64_t best = nsplit;
        double best_t = cost(nsplit);
        for (int64_t ns = 1; ns <= std::min<int64_t>(std::max<int64_t>(ntiles, 1), 64); ++ns)
            if (cost(ns) < best_t * 0.97 && cost(ns) < cost(best)) best = ns;
        nsplit = best;
    }
    int64_t tiles_per = (ntiles + nsplit - 1) / nsplit;
    p.rps = std::max<int64_t>(tiles_per, 1) * rtile;
    p.nsplit = (int)std::max<int64_t>(1, (rows + p.rps - 1) / p.rps);
    p.cap = p.rps;
    return p;
}

// expect_given > 0: the caller supplies the thresholds (no sample pass) and
// expects about that many candidates per query over the n rows
FlatPlan make_plan(int metric, int dtype, int64_t nq, int64_t n, int d, int k, int flags,
                   bool tc_ok, int64_t expect_given = 0, bool x_i8 = false) {
    (void)metric;
    (void)d;
    FlatPlan P = {};
    P.tc = tc_ok && (dtype == RDB_F16 || dtype == RDB_BF16);
    const bool pair = P.tc && tc_use_pair(nq);
    P.qtile = P.tc ? (pair ? 2 * kTcQueries : kTcQueries) : kSimtQueries;
    P.rtile = P.tc ? kTcRows : kSimtRows;
    P.nq = nq;
    const int sms = num_sms();
    // CTAs that run at once: TMA-fed fp32 scans hold one per SM (their ring
    // fills the shared memory), the register-staged CUDA-core scan two
    // (SQ8 rows go through the register-staged scan)
    const int64_t target = P.tc ? (pair ? sms / 2 : sms) : (dtype == RDB_F32 && !x_i8) ? sms : 2LL * sms;

    // sample size S, a power of two >= 8 k: the sample pass costs S / n of the
    // main scan, the candidates (about n k / S per query) cost the main scan's
    // epilogue and the select.  The tensor-core sample pass keeps group maxima
    // and its candidates are costly relative to its cheap per-row MMA work:
    // ~6 sqrt(n k) rows in [1024, 131072]; the CUDA-core sample pass emits
    // every sampled score as a candidate: ~1.5 sqrt(n k) in [1024, 32768].
    double sd = (P.tc ? 6.0 : 1.5) * sqrt((double)n * (double)k);
    // one CUDA-core query block: the sample pass runs one CTA per 256-row
    // tile, each as long as any other, so up to 32 tiles cost no more than
    // one and tighten the threshold (fewer candidates for the main pass)
    if (!P.tc && nq <= kSimtQueries) sd = std::max(sd, 8192.0);
    const int64_t smax = P.tc ? 131072 : 32768;
    int64_t S = 1024;
    while (S < sd && S < smax) S <<= 1;
    while (S > 1024 && 4 * S > n) S >>= 1;  // at most a quarter of the rows
    while (S < 8LL * k) S <<= 1;
    P.sample = !(flags & RDB_SEARCH_EXHAUSTIVE) && n >= 4 * S && expect_given <= 0;
    P.given = expect_given > 0 && !(flags & RDB_SEARCH_EXHAUSTIVE);
    if (P.sample) {
        int64_t step = n / S;
        P.s = plan_pass(S, step, nq, P.qtile, P.rtile, target);
        // tensor-core sample pass keeps the best score of each group of
        // `group` sample rows; the k-th best of those group maxima is still a
        // lower bound on the k-th best score (k distinct rows reach it), and
        // with >= 10 k groups it is nearly as tight as the k-th best row
        // (pass rate 1 - (1 - k / G)^(1 / group) against k / S)
        P.group = 1;
        while (P.group < 128 && S / (2 * P.group) >= 10LL * k) P.group <<= 1;
        P.ngroups = S / P.group;
    }
    P.m = plan_pass(n, 1, nq, P.qtile, P.rtile, target);
    // capacities stay >= min(k, rows per split), so an overflowed list can be
    // replaced by its split's exact top-k (repair.cu)
    if (P.given) {
        const int64_t expect = (int64_t)ceil((double)P.m.rps * (double)expect_given / (double)n);
        P.m.cap = std::min<int64_t>(P.m.rps, std::max<int64_t>({1024, 8 * expect + 256, (int64_t)k}));
        P.expect = expect_given;
    }
    if (P.sample) {
        // expected candidates per split: rps * k / S; keep 8x headroom
        int64_t expect = (int64_t)ceil((double)P.m.rps * (double)k / (double)S);
        P.m.cap = std::min<int64_t>(P.m.rps, std::max<int64_t>({1024, 8 * expect + 256, (int64_t)k}));
    }
    size_t cand_main = (size_t)P.m.nsplit * nq * P.m.cap * sizeof(uint2);
    size_t cand_samp = !P.sample ? 0
                       : P.tc ? (size_t)nq * P.ngroups * sizeof(float)
                              : (size_t)P.s.nsplit * nq * P.s.cap * sizeof(uint2);
    size_t cnt_main = (size_t)P.m.nsplit * nq * sizeof(int);
    size_t cnt_samp = P.sample ? (size_t)P.s.nsplit * nq * sizeof(int) : 0;
    size_t off = 0;
    P.off_flag = off;  // first in every plan: one overflow word for all query chunks
    off = align_up(off + 16, 256);
    P.off_qv = off;
    off = align_up(off + nq * sizeof(float), 256);
    P.off_thr = off;
    off = align_up(off + nq * sizeof(float), 256);
    P.off_mark = off;
    off = align_up(off + nq * sizeof(unsigned), 256);
    P.off_cand = off;
    off = align_up(off + std::max(cand_main, cand_samp), 256);
    P.off_counts = off;
    off = align_up(off + std::max(cnt_main, cnt_samp), 256);
    P.ws_bytes = off;
    return P;
}

bool tc_layout_ok(int dtype, const void* q, int64_t ldq, const void* x, int64_t ldx, int d) {
    if (dtype != RDB_F16 && dtype != RDB_BF16) return false;
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
    if ((ldq * 2) % 16 || (ldx * 2) % 16) return false;
    return d >= 8;
}

int run_chunk(const FlatPlan& P, int metric, int dtype, const void* q, int64_t nq, int64_t ldq,
              const void* x, int64_t n, int64_t ldx, const float* xv, int d, int k,
              const int64_t* ids, int64_t id_offset, float* out_d, int64_t* out_i,
              unsigned char* ws, cudaStream_t s, const float* thr_given, const float* x_scale) {
    float* qv = reinterpret_cast<float*>(ws + P.off_qv);
    float* thr = reinterpret_cast<float*>(ws + P.off_thr);
    uint2* cand = reinterpret_cast<uint2*>(ws + P.off_cand);
    int* counts = reinterpret_cast<int*>(ws + P.off_counts);
    unsigned* flag = reinterpret_cast<unsigned*>(ws + P.off_flag);
    unsigned* mark = reinterpret_cast<unsigned*>(ws + P.off_mark);
    const int cos_small = d <= 128 ? 1 : 0;
    const bool largest = metric_largest(metric);
    cudaEvent_t ev;

    // per-query metric values (any query stride); clears the overflow word
    RDB_TRY(timing_begin(TIMING_FLAT_PREP, s, &ev));
    RDB_TRY(launch_query_prep(metric, dtype, q, nq, ldq, d, qv, flag, s));
    if (ev) RDB_CUDA_TRY(cudaEventRecord(ev, s));

    ScanArgs a = {};
    a.metric = metric;
    a.cos_small = cos_small;
    a.dtype = dtype;
    a.q = q;
    a.nq = nq;
    a.ldq = ldq;
    a.x = x;
    a.ldx = ldx;
    a.d = d;
    a.qv = qv;
    a.xv = xv;
    a.x_i8 = x_scale ? 1 : 0;
    a.x_scale = x_scale;
    a.cand = cand;
    a.counts = counts;

    SelectArgs sa = {};
    sa.input = SEL_CANDIDATES;
    sa.nq = nq;
    sa.k = k;
    sa.largest = largest ? 1 : 0;
    sa.cand = cand;
    sa.counts = counts;
    sa.metric = metric;
    sa.cos_small = cos_small;
    sa.qv = qv;
    sa.xv = xv;
    sa.dtype = dtype;
    sa.qdata = q;
    sa.ldq = ldq;
    sa.xdata = x;
    sa.ldx = ldx;
    sa.d = d;
    sa.x_i8 = x_scale ? 1 : 0;
    sa.x_scale = x_scale;

    auto scan = [&](const ScanArgs& sc) {
        return P.tc ? launch_scan_tc(sc, SCAN_FILTER, s) : launch_scan_simt(sc, SCAN_FILTER, s);
    };

    RDB_TRY(timing_begin(TIMING_FLAT_SAMPLE, s, &ev));
    if (P.sample && P.tc) {
        // group maxima over the strided sample, then the k-th best of them
        ScanArgs sc = a;
        sc.n = P.s.rows;
        sc.row_step = P.s.row_step;
        sc.thr = nullptr;
        sc.nsplit = P.s.nsplit;
        sc.rows_per_split = P.s.rps;
        sc.group_out = reinterpret_cast<float*>(cand);
        sc.group = P.group;
        sc.ngroups = P.ngroups;
        RDB_TRY(launch_scan_tc(sc, SCAN_GROUPMAX, s));
        SelectArgs ss = {};
        ss.input = SEL_DENSE;
        ss.output = SEL_OUT_THRESHOLD;
        ss.nq = nq;
        ss.k = k;
        ss.largest = largest ? 1 : 0;
        ss.dense = reinterpret_cast<const float*>(cand);
        ss.dense_n = P.ngroups;
        ss.out_thr = thr;
        RDB_TRY(launch_select(ss, s));
    } else if (P.sample) {
        ScanArgs sc = a;
        sc.n = P.s.rows;
        sc.row_step = P.s.row_step;
        sc.thr = nullptr;
        sc.nsplit = P.s.nsplit;
        sc.rows_per_split = P.s.rps;
        sc.cap = P.s.cap;
        const int64_t nchunk = (d + 31) / 32;
        const int64_t ctas = (int64_t)P.s.nsplit * ((nq + kSimtQueries - 1) / kSimtQueries);
        if (2 * ctas <= num_sms() && nchunk > 1 && simt_tma_ok(sc, SCAN_PARTIAL)) {
            // fewer sample tiles than half the SMs: split the K chunks of each
            // tile over several CTAs (partial dot products summed into a dense
            // [nq, S] block that fits in the candidate area), then final
            // scores and the k-th best of each row.  The sums are exact to a
            // few ulps, inside the filter's slack.
            sc.ksplit = (int)std::min<int64_t>(nchunk, num_sms() / ctas);
            sc.dense_out = reinterpret_cast<float*>(cand);
            sc.ld_out = P.s.rows;
            RDB_CUDA_TRY(cudaMemsetAsync(sc.dense_out, 0, sizeof(float) * (size_t)nq * P.s.rows, s));
            RDB_TRY(launch_scan_simt(sc, SCAN_PARTIAL, s));
            RDB_TRY(launch_partial_finalize(sc, s));
            SelectArgs ss = {};
            ss.input = SEL_DENSE;
            ss.output = SEL_OUT_THRESHOLD;
            ss.nq = nq;
            ss.k = k;
            ss.largest = largest ? 1 : 0;
            ss.dense = sc.dense_out;
            ss.dense_n = P.s.rows;
            ss.out_thr = thr;
            RDB_TRY(launch_select(ss, s));
        } else {
            RDB_TRY(scan(sc));
            SelectArgs ss = sa;
            ss.output = SEL_OUT_THRESHOLD;
            ss.cap = P.s.cap;
            ss.nsplit = P.s.nsplit;
            ss.row_step = P.s.row_step;
            ss.out_thr = thr;
            ss.overflow = nullptr;
            RDB_TRY(launch_select(ss, s));
        }
    }
    if (ev) RDB_CUDA_TRY(cudaEventRecord(ev, s));
    {
        ScanArgs sc = a;
        sc.n = n;
        sc.row_step = 1;
        sc.thr = P.given ? thr_given : (P.sample ? thr : nullptr);
        sc.nsplit = P.m.nsplit;
        sc.rows_per_split = P.m.rps;
        sc.cap = P.m.cap;
        cudaEvent_t stop_ev;
        RDB_TRY(timing_begin(TIMING_FLAT_SCAN, s, &stop_ev));
        RDB_TRY(scan(sc));
        if (stop_ev) RDB_CUDA_TRY(cudaEventRecord(stop_ev, s));
        RDB_TRY(timing_begin(TIMING_FLAT_SELECT, s, &ev));
        SelectArgs ss = sa;
        ss.output = SEL_OUT_TOPK;
        ss.cap = P.m.cap;
        ss.nsplit = P.m.nsplit;
        ss.row_step = 1;
        ss.out_v = out_d;
        ss.out_i = out_i;
        ss.ids = ids;
        ss.id_offset = id_offset;
        ss.overflow = flag;
        ss.mark_q = mark;
        ss.rescore_margin = metric == RDB_METRIC_L2 ? 16 : 0;
        // candidates per query: ~1.1 n k / S under a sampled threshold
        // (group maxima loosen it slightly), every row without one
        ss.expect = P.given ? P.expect : P.sample ? (int64_t)(1.1 * (double)n * (double)k / (double)(P.s.rows)) + 1 : n;
        RDB_TRY(launch_select(ss, s));
        if (ev) RDB_CUDA_TRY(cudaEventRecord(ev, s));

        // overflowed queries: exact rescan of their splits, then their select
        RDB_TRY(timing_begin(TIMING_FLAT_REPAIR, s, &ev));
        RepairArgs ra = {};
        ra.metric = metric;
        ra.cos_small = cos_small;
        ra.dtype = dtype;
        ra.q = q;
        ra.nq = nq;
        ra.ldq = ldq;
        ra.x = x;
        ra.n = n;
        ra.ldx = ldx;
        ra.d = d;
        ra.k = k;
        ra.x_i8 = x_scale ? 1 : 0;
        ra.x_scale = x_scale;
        ra.qv = qv;
        ra.xv = xv;
        ra.flag = flag;
        ra.mark_q = mark;
        ra.cand = cand;
        ra.counts = counts;
        ra.cap = P.m.cap;
        ra.nsplit = P.m.nsplit;
        ra.rows_per_split = P.m.rps;
        ra.buf_keys = repair_buffer_keys(k, P.m.cap);
        ra.status = device_status_word();
        ra.status_mirror = status_mirror_device();
        RDB_TRY(launch_flat_repair(ra, s));
        SelectArgs rs = ss;
        rs.overflow = nullptr;
        rs.mark_q = nullptr;
        rs.only_q = mark;
        rs.gate = flag;
        rs.force_cta = 1;
        RDB_TRY(launch_select(rs, s));
        if (ev) RDB_CUDA_TRY(cudaEventRecord(ev, s));
    }
    return RDB_OK;
}

}  // namespace
}  // namespace rdb

using namespace rdb;

extern "C" {

size_t rdb_flat_search_workspace(int metric, int dtype, int64_t nq, int64_t n, int d, int k,
                                 int flags) {
    if (nq <= 0 || n <= 0 || d <= 0 || k <= 0) return 256;
    return make_plan(metric, dtype, nq, n, d, k, flags, true).ws_bytes;
}

int rdb_flat_search_plan(int metric, int dtype, int64_t nq, int64_t n, int d, int k, int flags, int64_t* out) {
    RDB_CHECK_ARG(out != nullptr, "out is NULL");
    RDB_CHECK_ARG(nq >= 1 && n >= 1 && d >= 1 && k >= 1 && k <= n, "bad shape");
    const FlatPlan P = make_plan(metric, dtype, nq, n, d, k, flags, true);
    out[0] = P.sample ? P.s.rows : 0;
    out[1] = P.sample && P.tc ? P.group : 0;
    out[2] = P.m.nsplit;
    out[3] = P.m.cap;
    out[4] = P.m.rps;
    out[5] = P.tc ? 1 : 0;
    out[6] = P.nq;
    return RDB_OK;
}

}  // extern "C"

namespace rdb {
namespace {

int flat_search_impl(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, const void* x, int64_t n,
                     int64_t ldx, const float* xv, int d, int k, const int64_t* ids, int64_t id_offset, int flags,
                     const float* thr_given, int64_t expect_given, float* out_d, int64_t* out_i, void* ws,
                     size_t ws_bytes, void* stream, const float* x_scale = nullptr) {
    RDB_CHECK_ARG(metric >= 0 && metric <= 2, "unknown metric %d", metric);
    RDB_CHECK_ARG(elem_size(dtype) != 0, "unknown dtype %d", dtype);
    RDB_CHECK_ARG(nq >= 0 && d >= 1, "bad shape");
    RDB_CHECK_ARG(n >= 1, "index is empty");
    RDB_CHECK_ARG(k >= 1 && k <= n, "k must be in [1, %lld]", (long long)n);
    RDB_CHECK_ARG(k <= kMaxK, "k must be <= %d", kMaxK);
    RDB_CHECK_ARG(n < (1LL << 32), "at most 2^32 - 1 rows per device");
    RDB_CHECK_ARG(ldq >= d && ldx >= d, "row strides must be >= d");
    if (nq == 0) return RDB_OK;
    RDB_CHECK_ARG(q && x && out_d && out_i && ws, "NULL pointer");
    RDB_CHECK_ARG(metric != RDB_METRIC_COSINE || xv, "cosine needs per-row values");
    RDB_CHECK_ARG(metric != RDB_METRIC_L2 || xv, "L2 needs per-row values");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool x_i8 = x_scale != nullptr;
    bool tc_ok = !x_i8 && tc_layout_ok(dtype, q, ldq, x, ldx, d);
    const int64_t eg = thr_given ? std::max<int64_t>(expect_given, 1) : 0;

    // largest query chunk whose plan fits the workspace
    FlatPlan P = make_plan(metric, dtype, nq, n, d, k, flags, tc_ok, eg, x_i8);
    int64_t chunk = nq;
    while (P.ws_bytes > ws_bytes && chunk > P.qtile) {
        chunk = std::max<int64_t>(P.qtile, (chunk / 2 + P.qtile - 1) / P.qtile * P.qtile);
        P = make_plan(metric, dtype, chunk, n, d, k, flags, tc_ok, eg, x_i8);
    }
    if (P.ws_bytes > ws_bytes)
        return set_error(RDB_ERR_WORKSPACE, "workspace too small: %zu bytes, need %zu", ws_bytes,
                         P.ws_bytes);
    unsigned char* w = static_cast<unsigned char*>(ws);
    const size_t es = elem_size(dtype);
    for (int64_t c0 = 0; c0 < nq; c0 += chunk) {
        int64_t cn = std::min(chunk, nq - c0);
        FlatPlan Pc = cn == chunk ? P : make_plan(metric, dtype, cn, n, d, k, flags, tc_ok, eg, x_i8);
        RDB_TRY(run_chunk(Pc, metric, dtype, static_cast<const char*>(q) + c0 * ldq * es, cn, ldq,
                          x, n, ldx, xv, d, k, ids, id_offset, out_d + c0 * k, out_i + c0 * k, w,
                          s, thr_given ? thr_given + c0 : nullptr, x_scale));
    }
    if (flags & RDB_SEARCH_SYNC) {
        // wait for this call and report a bounded-wait timeout of its kernels
        unsigned* host = host_words();
        unsigned* st = device_status_word();
        if (!host || !st) return set_error(RDB_ERR_CUDA, "cannot allocate the status words");
        host[1] = 0;
        RDB_CUDA_TRY(cudaMemcpyAsync(&host[1], st, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
        RDB_CUDA_TRY(cudaStreamSynchronize(s));
        if (host[1]) return set_error(RDB_ERR_TIMEOUT, "a search kernel gave up on a device wait (status 0x%x)", host[1]);
    }
    return RDB_OK;
}

}  // namespace
}  // namespace rdb

extern "C" {

int rdb_flat_search(int metric, int dtype, const void* q, int64_t nq, int64_t ldq,
                    const void* x, int64_t n, int64_t ldx, const float* xv, int d, int k,
                    const int64_t* ids, int64_t id_offset, int flags, float* out_d,
                    int64_t* out_i, void* ws, size_t ws_bytes, void* stream) {
    return flat_search_impl(metric, dtype, q, nq, ldq, x, n, ldx, xv, d, k, ids, id_offset, flags, nullptr, 0,
                            out_d, out_i, ws, ws_bytes, stream);
}

size_t rdb_flat_search_sq8_workspace(int metric, int64_t nq, int64_t n, int d, int k, int flags) {
    if (nq <= 0 || n <= 0 || d <= 0 || k <= 0) return 256;
    return make_plan(metric, RDB_F32, nq, n, d, k, flags, false, 0, true).ws_bytes;
}

int rdb_flat_search_sq8(int metric, const float* q, int64_t nq, int64_t ldq, const int8_t* codes, const float* scales,
                        int64_t n, int64_t ldx, const float* xv, int d, int k, const int64_t* ids, int64_t id_offset,
                        int flags, float* out_d, int64_t* out_i, void* ws, size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(scales != nullptr || n == 0, "scales is NULL");
    RDB_CHECK_ARG(ldx % 4 == 0, "SQ8 row stride must be a multiple of 4 bytes");
    return flat_search_impl(metric, RDB_F32, q, nq, ldq, codes, n, ldx, xv, d, k, ids, id_offset, flags, nullptr, 0,
                            out_d, out_i, ws, ws_bytes, stream, scales ? scales : nullptr);
}

size_t rdb_flat_search_thr_workspace(int metric, int dtype, int64_t nq, int64_t n, int d, int k, int64_t expect) {
    if (nq <= 0 || n <= 0 || d <= 0 || k <= 0) return 256;
    return make_plan(metric, dtype, nq, n, d, k, 0, true, std::max<int64_t>(expect, 1)).ws_bytes;
}

int rdb_flat_search_thr(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, const void* x, int64_t n,
                        int64_t ldx, const float* xv, int d, int k, const int64_t* ids, int64_t id_offset,
                        const float* thr, int64_t expect, float* out_d, int64_t* out_i, void* ws, size_t ws_bytes,
                        void* stream) {
    RDB_CHECK_ARG(thr != nullptr, "thr is NULL");
    return flat_search_impl(metric, dtype, q, nq, ldq, x, n, ldx, xv, d, k, ids, id_offset, 0, thr, expect, out_d,
                            out_i, ws, ws_bytes, stream);
}

size_t rdb_flat_sample_workspace(int64_t nq) { return align_up(sizeof(float) * std::max<int64_t>(nq, 1), 256); }

int rdb_flat_sample_maxima(int metric, int dtype, const void* q, int64_t nq, int64_t ldq, const void* x, int64_t n,
                           int64_t ldx, const float* xv, int d, int64_t sample_rows, int group, float* out, void* ws,
                           size_t ws_bytes, void* stream) {
    RDB_CHECK_ARG(metric >= 0 && metric <= 2, "unknown metric %d", metric);
    RDB_CHECK_ARG(nq >= 0 && n >= 1 && d >= 1, "bad shape");
    RDB_CHECK_ARG(group >= 1 && group <= 128 && (group & (group - 1)) == 0, "group must be a power of two <= 128");
    RDB_CHECK_ARG(sample_rows >= group && sample_rows % group == 0 && sample_rows <= n,
                  "sample_rows must be a multiple of group in [group, n]");
    RDB_CHECK_ARG(metric == RDB_METRIC_DOT || xv, "cosine / L2 need per-row values");
    if (nq == 0) return RDB_OK;
    RDB_CHECK_ARG(q && x && out && ws, "NULL pointer");
    RDB_CHECK_ARG(ws_bytes >= rdb_flat_sample_workspace(nq), "workspace too small");
    if (!tc_layout_ok(dtype, q, ldq, x, ldx, d))
        return set_error(RDB_ERR_UNSUPPORTED, "sample maxima need fp16 / bf16 rows with 16-byte aligned strides");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* qv = static_cast<float*>(ws);
    RDB_TRY(row_sqnorms_ld(dtype, q, nq, d, ldq, qv, s));
    RDB_TRY(rdb_vec_values(metric, d, qv, nq, qv, s));
    const bool pair = tc_use_pair(nq);
    const int qtile = pair ? 2 * kTcQueries : kTcQueries;
    const int64_t target = pair ? num_sms() / 2 : num_sms();
    const PassPlan pp = plan_pass(sample_rows, n / sample_rows, nq, qtile, kTcRows, target);
    ScanArgs a = {};
    a.metric = metric;
    a.cos_small = d <= 128 ? 1 : 0;
    a.dtype = dtype;
    a.q = q;
    a.nq = nq;
    a.ldq = ldq;
    a.x = x;
    a.ldx = ldx;
    a.d = d;
    a.qv = qv;
    a.xv = xv;
    a.n = sample_rows;
    a.row_step = n / sample_rows;
    a.nsplit = pp.nsplit;
    a.rows_per_split = pp.rps;
    a.group_out = out;
    a.group = group;
    a.ngroups = sample_rows / group;
    return launch_scan_tc(a, SCAN_GROUPMAX, s);
}

int rdb_select_threshold(int largest, const float* scores, int64_t nq, int64_t G, int k, float* out_thr,
                         void* stream) {
    RDB_CHECK_ARG(nq >= 0 && G >= 1 && k >= 1 && k <= kMaxK, "bad shape");
    if (nq == 0) return RDB_OK;
    RDB_CHECK_ARG(scores && out_thr, "NULL pointer");
    SelectArgs ss = {};
    ss.input = SEL_DENSE;
    ss.output = SEL_OUT_THRESHOLD;
    ss.nq = nq;
    ss.k = k;
    ss.largest = largest ? 1 : 0;
    ss.dense = scores;
    ss.dense_n = G;
    ss.out_thr = out_thr;
    return launch_select(ss, static_cast<cudaStream_t>(stream));
}

size_t rdb_topk_workspace(int64_t B, int64_t N, int k) {
    (void)B;
    (void)N;
    (void)k;
    return 0;
}

int rdb_topk(const float* dist, int64_t B, int64_t N, int k, int largest, float* out_v,
             int64_t* out_i, void* ws, size_t ws_bytes, void* stream) {
    (void)ws;
    (void)ws_bytes;
    RDB_CHECK_ARG(B >= 0 && N >= 1, "bad shape");
    RDB_CHECK_ARG(k >= 1 && k <= N, "k must be in [1, num_vectors]");
    RDB_CHECK_ARG(k <= kMaxK, "k must be <= %d", kMaxK);
    RDB_CHECK_ARG(N < (1LL << 31), "rows longer than 2^31 - 1");
    if (B == 0) return RDB_OK;
    SelectArgs a = {};
    a.input = SEL_DENSE;
    a.output = SEL_OUT_TOPK;
    a.nq = B;
    a.k = k;
    a.largest = largest ? 1 : 0;
    a.dense = dist;
    a.dense_n = N;
    a.out_v = out_v;
    a.out_i = out_i;
    return launch_select(a, static_cast<cudaStream_t>(stream));
}

int rdb_topk_merge(int largest, const float* in_v, const int64_t* in_i, int G, int64_t nq,
                   int kin, int k, float* out_v, int64_t* out_i, void* stream) {
    return rdb_topk_merge_strided(largest, in_v, 0, in_i, 0, G, nq, kin, k, out_v, out_i, stream);
}

int rdb_topk_merge_strided(int largest, const float* in_v, int64_t gstride_v, const int64_t* in_i,
                           int64_t gstride_i, int G, int64_t nq, int kin, int k, float* out_v, int64_t* out_i,
                           void* stream) {
    return rdb_topk_merge_ld(largest, in_v, gstride_v, 0, in_i, gstride_i, 0, G, nq, kin, k, out_v, out_i, stream);
}

int rdb_topk_merge_ld(int largest, const float* in_v, int64_t gstride_v, int64_t ldv, const int64_t* in_i,
                      int64_t gstride_i, int64_t ldi, int G, int64_t nq, int kin, int k, float* out_v, int64_t* out_i,
                      void* stream) {
    RDB_CHECK_ARG(G >= 1 && kin >= 1 && k >= 1, "bad shape");
    RDB_CHECK_ARG(k <= (int64_t)G * kin, "k must be <= G * kin");
    RDB_CHECK_ARG(ldv == 0 || ldv >= kin, "row stride of the scores below kin");
    RDB_CHECK_ARG(ldi == 0 || ldi >= kin, "row stride of the ids below kin");
    const int64_t lv = ldv ? ldv : kin, li = ldi ? ldi : kin;
    RDB_CHECK_ARG(gstride_v == 0 || gstride_v >= (nq - 1) * lv + kin, "list stride of the scores too small");
    RDB_CHECK_ARG(gstride_i == 0 || gstride_i >= (nq - 1) * li + kin, "list stride of the ids too small");
    if (nq == 0) return RDB_OK;
    SelectArgs a = {};
    a.input = SEL_MERGE;
    a.output = SEL_OUT_TOPK;
    a.nq = nq;
    a.k = k;
    a.largest = largest ? 1 : 0;
    a.merge_v = in_v;
    a.merge_i = in_i;
    a.gstride_v = gstride_v;
    a.gstride_i = gstride_i;
    a.ldv = ldv;
    a.ldi = ldi;
    a.G = G;
    a.kin = kin;
    a.out_v = out_v;
    a.out_i = out_i;
    return launch_select(a, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
