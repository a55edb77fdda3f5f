// Host-side FlatIndex and raw ops over the C ABI.
//
// FlatIndex keeps the reference's semantics (csrc/index/flat_index.cpp):
// cloned storage, ids defaulting to arange(size, size + n), the same argument
// checks and messages; but rows live in an amortised-growth buffer (doubling
// capacity) instead of a torch::cat per add (flat_index.cpp:42-43), rows are
// padded to a 16-byte stride for TMA, and each row's metric value (squared
// norm or norm) is computed once at add time instead of per query pair.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <cstdio>

#include "host.h"

namespace rdbh {

void check_status(int status, const char* what) {
    TORCH_CHECK(status == RDB_OK, what, ": ", rdb_last_error());
}

int dtype_code(at::ScalarType t) {
    switch (t) {
        case at::kFloat: return RDB_F32;
        case at::kHalf: return RDB_F16;
        case at::kBFloat16: return RDB_BF16;
        default: TORCH_CHECK(false, "unsupported dtype ", t, " (expected float32, float16 or bfloat16)");
    }
    return -1;
}

at::ScalarType storage_type(Precision p) {
    switch (p) {
        case Precision::FP32: return at::kFloat;
        case Precision::FP16: return at::kHalf;
        case Precision::BF16: return at::kBFloat16;
        case Precision::INT8: return at::kChar;  // SQ8 codes (rdb_sq8_encode) + per-row scales
    }
    return at::kFloat;
}

void sq8_encode_into(const at::Tensor& vectors, at::Tensor codes, at::Tensor scales) {
    const int64_t n = vectors.size(0);
    if (n == 0) return;
    at::Tensor v = vectors;
    if (!(v.scalar_type() == at::kFloat || v.scalar_type() == at::kHalf || v.scalar_type() == at::kBFloat16))
        v = v.to(at::kFloat);
    if (v.stride(1) != 1) v = v.contiguous();
    TORCH_CHECK(codes.is_contiguous() || codes.stride(1) == 1, "codes rows must be dense");
    check_status(rdb_sq8_encode(dtype_code(v.scalar_type()), v.data_ptr(), n, v.stride(0), static_cast<int>(v.size(1)),
                                codes.data_ptr<int8_t>(), codes.stride(0), scales.data_ptr<float>(), stream_ptr()),
                 "sq8 encode");
}

at::Tensor sq8_row_values(Metric metric, const at::Tensor& codes, const at::Tensor& scales, int dim) {
    const int64_t n = codes.size(0);
    at::Tensor out = at::empty({n}, scales.options());
    if (n == 0) return out;
    check_status(rdb_sq8_row_values(static_cast<int>(metric), codes.data_ptr<int8_t>(), scales.data_ptr<float>(), n,
                                    codes.stride(0), dim, out.data_ptr<float>(), stream_ptr()),
                 "sq8 row values");
    return out;
}

at::Tensor sq8_dequantize(const at::Tensor& codes, const at::Tensor& scales, int dim) {
    // fl(scale * code), the value every SQ8 search scores against
    return codes.narrow(1, 0, dim).to(at::kFloat) * scales.unsqueeze(1);
}

void* stream_ptr() { return static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()); }

void check_pending_status() {
    unsigned v = 0;
    check_status(rdb_pending_status(&v), "device status");
    if (v != 0) {
        char buf[32];
        snprintf(buf, sizeof(buf), "0x%x", v);
        TORCH_CHECK(false, "a search kernel on this device gave up on a bounded device wait (status ", buf,
                    "); results of searches since then are not valid. Read and clear the status with "
                    "device_status(True)");
    }
}

int64_t padded_ld(int dim, at::ScalarType dtype) {
    int64_t per16 = 16 / static_cast<int64_t>(c10::elementSize(dtype));
    return (dim + per16 - 1) / per16 * per16;
}

static bool is_float_type(at::ScalarType t) {
    return t == at::kFloat || t == at::kHalf || t == at::kBFloat16;
}

at::Tensor prepare_rows(const at::Tensor& src, at::ScalarType dtype, int64_t ld) {
    const int64_t n = src.size(0), dim = src.size(1);
    if (src.scalar_type() == dtype && ld == dim && src.is_contiguous() &&
        (reinterpret_cast<uintptr_t>(src.data_ptr()) & 15) == 0)
        return src;
    at::Tensor out = ld == dim ? at::empty({n, ld}, src.options().dtype(dtype))
                               : at::zeros({n, ld}, src.options().dtype(dtype));
    out.narrow(1, 0, dim).copy_(src);
    return out;
}

at::Tensor row_values(Metric metric, const at::Tensor& rows_padded, int dim) {
    const int64_t n = rows_padded.size(0);
    at::Tensor out = at::empty({n}, rows_padded.options().dtype(at::kFloat));
    if (n == 0) return out;
    check_status(rdb_row_sqnorms(dtype_code(rows_padded.scalar_type()), rows_padded.data_ptr(), n,
                                 static_cast<int>(rows_padded.size(1)), out.data_ptr<float>(), stream_ptr()),
                 "row norms");
    check_status(rdb_vec_values(static_cast<int>(metric), dim, out.data_ptr<float>(), n,
                                out.data_ptr<float>(), stream_ptr()),
                 "row values");
    return out;
}

// ------------------------------------------------------------------ raw ops

at::Tensor distance(Metric metric, const at::Tensor& queries, const at::Tensor& database) {
    TORCH_CHECK(queries.is_cuda(), "queries must be a CUDA tensor");
    TORCH_CHECK(database.is_cuda(), "database must be a CUDA tensor");
    TORCH_CHECK(queries.dim() == 2, "queries must be 2D [batch, dim]");
    TORCH_CHECK(database.dim() == 2, "database must be 2D [n, dim]");
    TORCH_CHECK(queries.size(1) == database.size(1), "dimension mismatch");
    TORCH_CHECK(is_float_type(queries.scalar_type()), "queries must be float32");
    TORCH_CHECK(is_float_type(database.scalar_type()), "database must be float32");
    c10::cuda::CUDAGuard guard(queries.device());
    at::Tensor q = queries, x = database;
    if (q.scalar_type() != x.scalar_type()) {
        q = q.to(at::kFloat);
        x = x.to(at::kFloat);
    }
    q = q.contiguous();
    x = x.contiguous();
    at::Tensor out = at::empty({q.size(0), x.size(0)}, q.options().dtype(at::kFloat));
    if (q.size(0) == 0 || x.size(0) == 0) return out;
    check_status(rdb_distance(static_cast<int>(metric), dtype_code(q.scalar_type()), q.data_ptr(), q.size(0),
                              x.data_ptr(), x.size(0), static_cast<int>(q.size(1)), out.data_ptr<float>(),
                              stream_ptr()),
                 "distance");
    return out;
}

Result topk(const at::Tensor& distances, int64_t k, bool largest) {
    TORCH_CHECK(distances.is_cuda(), "distances must be a CUDA tensor");
    TORCH_CHECK(distances.dim() == 2, "distances must be 2D [batch, n]");
    TORCH_CHECK(k > 0 && k <= distances.size(1), "k must be in [1, num_vectors]");
    c10::cuda::CUDAGuard guard(distances.device());
    at::Tensor d = distances.to(at::kFloat).contiguous();
    const int64_t B = d.size(0), N = d.size(1);
    at::Tensor v = at::empty({B, k}, d.options());
    at::Tensor i = at::empty({B, k}, d.options().dtype(at::kLong));
    if (B == 0) return {v, i};
    check_status(rdb_topk(d.data_ptr<float>(), B, N, static_cast<int>(k), largest ? 1 : 0, v.data_ptr<float>(),
                          i.data_ptr<int64_t>(), nullptr, 0, stream_ptr()),
                 "topk");
    return {v, i};
}

Result topk_merge(const at::Tensor& vals, const at::Tensor& ids, int64_t k, bool largest) {
    TORCH_CHECK(vals.is_cuda() && ids.is_cuda(), "merge inputs must be CUDA tensors");
    TORCH_CHECK(vals.dim() == 3 && ids.sizes() == vals.sizes(), "merge inputs must be [G, Q, k]");
    c10::cuda::CUDAGuard guard(vals.device());
    // rows of k entries must be dense; rows and lists may be strided (the
    // per-rank blocks of a packed exchange buffer are read in place)
    auto readable = [](const at::Tensor& t) {
        return t.stride(2) == 1 && t.stride(1) >= t.size(2) &&
               t.stride(0) >= (t.size(1) > 0 ? (t.size(1) - 1) * t.stride(1) + t.size(2) : 0);
    };
    at::Tensor v = vals.scalar_type() == at::kFloat && readable(vals) ? vals : vals.to(at::kFloat).contiguous();
    at::Tensor i = ids.scalar_type() == at::kLong && readable(ids) ? ids : ids.to(at::kLong).contiguous();
    const int64_t G = v.size(0), Q = v.size(1), kin = v.size(2);
    TORCH_CHECK(k >= 1 && k <= G * kin, "k must be in [1, G * k_in]");
    at::Tensor ov = at::empty({Q, k}, v.options().memory_format(at::MemoryFormat::Contiguous));
    at::Tensor oi = at::empty({Q, k}, i.options().memory_format(at::MemoryFormat::Contiguous));
    if (Q == 0) return {ov, oi};
    check_status(rdb_topk_merge_ld(largest ? 1 : 0, v.data_ptr<float>(), v.stride(0), v.stride(1),
                                   i.data_ptr<int64_t>(), i.stride(0), i.stride(1), static_cast<int>(G), Q,
                                   static_cast<int>(kin), static_cast<int>(k), ov.data_ptr<float>(),
                                   oi.data_ptr<int64_t>(), stream_ptr()),
                 "topk merge");
    return {ov, oi};
}

// `out` (optional): a contiguous fp32 [nq] CUDA tensor to write into
static void check_out(const c10::optional<at::Tensor>& out, const at::Tensor& like, at::IntArrayRef shape,
                      const char* what) {
    if (!out.has_value()) return;
    const at::Tensor& o = *out;
    TORCH_CHECK(o.is_cuda() && o.device() == like.device() && o.scalar_type() == at::kFloat && o.is_contiguous() &&
                    o.sizes() == shape,
                what, ": out must be a contiguous float32 tensor of shape ", shape, " on ", like.device());
}

at::Tensor select_threshold(const at::Tensor& scores, int64_t k, bool largest, const c10::optional<at::Tensor>& out_opt) {
    TORCH_CHECK(scores.is_cuda() && scores.dim() == 2, "scores must be a [nq, G] CUDA tensor");
    c10::cuda::CUDAGuard guard(scores.device());
    at::Tensor sc = scores.to(at::kFloat).contiguous();
    check_out(out_opt, sc, {sc.size(0)}, "select_threshold");
    at::Tensor out = out_opt.has_value() ? *out_opt : at::empty({sc.size(0)}, sc.options());
    check_status(rdb_select_threshold(largest ? 1 : 0, sc.data_ptr<float>(), sc.size(0), sc.size(1),
                                      static_cast<int>(k), out.data_ptr<float>(), stream_ptr()),
                 "select threshold");
    return out;
}

// ---------------------------------------------------------------- FlatIndex

FlatIndex::FlatIndex(int dim, Metric metric, Precision precision)
    : dim_(dim), metric_(metric), precision_(precision) {
    TORCH_CHECK(dim > 0, "dim must be positive");
    ld_ = padded_ld(dim, storage_type(precision));
}

void FlatIndex::reserve(int64_t rows) {
    const int64_t cap = capacity();
    if (rows <= cap) return;
    const int64_t ncap = std::max<int64_t>({rows, 2 * cap, 1024});
    auto opts = storage_.defined() ? storage_.options() : at::TensorOptions();
    at::Tensor s = at::zeros({ncap, ld_}, opts.dtype(storage_type(precision_)));
    at::Tensor xv = at::empty({ncap}, s.options().dtype(at::kFloat));
    at::Tensor ids = at::empty({ncap}, s.options().dtype(at::kLong));
    at::Tensor sc = sq8() ? at::empty({ncap}, s.options().dtype(at::kFloat)) : at::Tensor();
    if (n_ > 0) {
        s.narrow(0, 0, n_).copy_(storage_.narrow(0, 0, n_));
        xv.narrow(0, 0, n_).copy_(xv_.narrow(0, 0, n_));
        ids.narrow(0, 0, n_).copy_(ids_.narrow(0, 0, n_));
        if (sq8()) sc.narrow(0, 0, n_).copy_(scales_.narrow(0, 0, n_));
    }
    storage_ = s;
    xv_ = xv;
    ids_ = ids;
    scales_ = sc;
}

void FlatIndex::add(const at::Tensor& vectors, const at::Tensor& ids) {
    TORCH_CHECK(vectors.is_cuda(), "vectors must be on CUDA");
    TORCH_CHECK(vectors.dim() == 2 && vectors.size(1) == dim_,
                "vectors must be [n, " + std::to_string(dim_) + "]");
    TORCH_CHECK(is_float_type(vectors.scalar_type()), "vectors must be float32");
    const int64_t n = vectors.size(0);
    at::Tensor new_ids;
    if (ids.defined() && ids.numel() > 0) {
        TORCH_CHECK(ids.size(0) == n, "ids length must match vectors");
        new_ids = ids.to(at::kLong).to(vectors.device());
    }
    if (storage_.defined() && storage_.device() != vectors.device())
        TORCH_CHECK(false, "vectors must be on ", storage_.device(), " (the index's device)");
    c10::cuda::CUDAGuard guard(vectors.device());
    if (!storage_.defined()) {
        // first add fixes the device
        storage_ = at::zeros({0, ld_}, vectors.options().dtype(storage_type(precision_)));
        xv_ = at::empty({0}, vectors.options().dtype(at::kFloat));
        ids_ = at::empty({0}, vectors.options().dtype(at::kLong));
        if (sq8()) scales_ = at::empty({0}, vectors.options().dtype(at::kFloat));
    }
    if (n == 0) return;
    reserve(n_ + n);
    at::Tensor dst = storage_.narrow(0, n_, n);
    if (sq8()) {
        at::Tensor sc = scales_.narrow(0, n_, n);
        sq8_encode_into(vectors, dst, sc);
        xv_.narrow(0, n_, n).copy_(sq8_row_values(metric_, dst, sc, dim_));
    } else {
        dst.narrow(1, 0, dim_).copy_(vectors);
        xv_.narrow(0, n_, n).copy_(row_values(metric_, dst, dim_));
    }
    if (new_ids.defined())
        ids_.narrow(0, n_, n).copy_(new_ids);
    else
        ids_.narrow(0, n_, n).copy_(at::arange(n_, n_ + n, ids_.options()));
    n_ += n;
}

static Result search_impl(Metric metric, const at::Tensor& rows, int dim, const at::Tensor& xv,
                          const at::Tensor& q, int64_t k, const at::Tensor& ids, int64_t id_offset) {
    const int64_t n = rows.size(0), nq = q.size(0);
    const int dt = dtype_code(rows.scalar_type());
    at::Tensor out_d = at::empty({nq, k}, rows.options().dtype(at::kFloat));
    at::Tensor out_i = at::empty({nq, k}, rows.options().dtype(at::kLong));
    if (nq == 0) return {out_d, out_i};
    const int m = static_cast<int>(metric);
    check_pending_status();
    // scratch from torch's stream-ordered caching allocator: a pool hit, no
    // device allocation once warm, and safe for concurrent searches on
    // different streams (a per-index cached buffer would not be)
    size_t ws_bytes = rdb_flat_search_workspace(m, dt, nq, n, dim, static_cast<int>(k), 0);
    at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes)}, rows.options().dtype(at::kByte));
    const int64_t* idp = ids.defined() ? ids.data_ptr<int64_t>() : nullptr;
    const float* xvp = xv.defined() ? xv.data_ptr<float>() : nullptr;
    // no host synchronisation: overflowed candidate lists are repaired on the device
    int st = rdb_flat_search(m, dt, q.data_ptr(), nq, q.size(1), rows.data_ptr(), n, rows.size(1), xvp, dim,
                             static_cast<int>(k), idp, id_offset, 0, out_d.data_ptr<float>(),
                             out_i.data_ptr<int64_t>(), ws.data_ptr(), ws_bytes, stream_ptr());
    check_status(st, "flat search");
    return {out_d, out_i};
}

Result FlatIndex::search_rows(Metric metric, const at::Tensor& rows, int dim, const at::Tensor& xv,
                              const at::Tensor& q, int64_t k, const at::Tensor& ids, int64_t id_offset) {
    TORCH_CHECK(rows.is_cuda() && q.is_cuda(), "rows and queries must be CUDA tensors");
    TORCH_CHECK(rows.dim() == 2 && q.dim() == 2 && rows.size(1) == q.size(1), "dimension mismatch");
    TORCH_CHECK(rows.scalar_type() == q.scalar_type(), "rows and queries must share a dtype");
    TORCH_CHECK(rows.size(0) > 0, "index is empty");
    TORCH_CHECK(k > 0 && k <= rows.size(0), "k must be in [1, " + std::to_string(rows.size(0)) + "]");
    c10::cuda::CUDAGuard guard(rows.device());
    return search_impl(metric, rows, dim, xv, q, k, ids, id_offset);
}

Result FlatIndex::search(const at::Tensor& queries, int64_t k) const {
    TORCH_CHECK(queries.is_cuda(), "queries must be on CUDA");
    TORCH_CHECK(queries.dim() == 2 && queries.size(1) == dim_,
                "queries must be [batch, " + std::to_string(dim_) + "]");
    TORCH_CHECK(n_ > 0, "index is empty");
    TORCH_CHECK(k > 0 && k <= n_, "k must be in [1, " + std::to_string(n_) + "]");
    TORCH_CHECK(is_float_type(queries.scalar_type()), "queries must be float32");
    c10::cuda::CUDAGuard guard(storage_.device());
    if (sq8()) {
        // SQ8 rows: fp32 queries against the dequantised rows
        at::Tensor q = prepare_rows(queries.to(storage_.device()), at::kFloat, padded_ld(dim_, at::kFloat));
        const int64_t nq = q.size(0);
        at::Tensor out_d = at::empty({nq, k}, q.options().dtype(at::kFloat));
        at::Tensor out_i = at::empty({nq, k}, q.options().dtype(at::kLong));
        if (nq == 0) return {out_d, out_i};
        check_pending_status();
        const int m = static_cast<int>(metric_);
        size_t wsb = rdb_flat_search_sq8_workspace(m, nq, n_, dim_, static_cast<int>(k), 0);
        at::Tensor ws = at::empty({static_cast<int64_t>(wsb)}, q.options().dtype(at::kByte));
        check_status(rdb_flat_search_sq8(m, q.data_ptr<float>(), nq, q.size(1), storage_.data_ptr<int8_t>(),
                                         scales_.data_ptr<float>(), n_, ld_, xv_.data_ptr<float>(), dim_,
                                         static_cast<int>(k), ids_.data_ptr<int64_t>(), 0, 0, out_d.data_ptr<float>(),
                                         out_i.data_ptr<int64_t>(), ws.data_ptr(), wsb, stream_ptr()),
                     "flat search");
        return {out_d, out_i};
    }
    at::Tensor q = prepare_rows(queries.to(storage_.device()), storage_.scalar_type(), ld_);
    return search_impl(metric_, storage_.narrow(0, 0, n_), dim_, xv_.narrow(0, 0, n_), q, k,
                       ids_.narrow(0, 0, n_), 0);
}

at::Tensor FlatIndex::sample_maxima(const at::Tensor& queries, int64_t sample_rows, int64_t group,
                                    const c10::optional<at::Tensor>& out_opt) const {
    TORCH_CHECK(queries.is_cuda(), "queries must be on CUDA");
    TORCH_CHECK(queries.dim() == 2 && queries.size(1) == dim_,
                "queries must be [batch, " + std::to_string(dim_) + "]");
    TORCH_CHECK(n_ > 0, "index is empty");
    TORCH_CHECK(sample_rows >= group && sample_rows <= n_ && group >= 1, "bad sample size");
    c10::cuda::CUDAGuard guard(storage_.device());
    at::Tensor q = prepare_rows(queries.to(storage_.device()), storage_.scalar_type(), ld_);
    const int64_t nq = q.size(0);
    check_out(out_opt, q, {nq, sample_rows / group}, "sample_maxima");
    at::Tensor out = out_opt.has_value() ? *out_opt : at::empty({nq, sample_rows / group}, q.options().dtype(at::kFloat));
    at::Tensor ws = at::empty({static_cast<int64_t>(rdb_flat_sample_workspace(nq))}, q.options().dtype(at::kByte));
    check_status(rdb_flat_sample_maxima(static_cast<int>(metric_), dtype_code(storage_.scalar_type()), q.data_ptr(),
                                        nq, ld_, storage_.data_ptr(), n_, ld_, xv_.data_ptr<float>(), dim_,
                                        sample_rows, static_cast<int>(group), out.data_ptr<float>(), ws.data_ptr(),
                                        ws.numel(), stream_ptr()),
                 "sample maxima");
    return out;
}

Result FlatIndex::search_threshold(const at::Tensor& queries, int64_t k, const at::Tensor& thr_in,
                                   int64_t expect) const {
    TORCH_CHECK(queries.is_cuda(), "queries must be on CUDA");
    TORCH_CHECK(queries.dim() == 2 && queries.size(1) == dim_,
                "queries must be [batch, " + std::to_string(dim_) + "]");
    TORCH_CHECK(n_ > 0, "index is empty");
    TORCH_CHECK(k > 0 && k <= n_, "k must be in [1, " + std::to_string(n_) + "]");
    TORCH_CHECK(thr_in.dim() == 1 && thr_in.size(0) == queries.size(0), "thr must be [batch]");
    c10::cuda::CUDAGuard guard(storage_.device());
    at::Tensor q = prepare_rows(queries.to(storage_.device()), storage_.scalar_type(), ld_);
    at::Tensor thr = thr_in.to(storage_.device()).to(at::kFloat).contiguous();
    const int64_t nq = q.size(0);
    const int m = static_cast<int>(metric_), dt = dtype_code(storage_.scalar_type());
    at::Tensor out_d = at::empty({nq, k}, q.options().dtype(at::kFloat));
    at::Tensor out_i = at::empty({nq, k}, q.options().dtype(at::kLong));
    if (nq == 0) return {out_d, out_i};
    check_pending_status();
    size_t wsb = rdb_flat_search_thr_workspace(m, dt, nq, n_, dim_, static_cast<int>(k), expect);
    at::Tensor ws = at::empty({static_cast<int64_t>(wsb)}, q.options().dtype(at::kByte));
    int st = rdb_flat_search_thr(m, dt, q.data_ptr(), nq, ld_, storage_.data_ptr(), n_, ld_, xv_.data_ptr<float>(),
                                 dim_, static_cast<int>(k), ids_.data_ptr<int64_t>(), 0, thr.data_ptr<float>(), expect,
                                 out_d.data_ptr<float>(), out_i.data_ptr<int64_t>(), ws.data_ptr(), wsb,
                                 stream_ptr());
    check_status(st, "flat search");
    return {out_d, out_i};
}

void FlatIndex::reset() {
    storage_ = at::Tensor();
    xv_ = at::Tensor();
    ids_ = at::Tensor();
    scales_ = at::Tensor();
    n_ = 0;
}

at::Tensor FlatIndex::vectors() const {
    if (!storage_.defined()) return at::empty({0, dim_});
    if (sq8()) return sq8_dequantize(storage_.narrow(0, 0, n_), scales_.narrow(0, 0, n_), dim_);
    return storage_.narrow(0, 0, n_).narrow(1, 0, dim_);
}

at::Tensor FlatIndex::sq8_codes() const {
    TORCH_CHECK(sq8(), "the index does not store INT8 (SQ8) rows");
    if (!storage_.defined()) return at::empty({0, dim_}, at::kChar);
    return storage_.narrow(0, 0, n_).narrow(1, 0, dim_);
}

at::Tensor FlatIndex::sq8_scales() const {
    TORCH_CHECK(sq8(), "the index does not store INT8 (SQ8) rows");
    if (!storage_.defined()) return at::empty({0}, at::kFloat);
    return scales_.narrow(0, 0, n_);
}

void FlatIndex::add_sq8(const at::Tensor& codes, const at::Tensor& scales, const at::Tensor& ids) {
    TORCH_CHECK(sq8(), "the index does not store INT8 (SQ8) rows");
    TORCH_CHECK(codes.is_cuda() && scales.is_cuda(), "codes and scales must be on CUDA");
    TORCH_CHECK(codes.dim() == 2 && codes.size(1) == dim_ && codes.scalar_type() == at::kChar,
                "codes must be int8 [n, " + std::to_string(dim_) + "]");
    TORCH_CHECK(scales.dim() == 1 && scales.size(0) == codes.size(0), "scales must be [n]");
    const int64_t n = codes.size(0);
    c10::cuda::CUDAGuard guard(codes.device());
    if (!storage_.defined()) {
        storage_ = at::zeros({0, ld_}, codes.options());
        xv_ = at::empty({0}, codes.options().dtype(at::kFloat));
        ids_ = at::empty({0}, codes.options().dtype(at::kLong));
        scales_ = at::empty({0}, codes.options().dtype(at::kFloat));
    }
    if (n == 0) return;
    reserve(n_ + n);
    at::Tensor dst = storage_.narrow(0, n_, n);
    dst.narrow(1, 0, dim_).copy_(codes);
    scales_.narrow(0, n_, n).copy_(scales.to(at::kFloat));
    xv_.narrow(0, n_, n).copy_(sq8_row_values(metric_, dst, scales_.narrow(0, n_, n), dim_));
    if (ids.defined() && ids.numel() > 0)
        ids_.narrow(0, n_, n).copy_(ids.to(at::kLong));
    else
        ids_.narrow(0, n_, n).copy_(at::arange(n_, n_ + n, ids_.options()));
    n_ += n;
}

at::Tensor FlatIndex::ids() const {
    if (!ids_.defined()) return at::empty({0}, at::kLong);
    return ids_.narrow(0, 0, n_);
}

}  // namespace rdbh
