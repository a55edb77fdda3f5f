// C++ host layer of rapidadb_b200: index classes owning device storage and
// calling the sm_100a kernels through the C ABI (include/rapidadb_b200.h).
// Mirrors the reference's C++ layer (csrc/index/flat_index.cpp,
// csrc/include/rapidadb/index/flat_index.h) and extends it with IVF-Flat,
// IVF-PQ and k-means.  Errors are raised as c10::Error (RuntimeError in
// Python) with the reference's messages.
#pragma once

#include <ATen/ATen.h>

#include <cstdint>
#include <string>
#include <tuple>

#include "rapidadb_b200.h"

namespace rdbh {

// Order of rapidadb::Metric / Precision (csrc/include/rapidadb/core/types.h:9-21).
enum class Metric : int { COSINE = RDB_METRIC_COSINE, L2 = RDB_METRIC_L2, DOT_PRODUCT = RDB_METRIC_DOT };
enum class Precision : int { FP32 = 0, FP16 = 1, BF16 = 2, INT8 = 3 };

using Result = std::tuple<at::Tensor, at::Tensor>;

// Throws RuntimeError with rdb_last_error() when status != RDB_OK.
void check_status(int status, const char* what);
int dtype_code(at::ScalarType t);
at::ScalarType storage_type(Precision p);
void* stream_ptr();
// Raises when a kernel on the current device reported a bounded-wait timeout
// (rdb_pending_status: a non-blocking read of mapped host memory).
void check_pending_status();

// ---------------------------------------------------------------- raw ops --
// csrc/kernels/distance.cu:471-610 (checks :475-481)
at::Tensor distance(Metric metric, const at::Tensor& queries, const at::Tensor& database);
// csrc/kernels/topk.cu:14-28 (checks :20-23)
Result topk(const at::Tensor& distances, int64_t k, bool largest);
// merge of per-shard [G, Q, kin] lists into [Q, k]
Result topk_merge(const at::Tensor& vals, const at::Tensor& ids, int64_t k, bool largest);
// k-th best of each row of scores [nq, G] (L2 smallest, else largest)
at::Tensor select_threshold(const at::Tensor& scores, int64_t k, bool largest,
                            const c10::optional<at::Tensor>& out = c10::nullopt);

// -------------------------------------------------------------- FlatIndex --
// csrc/include/rapidadb/index/flat_index.h:12-53, csrc/index/flat_index.cpp
class FlatIndex {
  public:
    FlatIndex(int dim, Metric metric, Precision precision = Precision::FP32);
    void add(const at::Tensor& vectors, const at::Tensor& ids);  // flat_index.cpp:15-47
    Result search(const at::Tensor& queries, int64_t k) const;    // flat_index.cpp:49-86
    void reset();                                                  // flat_index.cpp:88-92
    int64_t size() const { return n_; }
    int dim() const { return dim_; }
    Metric metric() const { return metric_; }
    Precision precision() const { return precision_; }
    // stored rows [size, dim] (a view, in the storage dtype) and ids [size]
    at::Tensor vectors() const;
    at::Tensor ids() const;
    int64_t capacity() const { return storage_.defined() ? storage_.size(0) : 0; }

    // Row-sharded search with a shared threshold (rdb_flat_sample_maxima /
    // rdb_flat_search_thr): group maxima [nq, sample_rows / group] of a
    // strided sample of the stored rows, and a search keeping only rows that
    // reach thr [nq] (expect: candidates per query expected over the rows).
    at::Tensor sample_maxima(const at::Tensor& queries, int64_t sample_rows, int64_t group,
                             const c10::optional<at::Tensor>& out = c10::nullopt) const;
    Result search_threshold(const at::Tensor& queries, int64_t k, const at::Tensor& thr, int64_t expect) const;
    bool tensor_core() const { return precision_ == Precision::FP16 || precision_ == Precision::BF16; }
    // INT8 storage (SQ8, rdb_sq8_encode): codes [size, dim] int8, scales [size];
    // vectors() returns the dequantised rows fl(scale * code)
    bool sq8() const { return precision_ == Precision::INT8; }
    at::Tensor sq8_codes() const;
    at::Tensor sq8_scales() const;
    void add_sq8(const at::Tensor& codes, const at::Tensor& scales, const at::Tensor& ids);

    // Search against externally owned rows (same layout rules): used by the
    // IVF coarse probe and by tests.
    // rows [n, ld] and queries [nq, ld] share dtype and padded stride; dim is
    // the logical dimension (<= ld, padding columns zero).
    static Result search_rows(Metric metric, const at::Tensor& rows, int dim, const at::Tensor& row_values,
                              const at::Tensor& queries, int64_t k, const at::Tensor& ids,
                              int64_t id_offset);

  private:
    void reserve(int64_t rows);
    int dim_;
    int64_t ld_;  // padded row stride (elements): rows start 16-byte aligned
    Metric metric_;
    Precision precision_;
    at::Tensor storage_;  // [capacity, ld_] in the storage dtype, padding zero
    at::Tensor xv_;       // [capacity] per-row metric values
    at::Tensor ids_;      // [capacity] int64
    at::Tensor scales_;   // [capacity] fp32 SQ8 row scales (INT8 storage only)
    int64_t n_ = 0;
};

// Converts queries to `dtype` with a 16-byte aligned row stride; returns the
// tensor to hand to the kernels (rows of `ld` elements).
at::Tensor prepare_rows(const at::Tensor& src, at::ScalarType dtype, int64_t ld);
int64_t padded_ld(int dim, at::ScalarType dtype);
at::Tensor row_values(Metric metric, const at::Tensor& rows_padded, int dim);
// SQ8 (INT8 storage): encode rows into codes [n, ld] / scales [n] (in place),
// per-row metric values of the dequantised rows, and the dequantised rows
void sq8_encode_into(const at::Tensor& vectors, at::Tensor codes, at::Tensor scales);
at::Tensor sq8_row_values(Metric metric, const at::Tensor& codes, const at::Tensor& scales, int dim);
at::Tensor sq8_dequantize(const at::Tensor& codes, const at::Tensor& scales, int dim);

}  // namespace rdbh
