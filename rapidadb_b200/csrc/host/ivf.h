// Host-side k-means primitives and IVF indices (see ivf_index.cpp).
#pragma once

#include <functional>
#include <vector>

#include "host.h"

namespace rdbh {

inline bool is_half(at::ScalarType t) { return t == at::kHalf || t == at::kBFloat16; }

// (labels int32 [n], squared distances [n]); exact = reference assign arithmetic
std::tuple<at::Tensor, at::Tensor> kmeans_assign(const at::Tensor& x, const at::Tensor& centroids, bool exact);
// (sums fp32 [K, d], counts int64 [K]) in ascending point order, atomic-free
std::tuple<at::Tensor, at::Tensor> kmeans_update(const at::Tensor& x, const at::Tensor& labels, int64_t K);
// sums / counts, keeping centroids whose count is 0
at::Tensor kmeans_finalize(const at::Tensor& sums, const at::Tensor& counts, const at::Tensor& centroids);
// (seg_start [K + 1], perm [n], counts [K]) of a stable sort by label
std::tuple<at::Tensor, at::Tensor, at::Tensor> label_sort(const at::Tensor& labels, int64_t K);
at::Tensor pq_row_terms(const at::Tensor& codes, const at::Tensor& labels, const at::Tensor& centroids,
                        const at::Tensor& codebooks);
at::Tensor pq_encode(const at::Tensor& x, const at::Tensor& labels, const at::Tensor& centroids,
                     const at::Tensor& codebooks);

// k-means (kmeans.cpp): the shape of rapidadb::KMeansResult / kmeans_cuda,
// csrc/include/rapidadb/clustering/kmeans.h:9-24
struct KMeansResult {
    at::Tensor centroids;  // [k, d] fp32
    at::Tensor labels;     // [n] int32
    at::Tensor inertia;    // scalar fp64: sum of squared distances (over all shards)
    int64_t iterations;
};
// Applied to each iteration's (sums [k, d], counts [k]) before finalize, and
// to ([1] inertia, [1] zero) at the end: sharded training all-reduces them.
using Reducer = std::function<void(at::Tensor&, at::Tensor&)>;
// k distinct indices of [0, n): Floyd's algorithm over a SplitMix64 stream
std::vector<int64_t> sample_rows(int64_t n, int64_t k, uint64_t seed);
KMeansResult kmeans(const at::Tensor& points, int64_t k, int64_t max_iters, double tol, int64_t seed,
                    const at::Tensor& init, bool exact, const Reducer& reduce);

class IVFBase {
  public:
    IVFBase(int dim, Metric metric, int nlist, int nprobe);
    virtual ~IVFBase() = default;
    void set_nprobe(int nprobe);
    int nprobe() const { return nprobe_; }
    int nlist() const { return nlist_; }
    int dim() const { return dim_; }
    int64_t size() const { return n_; }
    bool is_trained() const { return centroids_.defined(); }
    at::Tensor centroids() const { return centroids_; }
    // the stored rows, list by list without the free slots: offsets
    // [nlist + 1], per-list sizes, ids and list labels in that order
    at::Tensor list_offsets() const;
    at::Tensor list_sizes() const;
    at::Tensor stored_ids() const { return live_select(ids_); }
    at::Tensor stored_labels() const { return live_select(labels_); }
    // stored row slots, free ones included (each list keeps spare slots so
    // that adds append in place)
    int64_t capacity() const { return cap_; }
    virtual void reset();
    // coarse probe: [nq, min(nprobe, nlist)] nearest list ids (squared L2,
    // ties to the lower list).  With dim <= 128 and nprobe + 8 <= 128 the
    // centroids are ranked on the tensor cores (rdb_ivf_probe_tc) and the best
    // nprobe + 8 rescored exactly; set_probe_tensor_cores(false) uses the
    // CUDA-core flat search throughout.
    at::Tensor probe(const at::Tensor& queries) const;
    void set_probe_tensor_cores(bool on) { probe_tc_ = on; }
    bool probe_tensor_cores(int64_t nprobe) const;

  protected:
    // reinstalls stored-order labels (non-decreasing) and ids; rebuilds the
    // list ranges without free slots
    void restore_lists(const at::Tensor& labels, const at::Tensor& ids);
    // physical slot of each stored row, list by list ([n] int64)
    at::Tensor live_slots() const;
    at::Tensor live_select(const at::Tensor& t) const;
    // m new rows with list labels `lab` [m]: when every list has room, `dest`
    // gets the free slots after each list's rows (new rows in their given
    // order), list_end_ advances and true is returned; otherwise nothing
    // changes and false is returned.
    bool append_slots(const at::Tensor& lab, at::Tensor& dest);
    // new layout for the stored rows (in list order) followed by m new rows
    // with labels `lab`, every list with spare slots: `dest` gets the slot of
    // each of those rows; list_off_ / list_end_ / cap_ / n_ describe the new
    // layout (the caller moves its payloads there).
    void new_layout(const at::Tensor& lab, at::Tensor& dest);
    void set_centroids(const at::Tensor& centroids);
    void check_query(const at::Tensor& queries, int64_t k) const;
    at::Tensor new_ids(const at::Tensor& vectors, const at::Tensor& ids) const;

    int dim_;
    Metric metric_;
    int nlist_;
    int nprobe_ = 1;
    int64_t n_ = 0;
    at::Tensor centroids_;  // [nlist, dim] fp32
    at::Tensor cent_rows_;  // padded copy for the coarse probe
    int64_t cent_ld_ = 0;
    at::Tensor cent_xv_;    // |c|^2
    at::Tensor cent_hi_, cent_lo_, cent_rs_;  // fp16 planes of the centroids (tensor-core probe)
    bool probe_tc_ = true;
    at::Tensor labels_;     // [cap] list of each slot (-1: free)
    at::Tensor ids_;        // [cap] user id of each slot (-1: free)
    at::Tensor list_off_;   // [nlist + 1] slot ranges: list l owns list_off_[l] .. list_off_[l + 1] - 1
    at::Tensor list_end_;   // [nlist] its rows fill list_off_[l] .. list_end_[l] - 1
    int64_t cap_ = 0;       // slots
};

class IVFFlatIndex : public IVFBase {
  public:
    IVFFlatIndex(int dim, Metric metric, int nlist, int nprobe, Precision precision);
    void set_quantizer(const at::Tensor& centroids) { set_centroids(centroids); }
    void add(const at::Tensor& vectors, const at::Tensor& ids);
    Result search(const at::Tensor& queries, int64_t k) const;
    // scan with a given [nq, np] probe table (e.g. gathered from other ranks)
    Result search_probed(const at::Tensor& queries, const at::Tensor& probe, int64_t k) const;
    void reset() override;
    // stored rows in list order (INT8 storage: the dequantised rows)
    at::Tensor stored_vectors() const;
    // reinstalls a saved index: vectors [n, dim], list labels [n] (non-
    // decreasing) and ids [n], all in stored order (see stored_*())
    void restore(const at::Tensor& vectors, const at::Tensor& labels, const at::Tensor& ids);
    // INT8 storage (SQ8, rdb_sq8_encode): codes [n, dim] and scales [n] in
    // stored order, and their exact reinstallation
    bool sq8() const { return precision_ == Precision::INT8; }
    at::Tensor stored_sq8_codes() const;
    at::Tensor stored_sq8_scales() const;
    void restore_sq8(const at::Tensor& codes, const at::Tensor& scales, const at::Tensor& labels,
                     const at::Tensor& ids);
    // Tensor-core search with dim <= 128 and k <= 24, on by default: FP32 rows
    // (rdb_ivf_flat_search_tc) through fp16 hi / lo planes the index keeps
    // (rdb_f16_split, as many bytes again as the rows); FP16 / BF16 rows
    // (rdb_ivf_flat_search_tc_half) as stored.  Off frees the planes and
    // searches with the CUDA-core list scan (rdb_ivf_flat_scan).
    void set_tensor_cores(bool on);
    bool tensor_cores() const { return tc_wanted_; }
    // true when search(queries, k) runs on the tensor cores
    bool tensor_core_search(int64_t k) const;

  private:
    bool tc_rows() const;  // planes kept: FP32 rows, dim <= 128, switched on
    bool tc_half() const;  // FP16 / BF16 rows, dim <= 128, switched on: read as stored
    // planes (hi, lo, scale) of fp32 rows [m, ld_]; a value that is not
    // finite sets tc_bad_ (those rows are searched on CUDA cores)
    std::tuple<at::Tensor, at::Tensor, at::Tensor> split_rows(const at::Tensor& rows);
    void rebuild_planes();

    Precision precision_;
    int64_t ld_;
    at::Tensor rows_;    // [cap, ld] slots list by list, storage dtype (free slots zero)
    at::Tensor xv_;      // [cap]
    at::Tensor scales_;  // [cap] SQ8 row scales (INT8 storage only)
    bool tc_wanted_ = true;
    bool tc_bad_ = false;  // some stored value is not finite
    int64_t dp_ = 0;       // plane stride: dim rounded up to 64
    at::Tensor hi_, lo_;   // [cap, dp_] fp16 planes of rows_ (tensor-core search)
    at::Tensor rscale_;    // [cap] their power-of-two row scales
};

class IVFPQIndex : public IVFBase {
  public:
    IVFPQIndex(int dim, Metric metric, int nlist, int nprobe, int m, int ksub);
    void set_quantizer(const at::Tensor& centroids, const at::Tensor& codebooks);
    void add(const at::Tensor& vectors, const at::Tensor& ids);
    Result search(const at::Tensor& queries, int64_t k) const;
    Result search_probed(const at::Tensor& queries, const at::Tensor& probe, int64_t k) const;
    void reset() override;
    at::Tensor codebooks() const { return codebooks_; }
    // codes [n, M] in list order, as encoded (the stored copy may be rotated)
    at::Tensor stored_codes() const;
    at::Tensor stored_row_terms() const { return fast_ ? live_select(row_terms_) : row_terms_; }
    int pq_m() const { return M_; }
    int pq_k() const { return ksub_; }
    // true when search runs the query-major kernel (rotated code layout)
    bool query_major() const { return fast_; }
    // reinstalls a saved index: codes [n, M] as stored_codes(), list labels
    // [n] (non-decreasing) and ids [n] in stored order
    void restore(const at::Tensor& codes, const at::Tensor& labels, const at::Tensor& ids);

  private:
    int M_, ksub_;
    bool fast_;
    at::Tensor codebooks_;  // [M, ksub, dim / M] fp32
    at::Tensor codes_;      // [cap, M] uint8 slots list by list (rotated by slot when fast_)
    at::Tensor row_terms_;  // [cap] fp32 (fast_ only)
};

}  // namespace rdbh
