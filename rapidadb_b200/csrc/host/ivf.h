// Host-side k-means primitives and IVF indices (see ivf_index.cpp).
#pragma once

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
    at::Tensor list_offsets() const { return list_off_; }
    at::Tensor list_sizes() const;
    at::Tensor stored_ids() const { return ids_; }
    at::Tensor stored_labels() const { return labels_; }
    virtual void reset();
    // coarse probe: [nq, min(nprobe, nlist)] nearest list ids (squared L2,
    // ties to the lower list)
    at::Tensor probe(const at::Tensor& queries) const;

  protected:
    // reinstalls stored-order labels (non-decreasing) and ids; rebuilds list_off
    void restore_lists(const at::Tensor& labels, const at::Tensor& ids);
    void set_centroids(const at::Tensor& centroids);
    void check_query(const at::Tensor& queries, int64_t k) const;
    std::tuple<at::Tensor, at::Tensor> relist(const at::Tensor& labels_all);
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
    at::Tensor labels_;     // [n] list of each stored row (stored order)
    at::Tensor ids_;        // [n] user ids (stored order)
    at::Tensor list_off_;   // [nlist + 1]
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
    at::Tensor stored_vectors() const { return rows_.defined() ? rows_.narrow(1, 0, dim_) : at::Tensor(); }
    // reinstalls a saved index: vectors [n, dim], list labels [n] (non-
    // decreasing) and ids [n], all in stored order (see stored_*())
    void restore(const at::Tensor& vectors, const at::Tensor& labels, const at::Tensor& ids);

  private:
    Precision precision_;
    int64_t ld_;
    at::Tensor rows_;  // [n, ld] list-major, storage dtype
    at::Tensor xv_;    // [n]
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
    at::Tensor stored_row_terms() const { return row_terms_; }
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
    at::Tensor codes_;      // [n, M] uint8, list-major (rotated when fast_)
    at::Tensor row_terms_;  // [n] fp32, list-major (fast_ only)
};

}  // namespace rdbh
