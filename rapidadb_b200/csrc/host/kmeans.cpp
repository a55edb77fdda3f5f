// k-means training (Lloyd), the C++ host driver behind _C.kmeans.
//
// The reference declares kmeans_cuda(points, k, max_iters = 100, tol = 1e-4,
// seed = 42) -> KMeansResult{centroids, labels, inertia, iterations}
// (csrc/include/rapidadb/clustering/kmeans.h:9-24) and never defines it (its
// csrc/clustering/kmeans.cpp does not compile).  Each iteration here is
//   assign    labels + squared distances: fp16 / bf16 points on the tcgen05
//             scan with the argmin fused in its epilogue, fp32 on CUDA cores;
//             `exact` uses the reference assign arithmetic (kmeans.cu:31-35)
//   update    per-centroid sums and counts, atomic-free, ascending point order
//   reduce    optional hook (sharded training all-reduces sums and counts)
//   finalize  centroid = sum / count; a centroid with no points keeps its value
//             (kmeans.cu:88-93 leaves it unwritten)
// Initial centroids: k distinct rows drawn by Floyd's algorithm from a
// SplitMix64 stream seeded with `seed` (rapidadb_b200.utils.sample_rows draws
// the same rows).  Convergence: stop after an iteration whose summed squared
// centroid shift is <= tol * (sum of squared centroid norms); tol <= 0 runs
// max_iters iterations.  A final assignment gives the labels and the inertia.
#include <c10/cuda/CUDAGuard.h>

#include <unordered_set>
#include <vector>

#include "ivf.h"

namespace rdbh {

std::vector<int64_t> sample_rows(int64_t n, int64_t k, uint64_t seed) {
    TORCH_CHECK(k >= 0 && k <= n, "cannot sample ", k, " rows from ", n);
    uint64_t state = seed;
    auto next = [&state]() {
        state += 0x9E3779B97F4A7C15ull;
        uint64_t z = state;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    std::unordered_set<int64_t> chosen;
    std::vector<int64_t> order;
    order.reserve(static_cast<size_t>(k));
    for (int64_t j = n - k; j < n; ++j) {
        const int64_t t = static_cast<int64_t>(next() % static_cast<uint64_t>(j + 1));
        const int64_t pick = chosen.count(t) ? j : t;
        chosen.insert(pick);
        order.push_back(pick);
    }
    return order;
}

KMeansResult kmeans(const at::Tensor& points, int64_t k, int64_t max_iters, double tol, int64_t seed,
                    const at::Tensor& init, bool exact, const Reducer& reduce) {
    TORCH_CHECK(points.is_cuda(), "points must be a CUDA tensor");
    TORCH_CHECK(points.dim() == 2, "points must be 2D [n, dim]");
    TORCH_CHECK(points.scalar_type() == at::kFloat || is_half(points.scalar_type()),
                "points must be float32, float16 or bfloat16");
    TORCH_CHECK(k >= 1, "k must be >= 1");
    TORCH_CHECK(max_iters >= 0, "max_iters must be >= 0");
    c10::cuda::CUDAGuard guard(points.device());
    at::Tensor x = points.contiguous();
    at::Tensor cent;
    if (init.defined()) {
        TORCH_CHECK(init.dim() == 2 && init.size(0) == k && init.size(1) == x.size(1),
                    "init must be [k, dim] centroids");
        cent = init.to(x.device()).to(at::kFloat).contiguous();
    } else {
        TORCH_CHECK(k <= x.size(0), "k must be <= the number of points (", x.size(0), ")");
        const std::vector<int64_t> rows = sample_rows(x.size(0), k, static_cast<uint64_t>(seed));
        at::Tensor idx = at::tensor(rows, at::TensorOptions().dtype(at::kLong)).to(x.device());
        cent = x.index_select(0, idx).to(at::kFloat).contiguous();
    }
    int64_t it = 0;
    for (it = 1; it <= max_iters; ++it) {
        at::Tensor labels = std::get<0>(kmeans_assign(x, cent, exact));
        auto su = kmeans_update(x, labels, k);
        at::Tensor sums = std::get<0>(su), counts = std::get<1>(su);
        if (reduce) reduce(sums, counts);
        at::Tensor next = kmeans_finalize(sums, counts, cent);
        if (tol > 0) {
            const double shift = (next - cent).pow(2).sum().item<double>();
            const double norm = cent.pow(2).sum().item<double>();
            cent = next;
            if (shift <= tol * norm) break;
        } else {
            cent = next;
        }
    }
    if (it > max_iters) it = max_iters;
    auto fin = kmeans_assign(x, cent, exact);
    KMeansResult r;
    r.centroids = cent;
    r.labels = std::get<0>(fin);
    at::Tensor inertia = std::get<1>(fin).to(at::kDouble).sum().reshape({1});
    if (reduce) {
        at::Tensor none = at::zeros({1}, inertia.options().dtype(at::kLong));
        reduce(inertia, none);
    }
    r.inertia = inertia.reshape({});
    r.iterations = it;
    return r;
}

}  // namespace rdbh
