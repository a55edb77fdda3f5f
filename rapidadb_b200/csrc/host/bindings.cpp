// Python module rapidadb_b200._C: the names of the reference's rapidadb._C
// (csrc/bindings/torch_extension.cpp:16-90) plus the IVF / PQ / k-means
// additions.  Thin: argument conversion only; logic lives in host/*.cpp.
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <vector>

#include "host.h"
#include "ivf.h"

namespace py = pybind11;
using namespace rdbh;

static at::Tensor opt_tensor(const py::object& o) {
    if (o.is_none()) return at::Tensor();
    return o.cast<at::Tensor>();
}

PYBIND11_MODULE(_C, m) {
    m.doc() = "RapidaDB B200: sm_100a search kernels behind the RapidaDB API";

    py::enum_<Metric>(m, "Metric")
        .value("COSINE", Metric::COSINE)
        .value("L2", Metric::L2)
        .value("DOT_PRODUCT", Metric::DOT_PRODUCT);

    py::enum_<Precision>(m, "Precision")
        .value("FP32", Precision::FP32)
        .value("FP16", Precision::FP16)
        .value("BF16", Precision::BF16)
        .value("INT8", Precision::INT8);

    // ---- raw distance ops (torch_extension.cpp:34-44)
    m.def("cosine_similarity", [](const at::Tensor& q, const at::Tensor& x) { return distance(Metric::COSINE, q, x); },
          "Cosine similarity matrix [Q, N]", py::arg("queries"), py::arg("database"), py::call_guard<py::gil_scoped_release>());
    m.def("l2_distance", [](const at::Tensor& q, const at::Tensor& x) { return distance(Metric::L2, q, x); },
          "Squared L2 distance matrix [Q, N]", py::arg("queries"), py::arg("database"), py::call_guard<py::gil_scoped_release>());
    m.def("dot_product", [](const at::Tensor& q, const at::Tensor& x) { return distance(Metric::DOT_PRODUCT, q, x); },
          "Dot product matrix [Q, N]", py::arg("queries"), py::arg("database"), py::call_guard<py::gil_scoped_release>());

    // ---- top-k (torch_extension.cpp:47-63)
    m.def("topk", [](const at::Tensor& d, int64_t k, bool largest) { return topk(d, k, largest); },
          "Sorted top-k per row", py::arg("distances"), py::arg("k"), py::arg("largest") = true, py::call_guard<py::gil_scoped_release>());
    m.def("topk_thrust", [](const at::Tensor& d, int64_t k, bool largest) { return topk(d, k, largest); },
          "Sorted top-k per row (same kernel as topk)", py::arg("distances"), py::arg("k"),
          py::arg("largest") = true, py::call_guard<py::gil_scoped_release>());
    m.def(
        "topk_warp_heap",
        [](const at::Tensor& d, int64_t k, bool largest) {
            // the reference's warp-heap entry keeps its k <= 128 contract (topk_warp.cu:86)
            TORCH_CHECK(k > 0 && k <= 128, "warp heap supports k in [1, 128]");
            return topk(d, k, largest);
        },
        "Sorted top-k per row, k <= 128", py::arg("distances"), py::arg("k"), py::arg("largest") = true);
    m.def("topk_merge", &topk_merge, "Merge [G, Q, k_in] sorted lists into [Q, k]", py::arg("values"),
          py::arg("ids"), py::arg("k"), py::arg("largest"), py::call_guard<py::gil_scoped_release>());

    // ---- FlatIndex (torch_extension.cpp:66-89)
    py::class_<FlatIndex>(m, "FlatIndex")
        .def(py::init<int, Metric, Precision>(), py::arg("dim"), py::arg("metric") = Metric::COSINE,
             py::arg("precision") = Precision::FP32)
        .def(
            "add", [](FlatIndex& self, const at::Tensor& v, const py::object& ids) {
                at::Tensor t = opt_tensor(ids);
                py::gil_scoped_release release;
                self.add(v, t);
            },
            py::arg("vectors"), py::arg("ids") = py::none())
        .def(
            "search", [](const FlatIndex& self, const at::Tensor& q, int64_t k) { return self.search(q, k); },
            py::arg("queries"), py::arg("k"), py::call_guard<py::gil_scoped_release>())
        .def("reset", &FlatIndex::reset)
        .def("size", &FlatIndex::size)
        .def("dim", &FlatIndex::dim)
        .def("capacity", &FlatIndex::capacity)
        .def("vectors", &FlatIndex::vectors)
        .def("sample_maxima", &FlatIndex::sample_maxima, py::arg("queries"), py::arg("sample_rows"),
             py::arg("group"), py::arg("out") = py::none())
        .def("search_threshold", &FlatIndex::search_threshold, py::arg("queries"), py::arg("k"), py::arg("thr"),
             py::arg("expect"))
        .def("tensor_core", &FlatIndex::tensor_core)
        .def("sq8", &FlatIndex::sq8)
        .def("sq8_codes", &FlatIndex::sq8_codes)
        .def("sq8_scales", &FlatIndex::sq8_scales)
        .def("add_sq8", [](FlatIndex& self, const at::Tensor& codes, const at::Tensor& scales, const py::object& ids) {
            at::Tensor t = opt_tensor(ids);
            py::gil_scoped_release nogil;
            self.add_sq8(codes, scales, t);
        }, py::arg("codes"), py::arg("scales"), py::arg("ids") = py::none())
        .def("ids", &FlatIndex::ids)
        .def("__len__", &FlatIndex::size)
        .def("__repr__", [](const FlatIndex& self) {
            return "FlatIndex(dim=" + std::to_string(self.dim()) + ", size=" + std::to_string(self.size()) + ")";
        });

    m.def(
        "search_rows",
        [](Metric metric, const at::Tensor& rows, int dim, const at::Tensor& xv, const at::Tensor& q, int64_t k,
           const py::object& ids, int64_t id_offset) {
            return FlatIndex::search_rows(metric, rows, dim, xv, q, k, opt_tensor(ids), id_offset);
        },
        "Fused top-k search over caller-owned padded rows", py::arg("metric"), py::arg("rows"), py::arg("dim"),
        py::arg("row_values"), py::arg("queries"), py::arg("k"), py::arg("ids") = py::none(),
        py::arg("id_offset") = 0);
    // ---- k-means: the Lloyd driver (kmeans_cuda, csrc/include/rapidadb/clustering/kmeans.h:9-24)
    py::class_<KMeansResult>(m, "KMeansResult")
        .def_readonly("centroids", &KMeansResult::centroids)
        .def_readonly("labels", &KMeansResult::labels)
        .def_readonly("inertia", &KMeansResult::inertia)
        .def_readonly("iterations", &KMeansResult::iterations)
        .def("__iter__",
             [](const KMeansResult& r) {
                 return py::iter(py::make_tuple(r.centroids, r.labels, r.inertia, r.iterations));
             })
        .def("__repr__", [](const KMeansResult& r) {
            return "KMeansResult(k=" + std::to_string(r.centroids.size(0)) +
                   ", iterations=" + std::to_string(r.iterations) + ")";
        });
    m.def(
        "kmeans",
        [](const at::Tensor& points, int64_t k, int64_t max_iters, double tol, int64_t seed, const py::object& init,
           bool exact, const py::object& allreduce) {
            Reducer red;
            if (!allreduce.is_none()) {
                // sharded training: the Python callback all-reduces in place
                red = [allreduce](at::Tensor& a, at::Tensor& b) {
                    py::gil_scoped_acquire gil;
                    allreduce(a, b);
                };
            }
            at::Tensor it = opt_tensor(init);
            py::gil_scoped_release nogil;
            return kmeans(points, k, max_iters, tol, seed, it, exact, red);
        },
        "Lloyd k-means: (centroids, labels, inertia, iterations)", py::arg("points"), py::arg("k"),
        py::arg("max_iters") = 100, py::arg("tol") = 1e-4, py::arg("seed") = 42, py::arg("init") = py::none(),
        py::arg("exact") = false, py::arg("allreduce") = py::none());
    m.def("sample_rows", [](int64_t n, int64_t k, uint64_t seed) { return sample_rows(n, k, seed); },
          "k distinct rows of [0, n) (Floyd over SplitMix64)", py::arg("n"), py::arg("k"), py::arg("seed"));
    // ---- k-means primitives
    m.def("kmeans_assign", &kmeans_assign, "labels, squared distances", py::arg("points"), py::arg("centroids"),
          py::arg("exact") = false, py::call_guard<py::gil_scoped_release>());
    m.def("kmeans_update", &kmeans_update, "per-centroid sums and counts", py::arg("points"), py::arg("labels"),
          py::arg("k"), py::call_guard<py::gil_scoped_release>());
    m.def("kmeans_finalize", &kmeans_finalize, "sums / counts (empty clusters keep their centroid)",
          py::arg("sums"), py::arg("counts"), py::arg("centroids"), py::call_guard<py::gil_scoped_release>());
    m.def("label_sort", &label_sort, "stable counting sort by label", py::arg("labels"), py::arg("k"), py::call_guard<py::gil_scoped_release>());
    m.def("select_threshold", &select_threshold, "k-th best score of each row", py::arg("scores"), py::arg("k"),
          py::arg("largest"), py::arg("out") = py::none(), py::call_guard<py::gil_scoped_release>());
    m.def("pq_row_terms", &pq_row_terms, "per-row constant of the IVF-PQ distance", py::arg("codes"),
          py::arg("labels"), py::arg("centroids"), py::arg("codebooks"), py::call_guard<py::gil_scoped_release>());
    m.def("pq_encode", &pq_encode, "residual PQ codes", py::arg("points"), py::arg("labels"),
          py::arg("centroids"), py::arg("codebooks"), py::call_guard<py::gil_scoped_release>());

    // ---- IVF indices
    py::class_<IVFFlatIndex>(m, "IVFFlatIndex")
        .def(py::init<int, Metric, int, int, Precision>(), py::arg("dim"), py::arg("metric") = Metric::L2,
             py::arg("nlist") = 4096, py::arg("nprobe") = 64, py::arg("precision") = Precision::FP32)
        .def("set_quantizer", &IVFFlatIndex::set_quantizer, py::arg("centroids"))
        .def(
            "add", [](IVFFlatIndex& s, const at::Tensor& v, const py::object& ids) {
                at::Tensor t = opt_tensor(ids);
                py::gil_scoped_release release;
                s.add(v, t);
            },
            py::arg("vectors"), py::arg("ids") = py::none())
        .def("search", &IVFFlatIndex::search, py::arg("queries"), py::arg("k"), py::call_guard<py::gil_scoped_release>())
        .def("probe", &IVFFlatIndex::probe, py::arg("queries"), py::call_guard<py::gil_scoped_release>())
        .def("set_probe_tensor_cores", &IVFFlatIndex::set_probe_tensor_cores, py::arg("on"))
        .def("probe_tensor_cores", &IVFFlatIndex::probe_tensor_cores, py::arg("nprobe"))
        .def("search_probed", &IVFFlatIndex::search_probed, py::arg("queries"), py::arg("probe"), py::arg("k"), py::call_guard<py::gil_scoped_release>())
        .def("reset", &IVFFlatIndex::reset)
        .def("size", &IVFFlatIndex::size)
        .def("dim", &IVFFlatIndex::dim)
        .def("nlist", &IVFFlatIndex::nlist)
        .def("nprobe", &IVFFlatIndex::nprobe)
        .def("set_nprobe", &IVFFlatIndex::set_nprobe)
        .def("is_trained", &IVFFlatIndex::is_trained)
        .def("centroids", &IVFFlatIndex::centroids)
        .def("list_offsets", &IVFFlatIndex::list_offsets)
        .def("list_sizes", &IVFFlatIndex::list_sizes)
        .def("capacity", &IVFFlatIndex::capacity)
        .def("stored_ids", &IVFFlatIndex::stored_ids)
        .def("stored_labels", &IVFFlatIndex::stored_labels)
        .def("stored_vectors", &IVFFlatIndex::stored_vectors)
        .def("restore", &IVFFlatIndex::restore, py::arg("vectors"), py::arg("labels"), py::arg("ids"), py::call_guard<py::gil_scoped_release>())
        .def("sq8", &IVFFlatIndex::sq8)
        .def("stored_sq8_codes", &IVFFlatIndex::stored_sq8_codes)
        .def("stored_sq8_scales", &IVFFlatIndex::stored_sq8_scales)
        .def("restore_sq8", &IVFFlatIndex::restore_sq8, py::arg("codes"), py::arg("scales"), py::arg("labels"),
             py::arg("ids"), py::call_guard<py::gil_scoped_release>())
        .def("set_tensor_cores", &IVFFlatIndex::set_tensor_cores, py::arg("on"),
             py::call_guard<py::gil_scoped_release>())
        .def("tensor_cores", &IVFFlatIndex::tensor_cores)
        .def("tensor_core_search", &IVFFlatIndex::tensor_core_search, py::arg("k"))
        .def("__len__", &IVFFlatIndex::size)
        .def("__repr__", [](const IVFFlatIndex& s) {
            return "IVFFlatIndex(dim=" + std::to_string(s.dim()) + ", nlist=" + std::to_string(s.nlist()) +
                   ", size=" + std::to_string(s.size()) + ")";
        });

    py::class_<IVFPQIndex>(m, "IVFPQIndex")
        .def(py::init<int, Metric, int, int, int, int>(), py::arg("dim"), py::arg("metric") = Metric::L2,
             py::arg("nlist") = 4096, py::arg("nprobe") = 64, py::arg("m") = 16, py::arg("ksub") = 256)
        .def("set_quantizer", &IVFPQIndex::set_quantizer, py::arg("centroids"), py::arg("codebooks"))
        .def(
            "add", [](IVFPQIndex& s, const at::Tensor& v, const py::object& ids) {
                at::Tensor t = opt_tensor(ids);
                py::gil_scoped_release release;
                s.add(v, t);
            },
            py::arg("vectors"), py::arg("ids") = py::none())
        .def("search", &IVFPQIndex::search, py::arg("queries"), py::arg("k"), py::call_guard<py::gil_scoped_release>())
        .def("probe", &IVFPQIndex::probe, py::arg("queries"), py::call_guard<py::gil_scoped_release>())
        .def("set_probe_tensor_cores", &IVFPQIndex::set_probe_tensor_cores, py::arg("on"))
        .def("probe_tensor_cores", &IVFPQIndex::probe_tensor_cores, py::arg("nprobe"))
        .def("search_probed", &IVFPQIndex::search_probed, py::arg("queries"), py::arg("probe"), py::arg("k"), py::call_guard<py::gil_scoped_release>())
        .def("reset", &IVFPQIndex::reset)
        .def("size", &IVFPQIndex::size)
        .def("dim", &IVFPQIndex::dim)
        .def("nlist", &IVFPQIndex::nlist)
        .def("nprobe", &IVFPQIndex::nprobe)
        .def("set_nprobe", &IVFPQIndex::set_nprobe)
        .def("pq_m", &IVFPQIndex::pq_m)
        .def("pq_k", &IVFPQIndex::pq_k)
        .def("is_trained", &IVFPQIndex::is_trained)
        .def("centroids", &IVFPQIndex::centroids)
        .def("codebooks", &IVFPQIndex::codebooks)
        .def("list_offsets", &IVFPQIndex::list_offsets)
        .def("list_sizes", &IVFPQIndex::list_sizes)
        .def("capacity", &IVFPQIndex::capacity)
        .def("stored_ids", &IVFPQIndex::stored_ids)
        .def("stored_labels", &IVFPQIndex::stored_labels)
        .def("stored_codes", &IVFPQIndex::stored_codes)
        .def("stored_row_terms", &IVFPQIndex::stored_row_terms)
        .def("restore", &IVFPQIndex::restore, py::arg("codes"), py::arg("labels"), py::arg("ids"), py::call_guard<py::gil_scoped_release>())
        .def("query_major", &IVFPQIndex::query_major)
        .def("__len__", &IVFPQIndex::size)
        .def("__repr__", [](const IVFPQIndex& s) {
            return "IVFPQIndex(dim=" + std::to_string(s.dim()) + ", nlist=" + std::to_string(s.nlist()) +
                   ", m=" + std::to_string(s.pq_m()) + ", size=" + std::to_string(s.size()) + ")";
        });

    // ---- peer exchange arenas (CUDA IPC) and the exchange kernel of the
    // row-sharded search; pointers travel as integers
    m.def("peer_arena_alloc", [](int device, int64_t nbytes) {
        c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
        void* p = nullptr;
        unsigned char h[RDB_PEER_HANDLE_BYTES];
        check_status(rdb_peer_arena_alloc(static_cast<size_t>(nbytes), &p, h), "peer arena");
        return std::make_tuple(reinterpret_cast<uintptr_t>(p), py::bytes(reinterpret_cast<const char*>(h), sizeof h));
    }, py::arg("device"), py::arg("nbytes"));
    m.def("peer_arena_open", [](int device, const py::bytes& handle) {
        c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
        const std::string h = handle;
        TORCH_CHECK(h.size() == RDB_PEER_HANDLE_BYTES, "a peer arena handle has ", RDB_PEER_HANDLE_BYTES, " bytes");
        void* p = nullptr;
        check_status(rdb_peer_arena_open(reinterpret_cast<const unsigned char*>(h.data()), &p), "peer arena open");
        return reinterpret_cast<uintptr_t>(p);
    }, py::arg("device"), py::arg("handle"));
    m.def("peer_arena_close", [](int device, uintptr_t p) {
        c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
        check_status(rdb_peer_arena_close(reinterpret_cast<void*>(p)), "peer arena close");
    }, py::arg("device"), py::arg("ptr"));
    m.def("peer_arena_free", [](int device, uintptr_t p) {
        c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
        check_status(rdb_peer_arena_free(reinterpret_cast<void*>(p)), "peer arena free");
    }, py::arg("device"), py::arg("ptr"));
    m.def(
        "peer_gather",
        [](int rank, int slot, uint64_t epoch, const std::vector<uintptr_t>& base, int64_t arena_bytes, int64_t src_off,
           int64_t src_row_stride, int64_t row_bytes, const std::vector<int64_t>& row0,
           const std::vector<int64_t>& nrows, const at::Tensor& dst, const std::vector<int64_t>& dst_off,
           int64_t dst_row_stride, uint64_t limit_ns) {
            const size_t world = base.size();
            TORCH_CHECK(world >= 1 && world <= RDB_PEER_MAX_RANKS && row0.size() == world && nrows.size() == world &&
                            dst_off.size() == world,
                        "peer_gather: one base, row0, nrows and dst_off per rank (at most ", RDB_PEER_MAX_RANKS, ")");
            TORCH_CHECK(dst.is_cuda() && dst.is_contiguous(), "peer_gather: dst must be a contiguous CUDA tensor");
            int64_t end = 0;
            for (size_t p = 0; p < world; ++p)
                if (nrows[p] > 0) end = std::max(end, dst_off[p] + (nrows[p] - 1) * dst_row_stride + row_bytes);
            TORCH_CHECK(end <= static_cast<int64_t>(dst.numel() * dst.element_size()),
                        "peer_gather: the rows do not fit in dst");
            RdbPeerGather a{};
            a.world = static_cast<int>(world);
            a.rank = rank;
            a.slot = slot;
            a.epoch = epoch;
            a.arena_bytes = arena_bytes;
            a.src_off = src_off;
            a.src_row_stride = src_row_stride;
            a.row_bytes = row_bytes;
            a.dst = dst.data_ptr();
            a.dst_row_stride = dst_row_stride;
            for (size_t p = 0; p < world; ++p) {
                a.base[p] = reinterpret_cast<void*>(base[p]);
                a.row0[p] = row0[p];
                a.nrows[p] = nrows[p];
                a.dst_off[p] = dst_off[p];
            }
            c10::cuda::CUDAGuard guard(dst.device());
            check_status(rdb_peer_gather(&a, limit_ns, stream_ptr()), "peer gather");
        },
        py::arg("rank"), py::arg("slot"), py::arg("epoch"), py::arg("base"), py::arg("arena_bytes"), py::arg("src_off"),
        py::arg("src_row_stride"), py::arg("row_bytes"), py::arg("row0"), py::arg("nrows"), py::arg("dst"),
        py::arg("dst_off"), py::arg("dst_row_stride"), py::arg("limit_ns") = 2000000000ull);

    m.def("padded_ld", [](int dim, at::ScalarType t) { return padded_ld(dim, t); });
    m.def("prepare_rows", &prepare_rows, py::arg("src"), py::arg("dtype"), py::arg("ld"));
    m.def("row_values", &row_values, py::arg("metric"), py::arg("rows"), py::arg("dim"));
    m.def("abi_version", []() { return rdb_version(); });
    m.def("device_status", [](bool clear) {
        unsigned v = 0;
        check_status(rdb_device_status(&v, clear ? 1 : 0), "device status");
        return v;
    }, py::arg("clear") = true);
    m.def("pending_status", []() {
        unsigned v = 0;
        check_status(rdb_pending_status(&v), "pending status");
        return v;
    });
    // (status code, message) of the bounded-wait probe on the current stream
    m.def("probe_bounded_wait", [](unsigned long long limit_ns) {
        int st;
        {
            py::gil_scoped_release nogil;
            st = rdb_probe_bounded_wait(limit_ns, stream_ptr());
        }
        return std::make_tuple(st, std::string(st == RDB_OK ? "" : rdb_last_error()));
    }, py::arg("limit_ns") = 100000ull);
}
