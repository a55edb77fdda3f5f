"""FlatIndex tests mirroring the reference's tests/python/test_flat_index.py."""
import pytest
import torch

pytestmark = pytest.mark.gpu


class TestFlatIndexBasic:
    def test_create_index(self, device):
        import rapidadb._C as _C

        idx = _C.FlatIndex(128, _C.Metric.COSINE)
        assert idx.dim() == 128
        assert idx.size() == 0

    def test_add_and_size(self, device, random_vectors):
        import rapidadb._C as _C

        idx = _C.FlatIndex(128, _C.Metric.COSINE)
        idx.add(random_vectors(100, dim=128))
        assert idx.size() == 100
        idx.add(random_vectors(50, dim=128))
        assert idx.size() == 150

    def test_reset(self, device, random_vectors):
        import rapidadb._C as _C

        idx = _C.FlatIndex(128, _C.Metric.COSINE)
        idx.add(random_vectors(100, dim=128))
        assert idx.size() == 100
        idx.reset()
        assert idx.size() == 0

    def test_repr(self, device, random_vectors):
        import rapidadb._C as _C

        idx = _C.FlatIndex(768, _C.Metric.COSINE)
        idx.add(random_vectors(42, dim=768))
        s = repr(idx)
        assert "768" in s
        assert "42" in s


class TestFlatIndexSearch:
    def test_search_returns_correct_shape(self, device, random_vectors):
        import rapidadb._C as _C

        idx = _C.FlatIndex(128, _C.Metric.COSINE)
        idx.add(random_vectors(1000, dim=128))
        distances, indices = idx.search(random_vectors(8, dim=128), k=10)
        assert distances.shape == (8, 10)
        assert indices.shape == (8, 10)

    def test_top1_is_self(self, device):
        import rapidadb._C as _C

        db = torch.randn(100, 128, device=device)
        idx = _C.FlatIndex(128, _C.Metric.COSINE)
        idx.add(db)
        distances, indices = idx.search(db[:5], k=1)
        expected_ids = torch.arange(5, device=device).unsqueeze(1)
        assert torch.equal(indices, expected_ids)

    def test_cosine_100pct_recall(self, device):
        import rapidadb._C as _C

        torch.manual_seed(42)
        db = torch.randn(500, 64, device=device)
        queries = torch.randn(32, 64, device=device)
        k = 10
        idx = _C.FlatIndex(64, _C.Metric.COSINE)
        idx.add(db)
        _, rapida_ids = idx.search(queries, k=k)
        sims = torch.nn.functional.normalize(queries, dim=1) @ torch.nn.functional.normalize(db, dim=1).T
        _, ref_ids = sims.topk(k, dim=1)
        recall = 0.0
        for i in range(32):
            recall += len(set(rapida_ids[i].cpu().tolist()) & set(ref_ids[i].cpu().tolist())) / k
        recall /= 32
        assert recall >= 0.99, f"Recall too low: {recall:.3f}"

    def test_l2_metric(self, device, random_vectors):
        import rapidadb._C as _C

        idx = _C.FlatIndex(64, _C.Metric.L2)
        idx.add(random_vectors(200, dim=64))
        distances, indices = idx.search(random_vectors(4, dim=64), k=10)
        for i in range(4):
            assert (distances[i][:-1] <= distances[i][1:] + 1e-5).all()

    def test_dot_product_metric(self, device, random_vectors):
        import rapidadb._C as _C

        idx = _C.FlatIndex(64, _C.Metric.DOT_PRODUCT)
        idx.add(random_vectors(200, dim=64))
        distances, indices = idx.search(random_vectors(4, dim=64), k=10)
        for i in range(4):
            assert (distances[i][:-1] >= distances[i][1:] - 1e-5).all()

    def test_custom_ids(self, device, random_vectors):
        import rapidadb._C as _C

        db = random_vectors(50, dim=64)
        ids = torch.arange(1000, 1050, device=device, dtype=torch.long)
        idx = _C.FlatIndex(64, _C.Metric.COSINE)
        idx.add(db, ids)
        _, result_ids = idx.search(db[:3], k=1)
        assert (result_ids >= 1000).all() and (result_ids < 1050).all()

    def test_batch_sizes(self, device, random_vectors):
        import rapidadb._C as _C

        idx = _C.FlatIndex(128, _C.Metric.COSINE)
        idx.add(random_vectors(500, dim=128))
        for batch in [1, 4, 16, 64, 128]:
            distances, indices = idx.search(random_vectors(batch, dim=128), k=5)
            assert distances.shape == (batch, 5)
            assert indices.shape == (batch, 5)

    def test_various_k(self, device, random_vectors):
        import rapidadb._C as _C

        idx = _C.FlatIndex(128, _C.Metric.COSINE)
        idx.add(random_vectors(500, dim=128))
        queries = random_vectors(4, dim=128)
        for k in [1, 5, 10, 50, 100, 500]:
            distances, indices = idx.search(queries, k=k)
            assert distances.shape == (4, k)
            assert indices.shape == (4, k)


class TestFlatIndexErrors:
    """Error conventions of flat_index.cpp:16-20, :50-55."""

    def test_empty_index(self, device):
        import rapidadb._C as _C

        idx = _C.FlatIndex(16, _C.Metric.L2)
        with pytest.raises(RuntimeError, match="index is empty"):
            idx.search(torch.randn(2, 16, device=device), 1)

    def test_k_out_of_range(self, device):
        import rapidadb._C as _C

        idx = _C.FlatIndex(16, _C.Metric.L2)
        idx.add(torch.randn(10, 16, device=device))
        with pytest.raises(RuntimeError, match=r"k must be in \[1, 10\]"):
            idx.search(torch.randn(2, 16, device=device), 11)

    def test_cpu_vectors(self):
        import rapidadb._C as _C

        idx = _C.FlatIndex(16, _C.Metric.L2)
        with pytest.raises(RuntimeError, match="must be on CUDA"):
            idx.add(torch.randn(10, 16))

    def test_wrong_dim(self, device):
        import rapidadb._C as _C

        idx = _C.FlatIndex(16, _C.Metric.L2)
        with pytest.raises(RuntimeError, match=r"vectors must be \[n, 16\]"):
            idx.add(torch.randn(10, 8, device=device))

    def test_ids_length(self, device):
        import rapidadb._C as _C

        idx = _C.FlatIndex(16, _C.Metric.L2)
        with pytest.raises(RuntimeError, match="ids length must match vectors"):
            idx.add(torch.randn(10, 16, device=device), torch.arange(9, device=device))
