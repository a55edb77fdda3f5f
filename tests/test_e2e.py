"""End-to-end tests through the drop-in Python API, mirroring the reference's
tests/python/test_e2e.py."""
import pytest
import torch

pytestmark = pytest.mark.gpu


class TestRapidaDBE2E:
    def test_basic_workflow(self, device):
        from rapidadb import RapidaDB

        db = RapidaDB(dim=128, metric="cosine")
        db.add(torch.randn(1000, 128, device=device))
        assert len(db) == 1000
        assert db.dim == 128
        assert db.metric == "cosine"
        distances, indices = db.search(torch.randn(8, 128, device=device), k=10)
        assert distances.shape == (8, 10)
        assert indices.shape == (8, 10)

    def test_repr(self, device):
        from rapidadb import RapidaDB

        db = RapidaDB(dim=768)
        assert "768" in repr(db)
        assert "cosine" in repr(db)

    def test_reset(self, device):
        from rapidadb import RapidaDB

        db = RapidaDB(dim=64)
        db.add(torch.randn(100, 64, device=device))
        assert len(db) == 100
        db.reset()
        assert len(db) == 0

    def test_host_tensors_are_moved(self, device):
        """CPU inputs are copied to the GPU (index.py:82, :108)."""
        from rapidadb import RapidaDB

        db = RapidaDB(dim=32, metric="l2")
        x = torch.randn(300, 32)
        db.add(x)
        d, i = db.search(x[:4], k=1)
        assert i.flatten().tolist() == [0, 1, 2, 3]
        assert d.abs().max().item() < 1e-4
