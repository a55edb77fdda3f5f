"""Index persistence (save / load): the reference has none; a loaded index
must answer exactly like the saved one (same scores, same ids) for Flat,
IVF-Flat and IVF-PQ (query-major and list-major code widths)."""
import numpy as np
import pytest
import torch

from rapidadb_b200 import IndexConfig, RapidaDB
from rapidadb_b200.config import IndexType, Metric, Precision


def _data(seed=3, n=12000, d=32, nq=64):
    g = np.random.default_rng(seed)
    centres = g.standard_normal((40, d)).astype(np.float32) * 3
    x = centres[g.integers(0, 40, n)] + g.standard_normal((n, d)).astype(np.float32)
    q = centres[g.integers(0, 40, nq)] + g.standard_normal((nq, d)).astype(np.float32)
    return torch.from_numpy(x.astype(np.float32)), torch.from_numpy(q.astype(np.float32))


CASES = [
    dict(index_type=IndexType.FLAT, metric=Metric.COSINE, precision=Precision.FP32),
    dict(index_type=IndexType.FLAT, metric=Metric.L2, precision=Precision.BF16),
    dict(index_type=IndexType.IVF, metric=Metric.L2, precision=Precision.FP32, nlist=32, nprobe=5),
    dict(index_type=IndexType.IVF, metric=Metric.COSINE, precision=Precision.BF16, nlist=32, nprobe=5),
    dict(index_type=IndexType.IVF_PQ, metric=Metric.L2, nlist=32, nprobe=5, pq_m=8, pq_k=64),
    dict(index_type=IndexType.IVF_PQ, metric=Metric.L2, nlist=32, nprobe=5, pq_m=2, pq_k=64),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c['index_type'].value}-{c['metric'].value}-"
                         f"{c.get('precision', Precision.FP32).value}-m{c.get('pq_m', 0)}")
def test_save_load_same_answers(tmp_path, case):
    x, q = _data()
    cfg = IndexConfig(dim=32, kmeans_iters=5, **case)
    db = RapidaDB(config=cfg)
    db.train(x[:6000].cuda())
    db.add(x[:7000].cuda(), torch.arange(1000, 8000))
    db.add(x[7000:].cuda(), torch.arange(50000, 55000))
    d0, i0 = db.search(q.cuda(), 10)
    path = tmp_path / "index.rdb"
    db.save(path)
    db2 = RapidaDB.load(path)
    assert len(db2) == len(db) and db2.config == db.config
    d1, i1 = db2.search(q.cuda(), 10)
    torch.testing.assert_close(d1, d0, rtol=0, atol=0)
    assert torch.equal(i1, i0)
    if case["index_type"] == IndexType.IVF_PQ:
        assert torch.equal(db2.index.stored_codes(), db.index.stored_codes())
    # the loaded index keeps growing like the original
    db.add(x[:100].cuda(), torch.arange(90000, 90100))
    db2.add(x[:100].cuda(), torch.arange(90000, 90100))
    d0, i0 = db.search(q.cuda(), 10)
    d1, i1 = db2.search(q.cuda(), 10)
    torch.testing.assert_close(d1, d0, rtol=0, atol=0)
    assert torch.equal(i1, i0)


@pytest.mark.gpu
def test_save_load_empty_and_untrained(tmp_path):
    for it in (IndexType.FLAT, IndexType.IVF, IndexType.IVF_PQ):
        db = RapidaDB(config=IndexConfig(dim=16, index_type=it, metric=Metric.L2, nlist=8, pq_m=4, pq_k=16))
        db.save(tmp_path / f"{it.value}.rdb")
        db2 = RapidaDB.load(tmp_path / f"{it.value}.rdb")
        assert len(db2) == 0 and db2.config.index_type == it and db2.is_trained == db.is_trained


def test_load_rejects_foreign_files(tmp_path):
    path = tmp_path / "other.pt"
    torch.save({"format": "something-else", "version": 1}, path)
    with pytest.raises(ValueError, match="not a rapidadb_b200 index file"):
        RapidaDB.load(path)
