"""Host query pipeline (AsyncBatchSearcher / PinnedBuffer, the reference's
python/rapidadb/async_search.py and pinned_buffer.py): multi-stream results
equal plain searches, host-in / host-out equals device search."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _db(precision):
    from rapidadb import IndexConfig, RapidaDB
    from rapidadb_b200.config import Metric, Precision

    g = np.random.default_rng(4)
    x = torch.from_numpy(g.standard_normal((20000, 64), dtype=np.float32))
    db = RapidaDB(config=IndexConfig(dim=64, metric=Metric.COSINE, precision=Precision(precision)))
    db.add(x.cuda())
    q = g.standard_normal((1000, 64), dtype=np.float32)
    return db, q


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_search_host_equals_device_search(device, precision):
    from rapidadb.async_search import AsyncBatchSearcher

    db, q = _db(precision)
    rd, ri = db.search(torch.from_numpy(q).cuda(), 10)
    s = AsyncBatchSearcher(db, num_streams=3)
    d, i = s.search_host(q, 10, batch_size=128)
    s.close()
    np.testing.assert_array_equal(i, ri.cpu().numpy())
    np.testing.assert_array_equal(d, rd.cpu().numpy())


def test_search_batches_in_order(device):
    from rapidadb.async_search import AsyncBatchSearcher
    from rapidadb.pinned_buffer import PinnedBuffer

    db, q = _db("bf16")
    buf = PinnedBuffer(256, 64)
    batches = [buf.copy_to_device(q[j:j + 200]).clone() for j in range(0, 1000, 200)]
    s = AsyncBatchSearcher(db, num_streams=2)
    out = s.search_batches(batches, 5)
    s.close()
    for b, (d, i) in zip(batches, out):
        rd, ri = db.search(b, 5)
        assert torch.equal(i, ri) and torch.equal(d, rd)
    with pytest.raises(ValueError, match="exceeds buffer size"):
        buf.copy_to_device(q[:300])
