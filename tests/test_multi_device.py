"""IndexConfig.devices: one RapidaDB row-sharded over several GPUs of this
process.  Two shards on one GPU ([0, 0]) exercise the same split / gather /
merge logic on a single-GPU host; [0, 1] runs when two GPUs are present.
The sharded answer must equal the single-index answer (ids identical except
at score ties) and the exact oracle search."""
import numpy as np
import pytest
import torch

import oracle
from parity import assert_topk_match

pytestmark = pytest.mark.gpu


def _device_lists():
    lists = [[0, 0], [0, 0, 0]]
    if torch.cuda.is_available() and torch.cuda.device_count() >= 2:
        lists.append([0, 1])
    return lists


@pytest.mark.parametrize("devices", _device_lists(), ids=lambda d: "-".join(map(str, d)))
@pytest.mark.parametrize("precision,metric", [("bf16", "cosine"), ("fp32", "l2"), ("fp16", "dot_product")])
def test_flat_devices_equal_single_index(device, devices, precision, metric):
    from rapidadb import IndexConfig, Metric, RapidaDB
    from rapidadb_b200.config import Precision

    g = np.random.default_rng(5)
    x = g.standard_normal((30011, 96), dtype=np.float32)
    q = g.standard_normal((77, 96), dtype=np.float32)
    cfg = dict(dim=96, metric=Metric(metric), precision=Precision(precision))
    one = RapidaDB(config=IndexConfig(**cfg))
    many = RapidaDB(config=IndexConfig(devices=devices, **cfg))
    for lo, hi in ((0, 9000), (9000, 30011)):  # two adds: auto ids continue across calls
        one.add(torch.from_numpy(x[lo:hi]))
        many.add(torch.from_numpy(x[lo:hi]))
    assert len(many) == len(one) == 30011
    # each add splits its rows contiguously, the first n % G shards taking one more
    G = len(devices)
    expect = [sum(len(c) for c in (np.array_split(np.arange(n), G)[j] for n in (9000, 21011))) for j in range(G)]
    assert [s.size() for s in many.index.shards] == expect
    d1, i1 = one.search(torch.from_numpy(q), 25)
    d2, i2 = many.search(torch.from_numpy(q), 25)
    tol = 1e-5 if precision == "fp32" else 1e-4
    assert_topk_match(d1.cpu().numpy(), i1.cpu().numpy(), d2.cpu().numpy(), i2.cpu().numpy(), rtol=tol, atol=1e-5)
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[precision]
    xs = torch.from_numpy(x).to(dt).float().numpy()
    qs = torch.from_numpy(q).to(dt).float().numpy()
    rd, ri = oracle.flat_search(metric, qs, xs, 25)
    assert_topk_match(rd, ri, d2.cpu().numpy(), i2.cpu().numpy(), rtol=tol, atol=1e-5)


def test_devices_custom_ids_small_shards_and_k_above_a_shard(device):
    """k larger than one shard's rows: that shard's list is padded before the merge."""
    from rapidadb import IndexConfig, Metric, RapidaDB

    g = np.random.default_rng(9)
    x = g.standard_normal((9, 16), dtype=np.float32)
    ids = torch.arange(100, 109)
    db = RapidaDB(config=IndexConfig(dim=16, metric=Metric.L2, devices=[0, 0, 0, 0]))
    db.add(torch.from_numpy(x), ids)
    d, i = db.search(torch.from_numpy(x[:3]), 7)
    rd, ri = oracle.flat_search("l2", x[:3], x, 7, ids=np.arange(100, 109, dtype=np.int64))
    assert_topk_match(rd, ri, d.cpu().numpy(), i.cpu().numpy(), rtol=1e-5, atol=1e-5)
    with pytest.raises(RuntimeError, match="k must be in"):
        db.search(torch.from_numpy(x[:1]), 10)


def test_ivf_devices_train_add_search_and_persist(device, tmp_path):
    from rapidadb import IndexConfig, Metric, RapidaDB
    from rapidadb_b200.config import IndexType

    g = np.random.default_rng(2)
    centres = g.standard_normal((30, 32)).astype(np.float32) * 4
    x = (centres[g.integers(0, 30, 20000)] + g.standard_normal((20000, 32))).astype(np.float32)
    q = (x[:50] + 0.1 * g.standard_normal((50, 32))).astype(np.float32)
    cfg = dict(dim=32, metric=Metric.L2, index_type=IndexType.IVF, nlist=64, nprobe=8, kmeans_iters=5)
    one = RapidaDB(config=IndexConfig(**cfg))
    many = RapidaDB(config=IndexConfig(devices=[0, 0], **cfg))
    one.train(torch.from_numpy(x))
    many.train(torch.from_numpy(x))
    one.add(torch.from_numpy(x))
    many.add(torch.from_numpy(x))
    d1, i1 = one.search(torch.from_numpy(q), 10)
    d2, i2 = many.search(torch.from_numpy(q), 10)
    assert_topk_match(d1.cpu().numpy(), i1.cpu().numpy(), d2.cpu().numpy(), i2.cpu().numpy(), rtol=1e-5, atol=1e-5)
    path = tmp_path / "multi.pt"
    many.save(path)
    back = RapidaDB.load(path)
    d3, i3 = back.search(torch.from_numpy(q), 10)
    assert torch.equal(i3.cpu(), i2.cpu()) and torch.equal(d3.cpu(), d2.cpu())
