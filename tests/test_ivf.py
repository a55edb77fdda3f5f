"""IVF-Flat and IVF-PQ against the CPU oracle with identical centroids,
codebooks and list layout: list assignment and PQ codes must be identical,
top-k overlap >= 0.999 (the parity rule for IVF / IVF-PQ)."""
import numpy as np
import pytest
import torch

import oracle
from parity import recall

pytestmark = pytest.mark.gpu


def mixture(seed, n, d, ncent, spread=4.0, sigma=1.0):
    g = np.random.default_rng(seed)
    centres = g.standard_normal((ncent, d)).astype(np.float32) * spread
    x = centres[g.integers(0, ncent, n)] + sigma * g.standard_normal((n, d)).astype(np.float32)
    return x.astype(np.float32), g


def layout(idx, x):
    """The index's own list layout, as the oracle expects it."""
    off = idx.list_offsets().cpu().numpy()
    ids = idx.stored_ids().cpu().numpy()
    return off, ids, x[ids]


@pytest.mark.parametrize("metric", ["l2", "cosine", "dot_product"])
def test_ivf_flat_matches_oracle(device, metric):
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans

    x, g = mixture(0, 20000, 64, 40)
    q = (x[g.integers(0, len(x), 64)] + 0.5 * g.standard_normal((64, 64))).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    cent = kmeans(xt, 64, 8, 0.0, seed=1).centroids
    met = {"l2": _C.Metric.L2, "cosine": _C.Metric.COSINE, "dot_product": _C.Metric.DOT_PRODUCT}[metric]
    idx = _C.IVFFlatIndex(64, met, 64, 8)
    idx.set_quantizer(cent)
    idx.add(xt[:7000])
    idx.add(xt[7000:])
    # list assignment identical to the oracle's exact assignment
    lab_or, _, _ = oracle.kmeans_assign(x, cent.cpu().numpy())
    ids = idx.stored_ids().cpu().numpy()
    np.testing.assert_array_equal(idx.stored_labels().cpu().numpy(), lab_or[ids])
    off, row_ids, xs = layout(idx, x)
    assert (np.diff(row_ids[off[0]:off[1]]) > 0).all()  # stable within a list
    d, i = idx.search(torch.from_numpy(q).cuda(), 10)
    rd, ri = oracle.ivf_flat_search(metric, q, cent.cpu().numpy(), off, xs, row_ids, 8, 10)
    assert recall(i.cpu().numpy(), ri) >= 0.999
    np.testing.assert_allclose(d.cpu().numpy(), rd, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("k,shift", [(24, 0.0), (25, 0.0), (32, 0.0), (10, 20.0)])
def test_ivf_flat_l2_expansion_and_direct(device, k, shift):
    """L2 with k <= 24 over lists of >= 768 rows on average ranks by
    |q|^2 + |x|^2 - 2 q.x and rescores k + 8 rows per list directly; k > 24
    (and short lists, test_ivf_flat_matches_oracle) sum (q - x)^2 directly.
    Both report the direct distances, also when every vector carries a large
    common offset (|x|^2 far above the neighbour distances)."""
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans

    x, g = mixture(5, 40000, 48, 30)  # 1,250 rows per list
    x += shift
    q = (x[g.integers(0, len(x), 50)] + 0.5 * g.standard_normal((50, 48))).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    cent = kmeans(xt, 32, 8, 0.0, seed=2).centroids
    idx = _C.IVFFlatIndex(48, _C.Metric.L2, 32, 6)
    idx.set_quantizer(cent)
    idx.add(xt)
    off, row_ids, xs = layout(idx, x)
    d, i = idx.search(torch.from_numpy(q).cuda(), k)
    rd, ri = oracle.ivf_flat_search("l2", q, cent.cpu().numpy(), off, xs, row_ids, 6, k)
    assert recall(i.cpu().numpy(), ri) >= 0.999
    np.testing.assert_allclose(d.cpu().numpy(), rd, rtol=1e-5, atol=1e-5)


def test_ivf_flat_bf16_storage(device):
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans

    x, g = mixture(1, 8000, 32, 20)
    q = x[:40] + 0.1
    xt = torch.from_numpy(x).cuda()
    cent = kmeans(xt, 32, 5, 0.0, seed=2).centroids
    idx = _C.IVFFlatIndex(32, _C.Metric.L2, 32, 6, _C.Precision.BF16)
    idx.set_quantizer(cent)
    idx.add(xt)
    d, i = idx.search(torch.from_numpy(q).cuda(), 5)
    off, row_ids, _ = layout(idx, x)
    xs16 = torch.from_numpy(x).to(torch.bfloat16).float().numpy()[row_ids]
    q16 = torch.from_numpy(q).to(torch.bfloat16).float().numpy()
    rd, ri = oracle.ivf_flat_search("l2", q16, cent.cpu().numpy(), off, xs16, row_ids, 6, 5)
    # probe on fp32 queries vs bf16-rounded queries may pick different lists at ties
    assert recall(i.cpu().numpy(), ri) >= 0.99


@pytest.mark.parametrize("M,nlist,nprobe,query_major", [(4, 32, 6, True), (8, 32, 6, True), (16, 64, 40, True),
                                                          (32, 64, 40, True), (2, 32, 6, False)])
def test_ivfpq_codes_and_search_match_oracle(device, M, nlist, nprobe, query_major):
    """M = 4 / 8 / 16 / 32 run the query-major kernel (rotated code layout,
    per-row terms, the table built in registers), M = 2 the list-major scan
    + merge; both against the oracle's ADC."""
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans, train_pq

    x, g = mixture(2, 30000, 32, 50)
    q = (x[g.integers(0, len(x), 100)] + 0.3 * g.standard_normal((100, 32))).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    cent = kmeans(xt, nlist, 8, 0.0, seed=3).centroids
    lab, _ = _C.kmeans_assign(xt, cent, True)
    books = train_pq(xt - cent.index_select(0, lab.long()), M, 64, 6, seed=4)
    idx = _C.IVFPQIndex(32, _C.Metric.L2, nlist, nprobe, M, 64)
    assert idx.query_major() == query_major
    idx.set_quantizer(cent, books)
    idx.add(xt[:12345])
    idx.add(xt[12345:])
    off, row_ids, xs = layout(idx, x)
    cn, bn = cent.cpu().numpy(), books.cpu().numpy()
    lab_or, _, _ = oracle.kmeans_assign(x, cn)
    codes_or = oracle.pq_encode(x, lab_or, cn, bn)
    np.testing.assert_array_equal(idx.stored_codes().cpu().numpy(), codes_or[row_ids])
    if query_major:
        # T[row] = sum_m |cb[m][c_m]|^2 + 2 <(c_l)_m, cb[m][c_m]>
        c = codes_or[row_ids].astype(np.int64)
        rec = bn[np.arange(M)[None, :], c].reshape(len(c), -1).astype(np.float64)
        t = (rec * rec).sum(1) + 2.0 * (rec * cn[lab_or[row_ids]].astype(np.float64)).sum(1)
        np.testing.assert_allclose(idx.stored_row_terms().cpu().numpy(), t, rtol=1e-5, atol=1e-3)
    d, i = idx.search(torch.from_numpy(q).cuda(), 10)
    rd, ri = oracle.ivfpq_search(q, cn, off, codes_or[row_ids], row_ids, bn, nprobe, 10)
    assert recall(i.cpu().numpy(), ri) >= 0.999
    np.testing.assert_allclose(d.cpu().numpy(), rd, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("kind", ["flat_l2", "flat_cosine", "pq_m16", "pq_m2"])
def test_ivf_streaming_add_matches_bulk_add(device, kind):
    """Adds in many small and large batches -- appends into the free slots of
    every list when they have room, a new layout with spare slots when one
    runs out -- store exactly what one bulk add stores (lists, row order, ids,
    vectors / codes / row terms) and search identically (scores and ids
    equal, tolerance 0)."""
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans, train_pq

    d, nlist = 32, 32
    x, g = mixture(7, 12000, d, 24)
    q = (x[g.integers(0, len(x), 60)] + 0.3 * g.standard_normal((60, d))).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    ids = torch.arange(len(x), device=device) * 3 + 11
    cent = kmeans(xt, nlist, 6, 0.0, seed=3).centroids
    books = None
    if kind.startswith("pq"):
        lab, _ = _C.kmeans_assign(xt, cent, True)
        books = train_pq(xt - cent.index_select(0, lab.long()), int(kind[4:]), 64, 4, seed=4)

    def make():
        if kind.startswith("flat"):
            met = _C.Metric.L2 if kind == "flat_l2" else _C.Metric.COSINE
            ix = _C.IVFFlatIndex(d, met, nlist, 5)
            ix.set_quantizer(cent)
        else:
            ix = _C.IVFPQIndex(d, _C.Metric.L2, nlist, 5, int(kind[4:]), 64)
            ix.set_quantizer(cent, books)
        return ix

    bulk = make()
    bulk.add(xt, ids)
    stream = make()
    appends, lo = 0, 0
    for m in [1, 7, 300, 45, 2500, 2, 1200, 3000, 1, 4944]:
        cap0, n0 = stream.capacity(), stream.size()
        stream.add(xt[lo:lo + m], ids[lo:lo + m])
        lo += m
        assert stream.size() == n0 + m and stream.capacity() >= stream.size()
        appends += int(n0 > 0 and stream.capacity() == cap0)
    assert lo == len(x)
    assert appends >= 2  # some batches went into free slots without moving rows
    assert torch.equal(stream.list_offsets(), bulk.list_offsets())
    assert torch.equal(stream.list_sizes(), bulk.list_sizes())
    assert torch.equal(stream.stored_ids(), bulk.stored_ids())
    assert torch.equal(stream.stored_labels(), bulk.stored_labels())
    if kind.startswith("flat"):
        assert torch.equal(stream.stored_vectors(), bulk.stored_vectors())
    else:
        assert torch.equal(stream.stored_codes(), bulk.stored_codes())
        if stream.query_major():
            assert torch.equal(stream.stored_row_terms(), bulk.stored_row_terms())
    qt = torch.from_numpy(q).cuda()
    ds, is_ = stream.search(qt, 10)
    db, ib = bulk.search(qt, 10)
    assert torch.equal(is_, ib)
    assert torch.equal(ds, db)


def test_ivf_errors(device):
    import rapidadb._C as _C

    idx = _C.IVFFlatIndex(16, _C.Metric.L2, 8, 2)
    with pytest.raises(RuntimeError, match="not trained"):
        idx.add(torch.randn(10, 16, device=device))
    idx.set_quantizer(torch.randn(8, 16, device=device))
    idx.add(torch.randn(100, 16, device=device))
    with pytest.raises(RuntimeError, match=r"k in \[1, 32\]"):
        idx.search(torch.randn(2, 16, device=device), 33)
    with pytest.raises(RuntimeError, match="IVF-PQ supports the l2 metric"):
        _C.IVFPQIndex(16, _C.Metric.COSINE, 8, 2, 4, 16)


def test_rapidadb_ivf_train_add_search(device):
    """The drop-in facade: IVF / IVF-PQ index types train, add and search."""
    from rapidadb import IndexConfig, RapidaDB
    from rapidadb_b200.config import IndexType, Metric

    x, g = mixture(5, 10000, 32, 30)
    xt = torch.from_numpy(x).cuda()
    for it in (IndexType.IVF, IndexType.IVF_PQ):
        db = RapidaDB(config=IndexConfig(dim=32, metric=Metric.L2, index_type=it, nlist=32, nprobe=32,
                                         pq_m=16, pq_k=256, kmeans_iters=6, train_sample=5000))
        db.train(xt)
        db.add(xt)
        assert len(db) == 10000
        d, i = db.search(xt[:50], 5)
        exact = oracle.flat_search("l2", x[:50], x, 5)[1]
        # probing every list: IVF-Flat is exact; IVF-PQ (16 x 8-bit codes for
        # 32 dims) is approximate
        r = recall(i.cpu().numpy(), exact)
        assert r >= (0.999 if it == IndexType.IVF else 0.6), (it, r)
