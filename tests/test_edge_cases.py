"""Edge cases of the search paths against the oracle: empty query batches,
k equal to the table size, IVF lists holding fewer than k rows (padding),
nprobe above nlist (clamped), single queries."""
import numpy as np
import pytest
import torch

import oracle
from parity import assert_topk_match, recall

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision", ["FP32", "BF16"])
def test_flat_empty_batch_and_k_equals_n(device, precision):
    import rapidadb._C as _C

    g = np.random.default_rng(1)
    x = g.standard_normal((300, 40)).astype(np.float32)
    q = g.standard_normal((7, 40)).astype(np.float32)
    idx = _C.FlatIndex(40, _C.Metric.L2, getattr(_C.Precision, precision))
    xt = torch.from_numpy(x).cuda()
    idx.add(xt)
    d, i = idx.search(torch.empty(0, 40, device="cuda"), 5)
    assert tuple(d.shape) == (0, 5) and tuple(i.shape) == (0, 5)
    d, i = idx.search(torch.from_numpy(q).cuda(), 300)
    xs = idx.vectors().float().cpu().numpy()  # the stored (possibly rounded) rows
    qs = torch.from_numpy(q).to(idx.vectors().dtype).float().numpy()
    rd, ri = oracle.flat_search("l2", qs, xs, 300)
    assert_topk_match(rd, ri, d.cpu().numpy(), i.cpu().numpy(), rtol=1e-5, atol=1e-4)
    assert sorted(i[0].tolist()) == list(range(300))


def test_ivf_short_lists_pad_and_clamped_nprobe(device):
    import rapidadb._C as _C

    g = np.random.default_rng(2)
    x = (np.repeat(g.standard_normal((6, 16)) * 5, 4, axis=0) + 0.1 * g.standard_normal((24, 16))).astype(np.float32)
    q = x[:3] + 0.05
    cent = x[::4].copy()  # 6 lists of 4 rows
    xt = torch.from_numpy(x).cuda()
    for nprobe in (1, 50):  # 50 > nlist: every list is probed
        idx = _C.IVFFlatIndex(16, _C.Metric.L2, 6, nprobe)
        idx.set_quantizer(torch.from_numpy(cent).cuda())
        idx.add(xt)
        d, i = idx.search(torch.from_numpy(q).cuda(), 10)
        off = idx.list_offsets().cpu().numpy()
        ids = idx.stored_ids().cpu().numpy()
        rd, ri = oracle.ivf_flat_search("l2", q, cent, off, x[ids], ids, min(nprobe, 6), 10)
        np.testing.assert_array_equal(i.cpu().numpy(), ri)
        if nprobe == 1:
            # one list of 4 rows answers: the last 6 slots are padding
            assert (i[:, 4:] == -1).all() and torch.isinf(d[:, 4:]).all()


@pytest.mark.parametrize("m", [8, 2])
def test_ivfpq_single_query_and_all_lists(device, m):
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans, train_pq

    g = np.random.default_rng(3)
    x = (g.standard_normal((4000, 16)) * 2).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    cent = kmeans(xt, 8, 4, 0.0, seed=1).centroids
    lab, _ = _C.kmeans_assign(xt, cent, True)
    books = train_pq(xt - cent.index_select(0, lab.long()), m, 32, 4, seed=2)
    idx = _C.IVFPQIndex(16, _C.Metric.L2, 8, 100, m, 32)
    idx.set_quantizer(cent, books)
    idx.add(xt)
    q = x[:1] + 0.01
    d, i = idx.search(torch.from_numpy(q).cuda(), 10)
    off = idx.list_offsets().cpu().numpy()
    ids = idx.stored_ids().cpu().numpy()
    rd, ri = oracle.ivfpq_search(q, cent.cpu().numpy(), off, idx.stored_codes().cpu().numpy(), ids,
                                 books.cpu().numpy(), 8, 10)
    assert recall(i.cpu().numpy(), ri) >= 0.999
    np.testing.assert_allclose(d.cpu().numpy(), rd, rtol=1e-4, atol=1e-3)
