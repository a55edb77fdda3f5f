"""Shared-threshold sharded flat search emulated in one process: shards'
sample maxima are concatenated, the k-th best of them filters every shard,
and the merged per-shard answers must equal the unsharded search."""
import numpy as np
import pytest
import torch

from parity import assert_topk_match

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("metric,k,world", [("COSINE", 20, 2), ("L2", 10, 3), ("DOT_PRODUCT", 50, 4)])
def test_shared_threshold_equals_single(device, metric, k, world):
    import rapidadb._C as _C
    from rapidadb_b200.sharded import shard_range, shared_sample_plan

    g = np.random.default_rng(7)
    n, d, nq = 60000, 96, 300
    x = torch.from_numpy(g.standard_normal((n, d), dtype=np.float32)).cuda().to(torch.bfloat16)
    q = torch.from_numpy(g.standard_normal((nq, d), dtype=np.float32)).cuda().to(torch.bfloat16)
    m = getattr(_C.Metric, metric)
    largest = metric != "L2"
    full = _C.FlatIndex(d, m, _C.Precision.BF16)
    full.add(x)
    rd, ri = full.search(q, k)

    shards = []
    for r in range(world):
        lo, hi = shard_range(n, r, world)
        ix = _C.FlatIndex(d, m, _C.Precision.BF16)
        ix.add(x[lo:hi], torch.arange(lo, hi, device=x.device))
        shards.append(ix)
    per, grp, total = shared_sample_plan([ix.size() for ix in shards], k)
    maxima = torch.cat([ix.sample_maxima(q, per, grp) for ix in shards], dim=1)
    assert maxima.shape == (nq, world * per // grp)
    thr = _C.select_threshold(maxima, k, largest)
    # the threshold never beats the true k-th best score
    kth = rd[:, k - 1]
    tol = 1e-2 * kth.abs() + 1e-3
    assert bool(((thr <= kth + tol) if largest else (thr >= kth - tol)).all())
    outs = [ix.search_threshold(q, k, thr, int(1.1 * ix.size() * k / total) + 1) for ix in shards]
    vals = torch.stack([o[0] for o in outs])
    ids = torch.stack([o[1] for o in outs])
    md, mi = _C.topk_merge(vals, ids, k, largest)
    assert_topk_match(rd.cpu().numpy(), ri.cpu().numpy(), md.cpu().numpy(), mi.cpu().numpy(), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("largest", [True, False])
@pytest.mark.parametrize("k", [13, 10])
def test_merge_reads_packed_exchange_rows_in_place(device, largest, k):
    """The merge reads per-rank lists straight out of a packed exchange
    buffer (sharded.pack_lists: per row k score words, a pad word when k is
    odd, 2k id words), through the row strides, without copies."""
    import oracle
    import rapidadb._C as _C
    from rapidadb_b200.sharded import pack_lists, unpack_lists

    g = np.random.default_rng(3)
    G, Q = 5, 77
    v = np.sort(g.standard_normal((G, Q, k)).astype(np.float32), axis=2)
    if largest:
        v = v[:, :, ::-1].copy()
    ids = g.permutation(G * Q * k).astype(np.int64).reshape(G, Q, k)
    buf = torch.stack([pack_lists(torch.from_numpy(v[r]).cuda(), torch.from_numpy(ids[r]).cuda())
                       for r in range(G)])
    assert buf.shape == (G, Q, 3 * k + k % 2)
    vals, idv = unpack_lists(buf, k)
    assert not vals.is_contiguous() and not idv.is_contiguous()
    assert vals.data_ptr() == buf.data_ptr()
    md, mi = _C.topk_merge(vals, idv, k, largest)
    rd, ri = oracle.topk_merge(v, ids, k, largest)
    np.testing.assert_array_equal(md.cpu().numpy(), rd)
    np.testing.assert_array_equal(mi.cpu().numpy(), ri)
