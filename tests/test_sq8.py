"""INT8 storage (SQ8): per-row symmetric scalar quantisation.

The reference names INT8 among its storage precisions
(csrc/include/rapidadb/core/types.h:9-14, python/rapidadb/config.py:21-26,
README.md:13) but gives it no semantics; here it is defined as per-row SQ8
(oracle.sq8_encode restates the definition) and a search over INT8 rows is
the exact search over the dequantised rows fl(scale * code) with fp32
queries.  Tolerances: codes and scales bit-identical to the oracle's;
search scores within 1e-5 relative of the oracle's exact search over the
dequantised rows, ids identical except at such ties.
"""
import numpy as np
import pytest
import torch

import oracle
from parity import assert_topk_match, recall


def test_sq8_definition_properties():
    """CPU check of the oracle's definition: codes in [-127, 127], the
    largest |code| of a nonzero row is 127, zero rows map to zeros, and the
    dequantised value is within half a step of the input."""
    g = np.random.default_rng(1)
    x = g.standard_normal((200, 37)).astype(np.float32) * g.uniform(0.01, 100, (200, 1)).astype(np.float32)
    x[5] = 0.0
    c, s = oracle.sq8_encode(x)
    assert c.dtype == np.int8 and s.dtype == np.float32
    assert np.abs(c.astype(np.int32)).max() <= 127
    nz = s > 0
    assert (np.abs(c[nz].astype(np.int32)).max(1) == 127).all()
    assert s[5] == 0 and (c[5] == 0).all()
    xd = oracle.sq8_decode(c, s)
    assert (np.abs(xd - x) <= 0.5 * s[:, None] * (1 + 1e-6) + 1e-30).all()


def _data(seed, n, d, nq):
    g = np.random.default_rng(seed)
    x = g.standard_normal((n, d)).astype(np.float32) * g.uniform(0.5, 3.0, (n, 1)).astype(np.float32)
    q = g.standard_normal((nq, d)).astype(np.float32)
    return x, q


@pytest.mark.gpu
@pytest.mark.parametrize("metric", ["l2", "cosine", "dot_product"])
@pytest.mark.parametrize("shape", [(5000, 96, 33, 10), (40000, 200, 20, 50), (3000, 37, 5, 100)],
                         ids=lambda s: "N%d_d%d_Q%d_k%d" % s)
def test_flat_int8_matches_oracle(device, metric, shape):
    import rapidadb._C as _C

    N, d, Q, k = shape
    x, q = _data(N + d, N, d, Q)
    met = {"l2": _C.Metric.L2, "cosine": _C.Metric.COSINE, "dot_product": _C.Metric.DOT_PRODUCT}[metric]
    idx = _C.FlatIndex(d, met, _C.Precision.INT8)
    idx.add(torch.from_numpy(x[: N // 3]).cuda())
    idx.add(torch.from_numpy(x[N // 3:]).cuda().to(torch.bfloat16).float())  # any float input dtype
    codes, scales = oracle.sq8_encode(np.concatenate([x[: N // 3],
                                                      torch.from_numpy(x[N // 3:]).to(torch.bfloat16).float().numpy()]))
    np.testing.assert_array_equal(idx.sq8_codes().cpu().numpy(), codes)
    np.testing.assert_array_equal(idx.sq8_scales().cpu().numpy(), scales)
    xd = oracle.sq8_decode(codes, scales)
    np.testing.assert_array_equal(idx.vectors().cpu().numpy(), xd)
    dist, ids = idx.search(torch.from_numpy(q).cuda(), k)
    rd, ri = oracle.flat_search(metric, q, xd, k)
    assert_topk_match(rd, ri, dist.cpu().numpy(), ids.cpu().numpy(), rtol=1e-5, atol=1e-5,
                      name=f"int8 {metric} {shape}")


@pytest.mark.gpu
def test_flat_int8_overflow_repair(device):
    """Identical SQ8 rows: candidate lists overflow and the on-device repair
    returns the lowest rows of the tied block (as for the other precisions)."""
    import rapidadb._C as _C

    N, d, k = 200000, 64, 20
    x = np.ones((N, d), np.float32)
    idx = _C.FlatIndex(d, _C.Metric.DOT_PRODUCT, _C.Precision.INT8)
    idx.add(torch.from_numpy(x).cuda())
    dist, ind = idx.search(torch.ones(3, d, device=device), k)
    assert ind.cpu().tolist() == [list(range(k))] * 3
    torch.cuda.synchronize()
    assert _C.device_status(True) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("metric", ["l2", "cosine"])
def test_ivf_flat_int8_matches_oracle(device, metric):
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans

    g = np.random.default_rng(7)
    centres = g.standard_normal((40, 64)).astype(np.float32) * 4
    x = (centres[g.integers(0, 40, 20000)] + g.standard_normal((20000, 64))).astype(np.float32)
    q = (x[g.integers(0, 20000, 64)] + 0.5 * g.standard_normal((64, 64))).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    cent = kmeans(xt, 64, 6, 0.0, seed=1).centroids
    met = {"l2": _C.Metric.L2, "cosine": _C.Metric.COSINE}[metric]
    idx = _C.IVFFlatIndex(64, met, 64, 8, _C.Precision.INT8)
    assert idx.sq8()
    idx.set_quantizer(cent)
    idx.add(xt[:7000])
    idx.add(xt[7000:])
    off = idx.list_offsets().cpu().numpy()
    ids = idx.stored_ids().cpu().numpy()
    codes, scales = oracle.sq8_encode(x)
    np.testing.assert_array_equal(idx.stored_sq8_codes().cpu().numpy(), codes[ids])
    np.testing.assert_array_equal(idx.stored_sq8_scales().cpu().numpy(), scales[ids])
    xd = oracle.sq8_decode(codes, scales)
    np.testing.assert_array_equal(idx.stored_vectors().cpu().numpy(), xd[ids])
    d, i = idx.search(torch.from_numpy(q).cuda(), 10)
    rd, ri = oracle.ivf_flat_search(metric, q, cent.cpu().numpy(), off, xd[ids], ids, 8, 10)
    assert recall(i.cpu().numpy(), ri) >= 0.999
    np.testing.assert_allclose(d.cpu().numpy(), rd, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("index_type", ["flat", "ivf"])
def test_int8_persistence_is_exact(device, tmp_path, index_type):
    from rapidadb import IndexConfig, Metric, RapidaDB
    from rapidadb_b200.config import IndexType, Precision

    x, q = _data(3, 12000, 48, 30)
    db = RapidaDB(config=IndexConfig(dim=48, metric=Metric.L2, precision=Precision.INT8,
                                     index_type=IndexType(index_type), nlist=32, nprobe=6, kmeans_iters=4))
    db.train(torch.from_numpy(x))
    db.add(torch.from_numpy(x))
    d1, i1 = db.search(torch.from_numpy(q), 10)
    db.save(tmp_path / "int8.pt")
    back = RapidaDB.load(tmp_path / "int8.pt")
    d2, i2 = back.search(torch.from_numpy(q), 10)
    assert torch.equal(i1.cpu(), i2.cpu()) and torch.equal(d1.cpu(), d2.cpu())
