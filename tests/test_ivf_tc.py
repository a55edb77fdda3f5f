"""IVF-Flat search on the tensor cores (rdb_ivf_flat_search_tc).

FP32 indices with dim <= 128 and k <= 24 search on the tensor cores by
default: three fp16 products per element rank each probed list, and the best
k + 8 rows per query are scored again with the CUDA-core scan's fp32
arithmetic.  So against the CUDA-core list scan
(set_tensor_cores(False)) of the same index, scores are equal bit for bit and
ids identical except between rows whose scores are equal; against the oracle
(exact search of the probed lists) scores agree within 1e-5 relative.

Shapes cover: dim not a multiple of 64 (zero-padded K), lists longer than one
256-row tile, more than 128 probing queries on one list (several entry
chunks), empty lists, free slots between lists (streaming adds), probed lists
holding fewer than k rows (-1 padding), k = 1 and k = 24, every metric.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from parity import assert_topk_match

pytestmark = pytest.mark.gpu
LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rapidadb_b200", "librdb_kernels.so")


def overflow_counts(reset):
    """(entries rescanned exactly because their collected rows overflowed,
    probed queries that scored every centroid exactly)."""
    lib = ctypes.CDLL(LIB)
    lib.rdb_ivf_tc_overflows.argtypes = [ctypes.POINTER(ctypes.c_ulonglong), ctypes.c_int]
    v = (ctypes.c_ulonglong * 2)()
    assert lib.rdb_ivf_tc_overflows(v, 1 if reset else 0) == 0
    return v[0], v[1]


def overflows(reset):
    return overflow_counts(reset)[0]

METRICS = ["l2", "cosine", "dot_product"]


def _met(_C, metric):
    return {"l2": _C.Metric.L2, "cosine": _C.Metric.COSINE, "dot_product": _C.Metric.DOT_PRODUCT}[metric]


def mixture(seed, n, d, ncent, spread=3.0, sigma=1.0, offset=0.0):
    g = np.random.default_rng(seed)
    centres = g.standard_normal((ncent, d)).astype(np.float32) * spread
    x = centres[g.integers(0, ncent, n)] + sigma * g.standard_normal((n, d)).astype(np.float32)
    return (x + offset).astype(np.float32), g


def build(metric, x, d, nlist, nprobe, seed=1, adds=(0.35,)):
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans

    xt = torch.from_numpy(x).cuda()
    cent = kmeans(xt, nlist, 6, 0.0, seed=seed).centroids
    idx = _C.IVFFlatIndex(d, _met(_C, metric), nlist, nprobe, _C.Precision.FP32)
    idx.set_quantizer(cent)
    cuts = [0] + [int(f * len(x)) for f in adds] + [len(x)]
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        idx.add(xt[lo:hi])
    return idx, cent


def oracle_search(metric, idx, cent, x, q, nprobe, k):
    off = idx.list_offsets().cpu().numpy()
    ids = idx.stored_ids().cpu().numpy()
    return oracle.ivf_flat_search(metric, q, cent.cpu().numpy(), off, x[ids], ids, nprobe, k)


def both_paths(idx, q, k, max_overflows=0):
    qt = torch.from_numpy(q).cuda()
    assert idx.tensor_core_search(k)
    overflows(reset=True)
    d1, i1 = idx.search(qt, k)
    n_over = overflows(reset=True)
    if max_overflows is not None:
        assert n_over <= max_overflows, f"{n_over} entries overflowed their candidate buffers"
    idx.set_tensor_cores(False)
    assert not idx.tensor_core_search(k)
    d2, i2 = idx.search(qt, k)
    idx.set_tensor_cores(True)
    return d1.cpu().numpy(), i1.cpu().numpy(), d2.cpu().numpy(), i2.cpu().numpy()


@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("d", [128, 100, 32])
def test_tc_equals_cuda_core_scan_and_oracle(device, metric, d):
    x, g = mixture(3, 24000, d, 40)
    q = (x[g.integers(0, len(x), 300)] + 0.4 * g.standard_normal((300, d))).astype(np.float32)
    nlist, nprobe, k = 48, 6, 10
    idx, cent = build(metric, x, d, nlist, nprobe)
    dt, it, ds, is_ = both_paths(idx, q, k)
    # same rows, same fp32 arithmetic: equal scores; ids equal except at exact ties
    assert_topk_match(ds, is_, dt, it, rtol=0.0, atol=0.0, name=f"tc vs cuda-core {metric} d={d}")
    rd, ri = oracle_search(metric, idx, cent, x, q, nprobe, k)
    assert_topk_match(rd, ri, dt, it, rtol=1e-5, atol=1e-5, name=f"tc vs oracle {metric} d={d}")


@pytest.mark.parametrize("k", [1, 17, 24])
def test_tc_k_range_long_lists_many_probers(device, k):
    """Four lists of ~5,000 rows (20 row tiles each), 700 queries probing 2 of
    them (~350 entries per list: three 128-entry chunks)."""
    d = 64
    x, g = mixture(7, 20000, d, 4, spread=5.0)
    q = (x[g.integers(0, len(x), 700)] + 0.3 * g.standard_normal((700, d))).astype(np.float32)
    idx, cent = build("l2", x, d, 4, 2, adds=(0.5, 0.9))
    dt, it, ds, is_ = both_paths(idx, q, k)
    assert_topk_match(ds, is_, dt, it, rtol=0.0, atol=0.0, name=f"k={k}")
    rd, ri = oracle_search("l2", idx, cent, x, q, 2, k)
    assert_topk_match(rd, ri, dt, it, rtol=1e-5, atol=1e-5, name=f"k={k} oracle")


def test_tc_empty_lists_and_short_probes(device):
    """nlist = 64 centroids over data of 3 tight clusters: most lists are
    empty; with nprobe = 2 some queries probe fewer than k rows and get -1
    padding, exactly as the CUDA-core scan pads."""
    import rapidadb._C as _C

    d = 16
    g = np.random.default_rng(11)
    centres = g.standard_normal((3, d)).astype(np.float32) * 8
    x = (centres[g.integers(0, 3, 60)] + 0.1 * g.standard_normal((60, d))).astype(np.float32)
    cent = torch.from_numpy(np.concatenate([x[:40], g.standard_normal((24, d)).astype(np.float32) * 30])).cuda()
    idx = _C.IVFFlatIndex(d, _C.Metric.L2, 64, 2, _C.Precision.FP32)
    idx.set_quantizer(cent)
    idx.add(torch.from_numpy(x).cuda())
    sizes = idx.list_sizes().cpu().numpy()
    assert (sizes == 0).sum() >= 20
    q = np.concatenate([x[:10] + 0.01, g.standard_normal((5, d)).astype(np.float32) * 30])
    dt, it, ds, is_ = both_paths(idx, q, 8, max_overflows=None)
    np.testing.assert_array_equal(it, is_)
    np.testing.assert_array_equal(dt, ds)
    assert (it == -1).any()
    rd, ri = oracle_search("l2", idx, cent, x, q, 2, 8)
    np.testing.assert_array_equal(it, ri)


def test_tc_large_offset_l2(device):
    """Rows with a large common offset (|x|^2 ~ 2e4, neighbour distances ~10):
    the ranking value |x|^2 - 2 q.x cancels, the rescored top-k does not."""
    d = 48
    x, g = mixture(5, 30000, d, 30, offset=20.0)
    q = (x[g.integers(0, len(x), 80)] + 0.5 * g.standard_normal((80, d))).astype(np.float32)
    idx, cent = build("l2", x, d, 32, 6)
    dt, it, ds, is_ = both_paths(idx, q, 10)
    assert_topk_match(ds, is_, dt, it, rtol=0.0, atol=0.0, name="offset")
    rd, ri = oracle_search("l2", idx, cent, x, q, 6, 10)
    assert_topk_match(rd, ri, dt, it, rtol=1e-5, atol=1e-5, name="offset oracle")


def test_tc_duplicate_rows_tie_to_lower_row(device):
    """40 copies of one row: the best k are the copies at the lowest stored
    rows, as in the CUDA-core scan."""
    import rapidadb._C as _C

    d = 32
    g = np.random.default_rng(2)
    x = g.standard_normal((3000, d)).astype(np.float32)
    x[1000:1040] = x[5]
    cent = torch.from_numpy(x[:8].copy()).cuda()
    idx = _C.IVFFlatIndex(d, _C.Metric.DOT_PRODUCT, 8, 8, _C.Precision.FP32)
    idx.set_quantizer(cent)
    idx.add(torch.from_numpy(x).cuda())
    q = x[5:6] * 3.0
    dt, it, ds, is_ = both_paths(idx, q, 20, max_overflows=None)
    np.testing.assert_array_equal(it, is_)
    np.testing.assert_array_equal(dt, ds)


def test_tc_off_for_non_finite_rows_and_unsupported_shapes(device):
    import rapidadb._C as _C

    cent = torch.zeros((1, 16), device="cuda")
    idx = _C.IVFFlatIndex(16, _C.Metric.L2, 1, 1, _C.Precision.FP32)
    idx.set_quantizer(cent)
    x = torch.randn(100, 16, device="cuda")
    idx.add(x)
    assert idx.tensor_core_search(10) and idx.tensor_core_search(24) and not idx.tensor_core_search(25)
    bad = x[:2].clone()
    bad[0, 3] = float("inf")
    idx.add(bad)
    assert not idx.tensor_core_search(10)  # searched on CUDA cores from now on
    idx.reset()
    idx.add(x)
    assert idx.tensor_core_search(10)
    wide = _C.IVFFlatIndex(192, _C.Metric.L2, 1, 1, _C.Precision.FP32)
    wide.set_quantizer(torch.zeros((1, 192), device="cuda"))
    wide.add(torch.randn(50, 192, device="cuda"))
    assert not wide.tensor_core_search(10)  # dim > 128
    half = _C.IVFFlatIndex(16, _C.Metric.L2, 1, 1, _C.Precision.FP16)
    half.set_quantizer(cent)
    half.add(x)
    assert half.tensor_core_search(10)  # fp16 storage: the stored rows feed the MMA
    half.add(bad)
    assert not half.tensor_core_search(10)
    sq8 = _C.IVFFlatIndex(16, _C.Metric.L2, 1, 1, _C.Precision.INT8)
    sq8.set_quantizer(cent)
    sq8.add(x)
    assert not sq8.tensor_core_search(10)  # INT8 (SQ8) storage: CUDA-core scan


@pytest.mark.parametrize("precision", ["FP16", "BF16"])
@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("d", [128, 100, 32])
def test_tc_half_storage_equals_cuda_core_scan(device, precision, metric, d):
    """fp16 / bf16 rows: the MMA reads the stored rows (one exact product per
    element, K past d read as zero) and the kept rows are rescored with the
    CUDA-core scan's half-precision arithmetic: scores equal bit for bit."""
    import rapidadb._C as _C
    from rapidadb_b200.kmeans import kmeans

    x, g = mixture(12, 20000, d, 40)
    q = (x[g.integers(0, len(x), 300)] + 0.4 * g.standard_normal((300, d))).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    cent = kmeans(xt, 40, 5, 0.0, seed=3).centroids
    idx = _C.IVFFlatIndex(d, _met(_C, metric), 40, 5, getattr(_C.Precision, precision))
    idx.set_quantizer(cent)
    idx.add(xt[:7000])
    idx.add(xt[7000:])
    dt, it, ds, is_ = both_paths(idx, q, 10)
    assert_topk_match(ds, is_, dt, it, rtol=0.0, atol=0.0, name=f"{precision} {metric} d={d}")


def test_tc_restore_rebuilds_planes(device, tmp_path):
    from rapidadb import IndexConfig, Metric, RapidaDB
    from rapidadb_b200.config import IndexType

    x, g = mixture(9, 6000, 24, 12)
    q = x[:30] + 0.05
    db = RapidaDB(config=IndexConfig(dim=24, metric=Metric.COSINE, index_type=IndexType.IVF, nlist=16, nprobe=4,
                                     kmeans_iters=4))
    db.train(torch.from_numpy(x))
    db.add(torch.from_numpy(x))
    assert db.index.tensor_core_search(10)
    d1, i1 = db.search(torch.from_numpy(q), 10)
    path = tmp_path / "tc.pt"
    db.save(path)
    back = RapidaDB.load(path)
    assert back.index.tensor_core_search(10)
    d2, i2 = back.search(torch.from_numpy(q), 10)
    assert torch.equal(i1.cpu(), i2.cpu()) and torch.equal(d1.cpu(), d2.cpu())


@pytest.mark.parametrize("metric", METRICS)
def test_tc_overflow_rescans_the_list_exactly(device, metric):
    """200 copies of one row in a single list: every copy reaches the entry's
    threshold, the collected rows overflow their buffers, and the finishing
    kernel rescans that list exactly -- same answer as the CUDA-core scan."""
    import rapidadb._C as _C

    d = 40
    g = np.random.default_rng(4)
    x = g.standard_normal((3000, d)).astype(np.float32)
    x[500:700] = x[3]
    idx = _C.IVFFlatIndex(d, _met(_C, metric), 1, 1, _C.Precision.FP32)
    idx.set_quantizer(torch.from_numpy(x[:1].copy()).cuda())
    idx.add(torch.from_numpy(x).cuda())
    q = np.concatenate([x[3:4] + 0.01, g.standard_normal((5, d)).astype(np.float32)])
    qt = torch.from_numpy(q).cuda()
    overflows(reset=True)
    dt, it = idx.search(qt, 10)
    assert overflows(reset=True) >= 1
    idx.set_tensor_cores(False)
    ds, is_ = idx.search(qt, 10)
    np.testing.assert_array_equal(it.cpu().numpy(), is_.cpu().numpy())
    np.testing.assert_array_equal(dt.cpu().numpy(), ds.cpu().numpy())


@pytest.mark.parametrize("d,nlist,nprobe", [(128, 4096, 32), (100, 300, 56), (32, 64, 64), (16, 1000, 1),
                                           (64, 20000 // 7, 24), (128, 16384, 64), (96, 1500, 120)])
def test_tc_probe_equals_cuda_core_probe(device, d, nlist, nprobe):
    """The coarse probe ranks centroids on the tensor cores and rescores the
    best nprobe + 8 exactly: the same lists, in the same order, as the
    CUDA-core flat search over the centroids."""
    import rapidadb._C as _C

    x, g = mixture(8, nlist, d, max(8, nlist // 20))
    q = (x[g.integers(0, nlist, 3000)] + 0.5 * g.standard_normal((3000, d))).astype(np.float32)
    idx = _C.IVFFlatIndex(d, _C.Metric.L2, nlist, nprobe, _C.Precision.FP32)
    idx.set_quantizer(torch.from_numpy(x).cuda())
    qt = torch.from_numpy(q).cuda()
    assert idx.probe_tensor_cores(nprobe)
    overflow_counts(reset=True)
    p_tc = idx.probe(qt)
    assert overflow_counts(reset=True)[1] == 0
    idx.set_probe_tensor_cores(False)
    assert not idx.probe_tensor_cores(nprobe)
    p_cc = idx.probe(qt)
    assert torch.equal(p_tc.cpu(), p_cc.cpu())


def test_tc_probe_limits(device):
    import rapidadb._C as _C

    idx = _C.IVFFlatIndex(32, _C.Metric.L2, 200, 130, _C.Precision.FP32)
    idx.set_quantizer(torch.randn(200, 32, device="cuda"))
    assert idx.probe_tensor_cores(120) and not idx.probe_tensor_cores(121)  # nprobe + 8 <= 128
    small = _C.IVFFlatIndex(32, _C.Metric.L2, 100, 100, _C.Precision.FP32)
    small.set_quantizer(torch.randn(100, 32, device="cuda"))
    assert small.probe_tensor_cores(100)  # every list: min(nlist, nprobe + 8) <= 128
    wide = _C.IVFPQIndex(192, _C.Metric.L2, 16, 4, 8, 16)
    wide.set_quantizer(torch.randn(16, 192, device="cuda"), torch.randn(8, 16, 24, device="cuda"))
    assert not wide.probe_tensor_cores(4)  # d > 128


def test_tc_probe_equal_centroids_rescans_exactly(device):
    """300 copies of one centroid among 500: every copy reaches the probe's
    threshold, more than its buffer holds, so each query scores every
    centroid exactly -- same lists as the CUDA-core flat search (ties to the
    lower list)."""
    import rapidadb._C as _C

    d, nlist, nprobe = 48, 500, 20
    g = np.random.default_rng(21)
    c = g.standard_normal((nlist, d)).astype(np.float32) * 2
    c[100:400] = c[7]
    q = (c[7] + 0.05 * g.standard_normal((40, d))).astype(np.float32)
    idx = _C.IVFFlatIndex(d, _C.Metric.L2, nlist, nprobe, _C.Precision.FP32)
    idx.set_quantizer(torch.from_numpy(c).cuda())
    qt = torch.from_numpy(q).cuda()
    overflow_counts(reset=True)
    p_tc = idx.probe(qt)
    assert overflow_counts(reset=True)[1] == 40
    idx.set_probe_tensor_cores(False)
    p_cc = idx.probe(qt)
    assert torch.equal(p_tc.cpu(), p_cc.cpu())
