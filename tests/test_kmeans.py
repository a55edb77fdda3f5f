"""k-means kernels against the CPU oracle and the reference's own k-means
kernels (golden vectors D1 / D2 from csrc/kernels/kmeans.cu run on a B200)."""
import os

import numpy as np
import pytest
import torch

import oracle
from golden import cases

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")


def _C():
    from rapidadb_b200._lib import C

    return C()


@pytest.mark.parametrize("case", cases.KMEANS_CASES, ids=[c[0] for c in cases.KMEANS_CASES])
def test_exact_assign_matches_reference_kernels(device, case):
    """Sequential-FMA assignment is bit-identical to assign_clusters_kernel."""
    gold = np.load(GOLDEN)
    name, N, d, K, seed = case
    x, c0 = cases.kmeans_inputs(seed, N, d, K)
    lab, sq = _C().kmeans_assign(torch.from_numpy(x).cuda(), torch.from_numpy(c0).cuda(), True)
    np.testing.assert_array_equal(lab.cpu().numpy(), gold[f"{name}_labels"])
    # the reference stores a fast-math sqrt of the minimum
    np.testing.assert_allclose(np.sqrt(sq.cpu().numpy()), gold[f"{name}_dist"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("case", cases.KMEANS_CASES, ids=[c[0] for c in cases.KMEANS_CASES])
def test_update_matches_reference_kernels(device, case):
    gold = np.load(GOLDEN)
    name, N, d, K, seed = case
    x, c0 = cases.kmeans_inputs(seed, N, d, K)
    lab = torch.from_numpy(gold[f"{name}_labels"]).cuda()
    sums, counts = _C().kmeans_update(torch.from_numpy(x).cuda(), lab, K)
    np.testing.assert_array_equal(counts.cpu().numpy(), gold[f"{name}_counts"])
    cent = _C().kmeans_finalize(sums, counts, torch.from_numpy(c0).cuda())
    np.testing.assert_allclose(cent.cpu().numpy(), gold[f"{name}_centroids"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("d", [3, 16, 100])
def test_exact_assign_bitwise_oracle(device, d):
    g = np.random.default_rng(d)
    x = g.standard_normal((3000, d), dtype=np.float32)
    c = g.standard_normal((37, d), dtype=np.float32)
    lab, sq = _C().kmeans_assign(torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda(), True)
    rl, _, rsq = oracle.kmeans_assign(x, c)
    np.testing.assert_array_equal(lab.cpu().numpy(), rl)
    np.testing.assert_array_equal(sq.cpu().numpy(), rsq)


def test_exact_assign_past_65535_query_blocks(device):
    """2.2M points = 68,750 blocks of 32 queries: the grid continues in z."""
    g = np.random.default_rng(11)
    x = g.standard_normal((2_200_000, 8), dtype=np.float32)
    c = g.standard_normal((5, 8), dtype=np.float32)
    lab, sq = _C().kmeans_assign(torch.from_numpy(x).cuda(), torch.from_numpy(c).cuda(), True)
    rl, _, rsq = oracle.kmeans_assign(x, c)
    np.testing.assert_array_equal(lab.cpu().numpy(), rl)
    np.testing.assert_array_equal(sq.cpu().numpy(), rsq)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fast_assign_near_ties_only(device, dtype):
    """GEMM assignment may differ from the exact one only where the two
    candidate distances tie within the arithmetic's tolerance."""
    g = np.random.default_rng(1)
    x = g.standard_normal((5000, 64), dtype=np.float32)
    c = g.standard_normal((300, 64), dtype=np.float32)
    xt = torch.from_numpy(x).cuda().to(dtype)
    ct = torch.from_numpy(c).cuda().to(dtype)
    lab, sq = _C().kmeans_assign(xt, ct, False)
    xr, cr = xt.float().cpu().numpy(), ct.float().cpu().numpy()
    rl, _, rsq = oracle.kmeans_assign(xr, cr)
    lab = lab.cpu().numpy()
    rtol = 1e-5 if dtype == torch.float32 else 1e-3
    diff = np.nonzero(lab != rl)[0]
    assert len(diff) <= 0.001 * len(lab)
    for i in diff:
        got = ((xr[i] - cr[lab[i]]) ** 2).sum()
        assert got <= rsq[i] * (1 + rtol) + 1e-5
    np.testing.assert_allclose(sq.cpu().numpy(), rsq, rtol=rtol, atol=1e-3)


def test_update_empty_cluster_keeps_centroid(device):
    x = torch.randn(100, 8, device=device)
    lab = torch.zeros(100, dtype=torch.int32, device=device)  # everything in cluster 0
    cent = torch.randn(3, 8, device=device)
    sums, counts = _C().kmeans_update(x, lab, 3)
    new = _C().kmeans_finalize(sums, counts, cent)
    assert counts.cpu().tolist() == [100, 0, 0]
    assert torch.allclose(new[0], x.mean(0), atol=1e-5)
    assert torch.equal(new[1:], cent[1:])


def test_label_sort_is_stable(device):
    g = np.random.default_rng(3)
    lab = g.integers(0, 500, size=100_003).astype(np.int32)
    seg, perm, counts = _C().label_sort(torch.from_numpy(lab).cuda(), 500)
    order = np.argsort(lab, kind="stable")
    np.testing.assert_array_equal(perm.cpu().numpy(), order)
    np.testing.assert_array_equal(counts.cpu().numpy(), np.bincount(lab, minlength=500))
    np.testing.assert_array_equal(seg.cpu().numpy(), np.concatenate([[0], np.cumsum(np.bincount(lab, minlength=500))]))


def test_kmeans_matches_oracle_lloyd(device):
    """Full Lloyd iterations from the same initial centroids."""
    from rapidadb_b200.kmeans import kmeans

    g = np.random.default_rng(11)
    centres = g.standard_normal((20, 16)).astype(np.float32) * 4
    x = (centres[g.integers(0, 20, 8000)] + g.standard_normal((8000, 16))).astype(np.float32)
    init = x[:20].copy()
    res = kmeans(torch.from_numpy(x).cuda(), 20, max_iters=15, tol=0.0, init=torch.from_numpy(init).cuda(),
                 exact_assign=True)
    rc, rl, rin, rit = oracle.kmeans(x, init, 15)
    assert res.iterations == rit == 15
    np.testing.assert_allclose(res.centroids.cpu().numpy(), rc, rtol=1e-4, atol=1e-4)
    assert (res.labels.cpu().numpy() == rl).mean() >= 0.999
    assert abs(res.inertia - rin) <= 1e-4 * rin


def test_kmeans_bf16_tensor_core_quality(device):
    """bf16 assignment on the tensor cores converges to the same quality."""
    from rapidadb_b200.kmeans import kmeans

    g = np.random.default_rng(12)
    centres = g.standard_normal((64, 128)).astype(np.float32)
    x = (centres[g.integers(0, 64, 20000)] + 0.3 * g.standard_normal((20000, 128))).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    r16 = kmeans(xt.to(torch.bfloat16), 64, 10, 0.0, seed=5)
    r32 = kmeans(xt, 64, 10, 0.0, seed=5, exact_assign=True)
    assert abs(r16.inertia - r32.inertia) <= 0.02 * r32.inertia


@pytest.mark.parametrize("case", cases.LLOYD_CASES, ids=[c[0] for c in cases.LLOYD_CASES])
def test_kmeans_lloyd_matches_reference_iterations(device, case):
    """rapidadb_b200.kmeans.kmeans with the reference's assign arithmetic
    (exact_assign) against the reference's own kernels iterated the same
    number of times (golden): centroids within 1e-4, labels equal except at
    near-ties, inertia within 1e-5."""
    from lloyd import assert_lloyd_match
    from rapidadb_b200.kmeans import kmeans

    gold = np.load(GOLDEN)
    name, N, d, K, seed, iters = case
    x, c0 = cases.kmeans_inputs(seed, N, d, K)
    res = kmeans(torch.from_numpy(x).cuda(), K, max_iters=iters, tol=0.0, init=torch.from_numpy(c0).cuda(),
                 exact_assign=True)
    assert res.iterations == iters
    assert_lloyd_match(x, gold[f"{name}_centroids"], gold[f"{name}_labels"], res.centroids.cpu().numpy(),
                       res.labels.cpu().numpy(), name=name)
    ref_inertia = float((gold[f"{name}_dist"].astype(np.float64) ** 2).sum())
    assert abs(res.inertia - ref_inertia) <= 1e-5 * ref_inertia


def test_cpp_kmeans_driver_matches_oracle_lloyd(device):
    """_C.kmeans (the C++ Lloyd driver, kmeans_cuda's shape): seeded initial
    rows, exact assign, tol = 0 runs max_iters; the result unpacks as
    (centroids, labels, inertia, iterations) and matches the oracle's Lloyd
    from the same initial rows."""
    from lloyd import assert_lloyd_match
    from rapidadb_b200.utils import sample_rows

    g = np.random.default_rng(4)
    centres = g.standard_normal((24, 48)).astype(np.float32) * 3
    x = (centres[g.integers(0, 24, 5000)] + g.standard_normal((5000, 48))).astype(np.float32)
    r = _C().kmeans(torch.from_numpy(x).cuda(), 24, max_iters=7, tol=0.0, seed=11, exact=True)
    cent, labels, inertia, iters = r
    assert iters == 7 and cent.shape == (24, 48) and labels.dtype == torch.int32 and inertia.dim() == 0
    c0 = x[sample_rows(5000, 24, 11)]
    rc, rl, rin, rit = oracle.kmeans(x, c0, 7, 0.0)
    assert_lloyd_match(x, rc, rl, cent.cpu().numpy(), labels.cpu().numpy(), rtol=1e-5, name="cpp kmeans")
    assert abs(float(inertia) - rin) <= 1e-5 * rin
    # tolerance stop: converges well before 100 iterations on separated clusters
    r2 = _C().kmeans(torch.from_numpy(x).cuda(), 24)
    assert 1 <= r2.iterations < 100
    assert "KMeansResult(k=24" in repr(r2)
