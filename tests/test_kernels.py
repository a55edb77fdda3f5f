"""Raw-op tests mirroring the reference's tests/python/test_kernels.py, plus
parity of the product's raw ops against the reference's own golden outputs."""
import os

import numpy as np
import pytest
import torch

from golden import cases

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")


class TestCosineKernel:
    def test_basic_correctness(self, device, random_vectors):
        import rapidadb._C as _C

        queries = random_vectors(4, dim=128)
        database = random_vectors(100, dim=128)
        result = _C.cosine_similarity(queries, database)
        q_norm = torch.nn.functional.normalize(queries, dim=1)
        d_norm = torch.nn.functional.normalize(database, dim=1)
        expected = q_norm @ d_norm.T
        assert result.shape == (4, 100)
        assert torch.allclose(result, expected, rtol=1e-3, atol=1e-5), \
            f"Max diff: {(result - expected).abs().max().item()}"

    def test_single_query(self, device, random_vectors):
        import rapidadb._C as _C

        result = _C.cosine_similarity(random_vectors(1, dim=64), random_vectors(50, dim=64))
        assert result.shape == (1, 50)

    def test_identical_vectors(self, device):
        import rapidadb._C as _C

        v = torch.randn(1, 256, device=device)
        result = _C.cosine_similarity(v, v.repeat(10, 1))
        assert torch.allclose(result, torch.ones_like(result), atol=1e-4)

    def test_orthogonal_vectors(self, device):
        import rapidadb._C as _C

        q = torch.zeros(1, 4, device=device)
        q[0, 0] = 1.0
        db = torch.zeros(1, 4, device=device)
        db[0, 1] = 1.0
        assert _C.cosine_similarity(q, db).abs().item() < 1e-5

    def test_large_dim(self, device, random_vectors):
        import rapidadb._C as _C

        result = _C.cosine_similarity(random_vectors(2, dim=768), random_vectors(500, dim=768))
        assert result.shape == (2, 500)
        assert result.min() >= -1.1 and result.max() <= 1.1


class TestL2Kernel:
    def test_basic_correctness(self, device, random_vectors):
        import rapidadb._C as _C

        queries = random_vectors(4, dim=128)
        database = random_vectors(100, dim=128)
        result = _C.l2_distance(queries, database)
        expected = torch.cdist(queries, database, p=2).pow(2)
        assert result.shape == (4, 100)
        assert torch.allclose(result, expected, rtol=1e-3, atol=1e-4)

    def test_self_distance_zero(self, device):
        import rapidadb._C as _C

        v = torch.randn(1, 64, device=device)
        assert _C.l2_distance(v, v).item() < 1e-5

    def test_non_negative(self, device, random_vectors):
        import rapidadb._C as _C

        result = _C.l2_distance(random_vectors(8, dim=128), random_vectors(200, dim=128))
        assert (result >= -1e-6).all()


class TestDotProductKernel:
    def test_basic_correctness(self, device, random_vectors):
        import rapidadb._C as _C

        queries = random_vectors(4, dim=128)
        database = random_vectors(100, dim=128)
        result = _C.dot_product(queries, database)
        assert result.shape == (4, 100)
        assert torch.allclose(result, queries @ database.T, rtol=1e-3, atol=1e-4)


class TestKernelEdgeCases:
    def test_dimension_mismatch_raises(self, device):
        import rapidadb._C as _C

        with pytest.raises(RuntimeError, match="dimension mismatch"):
            _C.cosine_similarity(torch.randn(1, 64, device=device), torch.randn(10, 128, device=device))

    def test_cpu_tensor_raises(self):
        import rapidadb._C as _C

        with pytest.raises(RuntimeError, match="CUDA"):
            _C.cosine_similarity(torch.randn(1, 64), torch.randn(10, 64))

    def test_1d_tensor_raises(self, device):
        import rapidadb._C as _C

        with pytest.raises(RuntimeError):
            _C.cosine_similarity(torch.randn(64, device=device), torch.randn(10, 64, device=device))


# ---------------------------------------------------------------- golden parity


@pytest.mark.parametrize("case", cases.DISTANCE_CASES, ids=[c[0] for c in cases.DISTANCE_CASES])
@pytest.mark.parametrize("metric", ["cosine", "l2", "dot_product"])
def test_distance_matches_reference_golden(device, case, metric):
    import rapidadb._C as _C

    gold = np.load(GOLDEN)
    name, Q, N, d, seed = case
    q, x = cases.distance_inputs(seed, Q, N, d)
    fn = {"cosine": _C.cosine_similarity, "l2": _C.l2_distance, "dot_product": _C.dot_product}[metric]
    got = fn(torch.from_numpy(q).to(device), torch.from_numpy(x).to(device)).cpu().numpy()
    # both sides sum d fp32 products in different orders: the absolute error
    # scales with sum |q_i x_i| (~d), not with the (possibly tiny) result
    atol = 2e-5 if metric == "cosine" else 2e-7 * d
    np.testing.assert_allclose(got, gold[f"{name}_{metric}"], rtol=1e-5, atol=atol)


@pytest.mark.parametrize("case", cases.TOPK_CASES, ids=[c[0] for c in cases.TOPK_CASES])
def test_topk_matches_reference_golden(device, case):
    import rapidadb._C as _C

    gold = np.load(GOLDEN)
    name, B, N, seed, ks = case
    m = torch.from_numpy(cases.topk_input(seed, B, N)).to(device)
    for k in ks:
        for largest in (True, False):
            for fn in (_C.topk, _C.topk_thrust):
                v, i = fn(m, k, largest)
                np.testing.assert_array_equal(v.cpu().numpy(), gold[f"{name}_k{k}_{int(largest)}_v"])
                np.testing.assert_array_equal(i.cpu().numpy(), gold[f"{name}_k{k}_{int(largest)}_i"])


def test_topk_warp_heap_contract(device):
    import rapidadb._C as _C

    m = torch.randn(3, 500, device=device)
    v, i = _C.topk_warp_heap(m, 128, True)
    assert v.shape == (3, 128)
    with pytest.raises(RuntimeError, match="warp heap"):
        _C.topk_warp_heap(m, 129, True)


def test_dense_distance_bf16_fp16(device):
    """Raw ops accept half-precision inputs (computed in fp32 on the upcast values)."""
    import rapidadb._C as _C
    import oracle

    q = torch.randn(5, 96, device=device).to(torch.bfloat16)
    x = torch.randn(70, 96, device=device).to(torch.bfloat16)
    for metric, fn in (("l2", _C.l2_distance), ("cosine", _C.cosine_similarity), ("dot_product", _C.dot_product)):
        got = fn(q, x).cpu().numpy()
        ref = oracle.distance(metric, q.float().cpu().numpy(), x.float().cpu().numpy())
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=2e-5)
