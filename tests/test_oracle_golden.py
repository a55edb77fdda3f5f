"""Pin the CPU oracle to the reference itself.

``tests/golden/ref_golden.npz`` holds outputs of the unmodified reference
(its rapidadb._C extension and its two k-means kernels, built for sm_100a by
oracle/build_ref.sh and run on a B200 by tests/golden/make_golden.py).  The
inputs are regenerated from the seeds in tests/golden/cases.py.  CPU only.
"""
import os

import numpy as np
import pytest

import oracle
from golden import cases
from parity import assert_topk_match

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


@pytest.mark.parametrize("case", cases.DISTANCE_CASES, ids=[c[0] for c in cases.DISTANCE_CASES])
@pytest.mark.parametrize("metric", ["cosine", "l2", "dot_product"])
def test_distance_matches_reference(gold, case, metric):
    name, Q, N, d, seed = case
    q, x = cases.distance_inputs(seed, Q, N, d)
    got = oracle.distance(metric, q, x)
    ref = gold[f"{name}_{metric}"]
    # reference: fp32 FMA accumulation + fast-math sqrt/div; oracle: fp64
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=2e-5)


@pytest.mark.parametrize("case", cases.TOPK_CASES, ids=[c[0] for c in cases.TOPK_CASES])
def test_topk_matches_reference(gold, case):
    name, B, N, seed, ks = case
    m = cases.topk_input(seed, B, N)
    for k in ks:
        for largest in (True, False):
            v, i = oracle.topk(m, k, largest)
            rv = gold[f"{name}_k{k}_{int(largest)}_v"]
            ri = gold[f"{name}_k{k}_{int(largest)}_i"]
            np.testing.assert_array_equal(v, rv)
            np.testing.assert_array_equal(i, ri)


@pytest.mark.parametrize("case", cases.FLAT_CASES, ids=[c[0] for c in cases.FLAT_CASES])
def test_flat_search_matches_reference(gold, case):
    name, metric, N, Q, d, k, seed = case
    q, x = cases.flat_inputs(seed, N, Q, d)
    dist, ids = oracle.flat_search(metric, q, x, k)
    assert_topk_match(gold[f"{name}_d"], gold[f"{name}_i"], dist, ids, rtol=1e-5, atol=2e-5,
                      name=name)


@pytest.mark.parametrize("case", cases.KMEANS_CASES, ids=[c[0] for c in cases.KMEANS_CASES])
def test_kmeans_step_matches_reference(gold, case):
    name, N, d, K, seed = case
    x, c0 = cases.kmeans_inputs(seed, N, d, K)
    labels, dist, sq = oracle.kmeans_assign(x, c0)
    # identical arithmetic (sequential fused FMA) -> identical labels
    np.testing.assert_array_equal(labels, gold[f"{name}_labels"])
    # reference takes a fast-math sqrtf
    np.testing.assert_allclose(dist, gold[f"{name}_dist"], rtol=1e-6, atol=1e-6)
    cent, counts = oracle.kmeans_update(x, labels, c0)
    np.testing.assert_array_equal(counts, gold[f"{name}_counts"])
    # reference sums with float atomics (order varies) and a fast-math divide
    np.testing.assert_allclose(cent, gold[f"{name}_centroids"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("case", cases.LLOYD_CASES, ids=[c[0] for c in cases.LLOYD_CASES])
def test_lloyd_iterations_match_reference(gold, case):
    """Several Lloyd iterations of the oracle against the reference's own
    assign + update kernels iterated the same number of times."""
    from lloyd import assert_lloyd_match

    name, N, d, K, seed, iters = case
    x, c0 = cases.kmeans_inputs(seed, N, d, K)
    cent, labels, inertia, it = oracle.kmeans(x, c0, iters, 0.0)
    assert it == iters
    assert_lloyd_match(x, gold[f"{name}_centroids"], gold[f"{name}_labels"], cent, labels, name=name)
    ref_inertia = float((gold[f"{name}_dist"].astype(np.float64) ** 2).sum())
    assert abs(inertia - ref_inertia) <= 1e-5 * ref_inertia


def test_planted_oracle_mistake_is_caught(gold):
    """The golden check is sensitive: an oracle answer with one id swapped for
    a non-tied row must fail the comparison."""
    name, metric, N, Q, d, k, seed = cases.FLAT_CASES[1]
    q, x = cases.flat_inputs(seed, N, Q, d)
    dist, ids = oracle.flat_search(metric, q, x, k)
    bad = ids.copy()
    bad[0, 3] = ids[0, -1] + 1 if ids[0, -1] + 1 not in ids[0] else ids[0, -1] + 2
    with pytest.raises(AssertionError):
        assert_topk_match(gold[f"{name}_d"], gold[f"{name}_i"], dist, bad, name=name)
