"""Seeded inputs for the golden-vector cases.

Inputs are regenerated from their seeds (numpy's PCG64 ``default_rng`` is
bit-stable across machines), so the committed fixture ``ref_golden.npz`` only
holds the reference's outputs.  Shapes mirror the reference's own tests
(tests/python/test_kernels.py, test_flat_index.py) and the two distance-kernel
branches of csrc/kernels/distance.cu (d <= 128 and d > 128).
"""
from __future__ import annotations

import numpy as np


def randn(seed: int, n: int, d: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((n, d), dtype=np.float32)


# raw distance ops: (case, Q, N, d, seed)
DISTANCE_CASES = [
    ("A1", 4, 100, 128, 1),
    ("A2", 3, 257, 768, 2),
    ("A3", 2, 50, 64, 3),
    ("A4", 5, 33, 200, 4),
]

# top-k over a dense matrix: (case, B, N, seed, ks)
TOPK_CASES = [("B1", 6, 1000, 5, (1, 10, 100))]

# FlatIndex searches: (case, metric, N, Q, d, k, seed)
FLAT_CASES = [
    ("C1", "cosine", 500, 32, 64, 10, 42),
    ("C2", "l2", 1000, 8, 128, 10, 11),
    ("C3", "dot_product", 200, 4, 64, 10, 12),
    ("C4", "l2", 3000, 16, 768, 100, 13),
    ("C5", "cosine", 3000, 16, 768, 100, 14),
    ("C6", "cosine", 500, 4, 128, 500, 15),
    ("C7", "dot_product", 2048, 24, 256, 64, 16),
]

# k-means single Lloyd step from the first K rows: (case, N, d, K, seed)
KMEANS_CASES = [("D1", 3000, 32, 16, 7), ("D2", 2000, 128, 64, 8)]

# k-means, several Lloyd iterations from the first K rows, then one more
# assignment with the final centroids: (case, N, d, K, seed, iterations)
LLOYD_CASES = [("E1", 4000, 64, 32, 21, 5), ("E2", 3000, 128, 48, 22, 5)]


def flat_inputs(seed: int, N: int, Q: int, d: int):
    x = randn(seed, N, d)
    q = randn(seed + 1000, Q, d)
    return q, x


def distance_inputs(seed: int, Q: int, N: int, d: int):
    return randn(seed + 1000, Q, d), randn(seed, N, d)


def topk_input(seed: int, B: int, N: int):
    return randn(seed, B, N)


def kmeans_inputs(seed: int, N: int, d: int, K: int):
    x = randn(seed, N, d)
    return x, x[:K].copy()
