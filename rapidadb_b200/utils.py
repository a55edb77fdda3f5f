"""Helpers mirroring the reference's python/rapidadb/utils.py."""
from __future__ import annotations

import time
from contextlib import contextmanager
from typing import Optional

import torch


@contextmanager
def cuda_timer(label: str = ""):
    """Synchronised wall-clock timer (utils.py:10-26)."""
    torch.cuda.synchronize()
    start = time.perf_counter()
    yield
    torch.cuda.synchronize()
    elapsed_ms = (time.perf_counter() - start) * 1000
    if label:
        print(f"{label}: {elapsed_ms:.2f} ms")


def compute_recall(predicted: torch.Tensor, ground_truth: torch.Tensor,
                   k: Optional[int] = None) -> float:
    """Mean per-row set overlap |pred & truth| / |truth| (utils.py:29-57)."""
    if k is not None:
        predicted = predicted[:, :k]
        ground_truth = ground_truth[:, :k]
    p = predicted.cpu().tolist()
    g = ground_truth.cpu().tolist()
    total = 0.0
    for pr, gt in zip(p, g):
        gs = set(gt)
        if gs:
            total += len(set(pr) & gs) / len(gs)
    return total / max(len(p), 1)


def generate_random_vectors(n: int, dim: int, normalized: bool = False,
                            device: str = "cuda") -> torch.Tensor:
    """[n, dim] float32 N(0, 1) vectors, optionally L2-normalised (utils.py:60-80)."""
    v = torch.randn(n, dim, device=device, dtype=torch.float32)
    if normalized:
        v = torch.nn.functional.normalize(v, dim=1)
    return v


def splitmix64(seed: int):
    """Deterministic 64-bit generator (SplitMix64, Steele et al. 2014) used for
    seeded initialisation so host code and tests draw the same sequence."""
    state = seed & 0xFFFFFFFFFFFFFFFF
    while True:
        state = (state + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
        z = state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        yield z ^ (z >> 31)


def sample_rows(n: int, k: int, seed: int) -> list:
    """k distinct row indices of [0, n) drawn with Floyd's algorithm from a
    SplitMix64 stream (seeded random-row initialisation of k-means)."""
    if k > n:
        raise ValueError(f"cannot sample {k} rows from {n}")
    rng = splitmix64(seed)
    chosen = {}
    order = []
    for j in range(n - k, n):
        t = next(rng) % (j + 1)
        pick = t if t not in chosen else j
        chosen[pick] = True
        order.append(pick)
    return order
