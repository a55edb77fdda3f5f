"""pytest configuration: the ``gpu`` marker and shared fixtures.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on a
CPU-only host.  Mirrors the fixtures of the reference's tests/python/conftest.py
(device, random_vectors, small_db, small_queries), seeded here.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture
def device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    return torch.device("cuda")


@pytest.fixture
def random_vectors(device):
    import torch

    gen = torch.Generator(device="cpu").manual_seed(1234)

    def _make(n: int, dim: int = 768, normalized: bool = False):
        v = torch.randn(n, dim, generator=gen, dtype=torch.float32).to(device)
        if normalized:
            v = torch.nn.functional.normalize(v, dim=1)
        return v

    return _make


@pytest.fixture
def small_db(random_vectors):
    return random_vectors(1000, dim=128)


@pytest.fixture
def small_queries(random_vectors):
    return random_vectors(8, dim=128)
