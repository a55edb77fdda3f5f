"""Parity of the fused flat search at the sizes the benchmark runs.

* The headline table: 1,000,000 x 768 bf16 rows (i.i.d. N(0,1), L2-normalised,
  rounded to bf16), 1,024 queries of the same distribution, k = 100, cosine.
  All 1,024 queries are searched together, so the call follows the plan the
  benchmark times (tensor-core sample pass with groups of 64 sampled rows,
  CTA-pair main pass); every fourth query (256) is checked against the
  oracle's exact search (fp64 accumulation) over the same bf16 values.
* 262,144-row tables for each metric, with k chosen so that the sample pass
  keeps group maxima over 128, 64 and 32 rows (asserted from the plan the
  library reports), 300 queries (CTA pairs, a ragged last pair).

Tolerance: scores within 1e-4 relative of the exact search, ids identical
except between scores tied within that tolerance (tests/parity.py).
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from parity import assert_topk_match

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "rapidadb_b200", "librdb_kernels.so")
METRIC_CODE = {"cosine": 0, "l2": 1, "dot_product": 2}


def plan(metric, nq, n, d, k, dtype=2):
    """(sample rows, group, splits, cap, rows per split, tensor cores, chunk)."""
    lib = ctypes.CDLL(LIB)
    lib.rdb_flat_search_plan.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)]
    out = (ctypes.c_int64 * 7)()
    assert lib.rdb_flat_search_plan(METRIC_CODE[metric], dtype, nq, n, d, k, 0, out) == 0
    return list(out)


def seeded_rows(n, d, seed, normalize, device):
    """Seeded N(0,1) rows in 65,536-row chunks drawn on the device."""
    out = torch.empty((n, d), dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device)
    for c0 in range(0, n, 65536):
        c1 = min(n, c0 + 65536)
        g.manual_seed(seed * 1_000_003 + c0 // 65536)
        blk = torch.randn((c1 - c0, d), generator=g, device=device)
        if normalize:
            blk = torch.nn.functional.normalize(blk, dim=1)
        out[c0:c1] = blk.to(torch.bfloat16)
    return out


def _index(metric, x):
    import rapidadb._C as _C

    met = {"l2": _C.Metric.L2, "cosine": _C.Metric.COSINE, "dot_product": _C.Metric.DOT_PRODUCT}[metric]
    idx = _C.FlatIndex(x.shape[1], met, _C.Precision.BF16)
    idx.add(x)
    return idx


def test_headline_cosine_1m_x_768_bf16(device):
    import rapidadb._C as _C

    N, d, Q, k = 1_000_000, 768, 1024, 100
    p = plan("cosine", Q, N, d, k)
    assert p[0] == 65536 and p[1] == 64 and p[5] == 1 and p[6] == Q, p
    x = seeded_rows(N, d, 42, True, device)
    q = seeded_rows(Q, d, 7, True, device)
    idx = _index("cosine", x)
    dist, ids = idx.search(q, k)
    torch.cuda.synchronize()
    assert _C.device_status(True) == 0
    sel = np.arange(0, Q, 4)
    xr = x.float().cpu().numpy()
    qr = q[sel].float().cpu().numpy()
    rd, ri = oracle.flat_search("cosine", qr, xr, k, acc64=True)
    assert_topk_match(rd, ri, dist.cpu().numpy()[sel], ids.cpu().numpy()[sel], rtol=1e-4, atol=1e-5,
                      name="cosine 1M x 768 bf16")


@pytest.mark.parametrize("metric", ["cosine", "l2", "dot_product"])
def test_262k_rows_each_sample_group_size(device, metric):
    N, d, Q = 262_144, 384, 300
    groups = {k: plan(metric, Q, N, d, k)[1] for k in (10, 50, 100)}
    assert groups == {10: 128, 50: 64, 100: 32}, groups
    x = seeded_rows(N, d, 11, False, device)
    q = seeded_rows(Q, d, 13, False, device)
    idx = _index(metric, x)
    # the exact top-100 holds the exact top-10 and top-50 as prefixes (sorted, ties to the lower row)
    rd, ri = oracle.flat_search(metric, q.float().cpu().numpy(), x.float().cpu().numpy(), 100, acc64=True)
    for k in (10, 50, 100):
        dist, ids = idx.search(q, k)
        assert_topk_match(rd[:, :k], ri[:, :k], dist.cpu().numpy(), ids.cpu().numpy(), rtol=1e-4, atol=1e-5,
                          name=f"{metric} 262144 x {d} k={k} group {groups[k]}")
