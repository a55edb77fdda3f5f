"""Flat search parity: the fused CUDA paths against the CPU oracle and the
reference's golden outputs.

fp32 rows run the CUDA-core scan, fp16 / bf16 rows the tcgen05 scan.  Half
precision is compared against the exact search over the same half-precision
values upcast to fp32 (the reference semantics for bf16 data); the tolerance
written here (1e-4 relative) is tighter than the 1e-2 the parity rule allows.
Shapes cover query counts that are not multiples of the 128-query tile, rows
that are not multiples of the 256-row tile, dimensions that are not multiples
of the 64-wide K block, k = 1, k = N, and sizes large enough for the sampled
threshold pass.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from golden import cases
from parity import assert_topk_match

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz")

TORCH_DT = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}
RTOL = {"fp32": 1e-5, "fp16": 1e-4, "bf16": 1e-4}

SHAPES = [  # (N, Q, d, k)
    (1000, 7, 64, 10),
    (5000, 130, 96, 50),
    (300, 5, 8, 300),
    (4097, 1, 200, 1),
    (20000, 33, 768, 100),
    (20000, 300, 64, 10),  # at least one query per SM: the warp-per-query selects
    (40000, 7, 64, 10),    # one query block: the fp32 sample pass split over K (2 chunks)
    (36000, 20, 300, 30),  # the same over 10 K chunks, the last one partial
    (80000, 150, 64, 100),  # sample groups of 16 rows with d <= 128; ~540 candidates per query (CTA select)
]


def _run(metric, dtype, N, Q, d, k, seed, ids=None):
    import rapidadb._C as _C

    g = np.random.default_rng(seed)
    x = g.standard_normal((N, d), dtype=np.float32)
    q = g.standard_normal((Q, d), dtype=np.float32)
    xt = torch.from_numpy(x).cuda().to(TORCH_DT[dtype])
    qt = torch.from_numpy(q).cuda().to(TORCH_DT[dtype])
    prec = {"fp32": _C.Precision.FP32, "fp16": _C.Precision.FP16, "bf16": _C.Precision.BF16}[dtype]
    met = {"l2": _C.Metric.L2, "cosine": _C.Metric.COSINE, "dot_product": _C.Metric.DOT_PRODUCT}[metric]
    idx = _C.FlatIndex(d, met, prec)
    idx.add(xt[: N // 3])
    idx.add(xt[N // 3:])
    if ids is not None:
        idx.reset()
        idx.add(xt, torch.from_numpy(ids).cuda())
    dist, ind = idx.search(qt, k)
    xr = xt.float().cpu().numpy()
    qr = qt.float().cpu().numpy()
    rd, ri = oracle.flat_search(metric, qr, xr, k, ids=ids)
    return dist.cpu().numpy(), ind.cpu().numpy(), rd, ri


@pytest.mark.parametrize("dtype", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("metric", ["l2", "cosine", "dot_product"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"N{s[0]}_Q{s[1]}_d{s[2]}_k{s[3]}" for s in SHAPES])
def test_flat_matches_oracle(device, dtype, metric, shape):
    N, Q, d, k = shape
    got_d, got_i, ref_d, ref_i = _run(metric, dtype, N, Q, d, k, seed=N + Q + d + k)
    assert_topk_match(ref_d, ref_i, got_d, got_i, rtol=RTOL[dtype], atol=1e-5,
                      name=f"{metric}/{dtype}/{shape}")


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_flat_custom_ids_oracle(device, dtype):
    N = 3000
    ids = (np.arange(N, dtype=np.int64) * 7 + 100000)[::-1].copy()
    got_d, got_i, ref_d, ref_i = _run("l2", dtype, N, 9, 40, 15, seed=5, ids=ids)
    assert_topk_match(ref_d, ref_i, got_d, got_i, rtol=RTOL[dtype], atol=1e-5)


@pytest.mark.parametrize("case", cases.FLAT_CASES, ids=[c[0] for c in cases.FLAT_CASES])
def test_flat_matches_reference_golden(device, case):
    """The product's fp32 flat search against the reference FlatIndex's own outputs."""
    import rapidadb._C as _C

    gold = np.load(GOLDEN)
    name, metric, N, Q, d, k, seed = case
    q, x = cases.flat_inputs(seed, N, Q, d)
    met = {"l2": _C.Metric.L2, "cosine": _C.Metric.COSINE, "dot_product": _C.Metric.DOT_PRODUCT}[metric]
    idx = _C.FlatIndex(d, met)
    idx.add(torch.from_numpy(x[: N // 2]).cuda())
    idx.add(torch.from_numpy(x[N // 2:]).cuda())
    dist, ids = idx.search(torch.from_numpy(q).cuda(), k)
    assert_topk_match(gold[f"{name}_d"], gold[f"{name}_i"], dist.cpu().numpy(), ids.cpu().numpy(),
                      rtol=1e-5, atol=2e-5, name=name)


def test_overflow_repair_duplicates(device):
    """All rows identical: every score ties, the sampled threshold admits every
    row, candidate lists overflow and the on-device repair must still return
    the k lowest row ids (ties go to the lower row)."""
    import rapidadb._C as _C

    N, d, k = 200000, 64, 20
    cap, rps = _plan_cap("dot_product", "bf16", 3, N, d, k)
    assert cap < rps  # every split's list overflows
    x = torch.ones(N, d, device=device, dtype=torch.bfloat16)
    idx = _C.FlatIndex(d, _C.Metric.DOT_PRODUCT, _C.Precision.BF16)
    idx.add(x)
    dist, ind = idx.search(torch.ones(3, d, device=device, dtype=torch.bfloat16), k)
    assert ind.cpu().tolist() == [list(range(k))] * 3
    assert torch.allclose(dist, torch.full_like(dist, float(d)))


def test_search_leaves_no_device_error(device):
    import rapidadb._C as _C

    idx = _C.FlatIndex(64, _C.Metric.L2, _C.Precision.BF16)
    idx.add(torch.randn(9000, 64, device=device))
    idx.search(torch.randn(200, 64, device=device), 10)
    torch.cuda.synchronize()
    assert _C.device_status(True) == 0


def _plan_cap(metric, dtype, nq, n, d, k):
    import ctypes

    lib = ctypes.CDLL(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rapidadb_b200",
                                   "librdb_kernels.so"))
    lib.rdb_flat_search_plan.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)]
    out = (ctypes.c_int64 * 7)()
    code = {"fp32": 0, "fp16": 1, "bf16": 2}[dtype]
    assert lib.rdb_flat_search_plan({"cosine": 0, "l2": 1, "dot_product": 2}[metric], code, nq, n, d, k, 0, out) == 0
    return out[3], out[4]


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("metric", ["l2", "cosine", "dot_product"])
def test_overflow_repair_only_marked_queries(device, dtype, metric):
    """A block of 6,000 identical rows equal to query 0: query 0's candidates
    overflow their list capacity and are repaired on the device, while the
    other queries (random) take the normal path in the same call.  Every
    query must equal the exact search (the repaired one returns the lowest
    rows of the tied block)."""
    import rapidadb._C as _C

    N, d, Q, k, lo, hi = 200000, 64, 40, 20, 70000, 76000
    cap, rps = _plan_cap(metric, dtype, Q, N, d, k)
    # the block covers at least one whole split, whose list overflows
    assert cap < rps and hi - lo >= 2 * rps
    g = np.random.default_rng(99)
    x = g.standard_normal((N, d), dtype=np.float32)
    v = (g.standard_normal(d).astype(np.float32) * 3.0)
    x[lo:hi] = v
    q = g.standard_normal((Q, d), dtype=np.float32)
    q[0] = v
    xt = torch.from_numpy(x).cuda().to(TORCH_DT[dtype])
    qt = torch.from_numpy(q).cuda().to(TORCH_DT[dtype])
    prec = {"fp32": _C.Precision.FP32, "bf16": _C.Precision.BF16}[dtype]
    met = {"l2": _C.Metric.L2, "cosine": _C.Metric.COSINE, "dot_product": _C.Metric.DOT_PRODUCT}[metric]
    idx = _C.FlatIndex(d, met, prec)
    idx.add(xt)
    dist, ind = idx.search(qt, k)
    rd, ri = oracle.flat_search(metric, qt.float().cpu().numpy(), xt.float().cpu().numpy(), k)
    assert_topk_match(rd, ri, dist.cpu().numpy(), ind.cpu().numpy(), rtol=RTOL[dtype], atol=1e-5,
                      name=f"repair {metric}/{dtype}")
    assert ind[0].cpu().tolist() == list(range(lo, lo + k))
    torch.cuda.synchronize()
    assert _C.device_status(True) == 0
