"""k-means training (Lloyd) over the GPU kernels, optionally row-sharded.

The reference declares ``kmeans_cuda(points, k, max_iters=100, tol=1e-4,
seed=42) -> KMeansResult{centroids, labels, inertia, iterations}``
(csrc/include/rapidadb/clustering/kmeans.h:9-24) but never implements it.
The Lloyd driver is the C++ host layer's ``_C.kmeans`` (csrc/host/kmeans.cpp);
``kmeans()`` here calls it, adding the process-group all-reduce of centroid
sums and counts for sharded rows.  Each iteration is

    assign    labels, squared distances   (fused GEMM + argmin kernel)
    update    per-centroid sums, counts   (atomic-free segmented reduction)
    [all-reduce sums and counts over the process group: NCCL on GPUs]
    finalize  centroid = sum / count      (empty clusters keep their centroid)

Initialisation draws k distinct global row indices with Floyd's algorithm from
a SplitMix64 stream seeded by ``seed`` (rapidadb_b200.utils.sample_rows); with
a process group every rank contributes the initial rows it holds.
Convergence: stop after an iteration whose summed squared centroid shift is
<= tol * (sum of squared centroid norms); tol <= 0 runs max_iters iterations.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from rapidadb_b200.utils import sample_rows


@dataclass
class KMeansResult:
    centroids: torch.Tensor  # [k, d] fp32
    labels: torch.Tensor     # [n] int32 (this rank's rows)
    inertia: float           # sum of squared distances over all ranks
    iterations: int


class GpuOps:
    """The three kernel steps through the compiled extension."""

    def __init__(self, exact_assign: bool = False):
        from rapidadb_b200._lib import C

        self._C = C()
        self.exact = exact_assign

    def assign(self, x, centroids):
        return self._C.kmeans_assign(x, centroids, self.exact)

    def update(self, x, labels, k):
        return self._C.kmeans_update(x, labels, k)

    def finalize(self, sums, counts, centroids):
        return self._C.kmeans_finalize(sums, counts, centroids)


def _world(group) -> int:
    if not dist.is_available() or not dist.is_initialized():
        return 1
    return dist.get_world_size(group)


def _allreduce(t: torch.Tensor, group) -> torch.Tensor:
    if _world(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def init_centroids(x: torch.Tensor, k: int, seed: int, group=None) -> torch.Tensor:
    """Seeded random-row initialisation over the (possibly sharded) rows."""
    n_local = x.shape[0]
    world = _world(group)
    if world > 1:
        sizes = torch.tensor([n_local], dtype=torch.int64, device=x.device)
        all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
        dist.all_gather(all_sizes, sizes, group=group)
        all_sizes = [int(s.item()) for s in all_sizes]
        rank = dist.get_rank(group)
        lo = sum(all_sizes[:rank])
        n_global = sum(all_sizes)
    else:
        lo, n_global = 0, n_local
    idx = sample_rows(n_global, k, seed)
    cent = torch.zeros((k, x.shape[1]), dtype=torch.float32, device=x.device)
    sel = [(j, g - lo) for j, g in enumerate(idx) if lo <= g < lo + n_local]
    if sel:
        js = torch.tensor([a for a, _ in sel], dtype=torch.long, device=x.device)
        rs = torch.tensor([b for _, b in sel], dtype=torch.long, device=x.device)
        cent[js] = x[rs].float()
    return _allreduce(cent, group)


def kmeans(x: torch.Tensor, k: int, max_iters: int = 100, tol: float = 1e-4, seed: int = 42,
           init: Optional[torch.Tensor] = None, group=None, exact_assign: bool = False,
           ops=None) -> KMeansResult:
    """Lloyd's algorithm; ``x`` is this rank's [n, d] rows (fp32 / fp16 / bf16).

    fp16 / bf16 rows are assigned on the tensor cores; ``exact_assign`` uses
    the reference's sequential-FMA distance instead (fp32).  Runs the C++
    driver (_C.kmeans); ``ops`` (assign / update / finalize callables, e.g.
    the CPU oracle in tests) runs the same loop here instead."""
    if ops is None:
        from rapidadb_b200._lib import C

        sharded = _world(group) > 1
        if init is None and sharded:
            init = init_centroids(x, k, seed, group)

        def allreduce(a, b):
            _allreduce(a, group)
            _allreduce(b, group)

        r = C().kmeans(x, k, max_iters, tol, seed, init, exact_assign, allreduce if sharded else None)
        return KMeansResult(r.centroids, r.labels, float(r.inertia.item()), int(r.iterations))
    cent = init.float().contiguous() if init is not None else init_centroids(x, k, seed, group)
    it = 0
    for it in range(1, max_iters + 1):
        labels, _ = ops.assign(x, cent)
        sums, counts = ops.update(x, labels, k)
        _allreduce(sums, group)
        _allreduce(counts, group)
        new = ops.finalize(sums, counts, cent)
        if tol > 0:
            shift = float(((new - cent) ** 2).sum())
            norm = float((cent ** 2).sum())
            cent = new
            if shift <= tol * norm:
                break
        else:
            cent = new
    labels, sqd = ops.assign(x, cent)
    inertia = _allreduce(sqd.double().sum().reshape(1), group)
    return KMeansResult(cent, labels, float(inertia.item()), it)


def train_pq(residuals: torch.Tensor, m: int, ksub: int, iters: int, seed: int, group=None,
             ops=None) -> torch.Tensor:
    """Per-subspace codebooks [m, ksub, d / m] by k-means on residual sub-vectors."""
    d = residuals.shape[1]
    if d % m:
        raise ValueError("pq_m must divide dim")
    dsub = d // m
    books = []
    for j in range(m):
        sub = residuals[:, j * dsub:(j + 1) * dsub].float().contiguous()
        books.append(kmeans(sub, ksub, iters, 0.0, seed + 1 + j, group=group, ops=ops).centroids)
    return torch.stack(books)
