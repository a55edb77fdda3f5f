"""One index row-sharded over several GPUs of one process (``IndexConfig.devices``).

The reference is single-GPU (its README.md:14 only claims multi-GPU).  With
``IndexConfig(devices=[0, 1, ...])`` a ``RapidaDB`` keeps one extension index
per listed device:

* ``add`` splits each batch into contiguous row ranges, one per device (the
  first ``n % G`` devices get one extra row), with global ids: the caller's
  ids, or ``arange(size, size + n)`` as the reference numbers rows
  (flat_index.cpp:31-34);
* ``search`` enqueues every shard's fused search from one host thread per
  device (the extension releases the GIL and returns without waiting for the
  device), gathers the per-shard ``[Q, k]`` lists on the first device and keeps
  the best k with the merge kernel (``rdb_topk_merge``);
* IVF / IVF-PQ train once (on the first device) and install the same
  quantizer on every shard.

Processes that each own one GPU use ``rapidadb_b200.sharded`` (NCCL) instead.
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor
from typing import Callable, List, Optional, Tuple

import torch

from rapidadb_b200.sharded import pad_results, shard_range


class MultiDeviceIndex:
    """Row-sharded index over ``devices``; ``make(device)`` builds one shard."""

    def __init__(self, make: Callable[[torch.device], object], devices: List[int], largest: bool):
        if not devices:
            raise ValueError("devices must list at least one CUDA device")
        self.devices = [torch.device("cuda", int(d)) for d in devices]
        self.largest = largest
        self.shards = []
        for dev in self.devices:
            with torch.cuda.device(dev):
                self.shards.append(make(dev))
        self._pool = ThreadPoolExecutor(len(self.devices)) if len(self.devices) > 1 else None

    # ------------------------------------------------------------ sizes
    def size(self) -> int:
        return sum(int(s.size()) for s in self.shards)

    def shard_sizes(self) -> List[int]:
        return [int(s.size()) for s in self.shards]

    def _map(self, fn):
        """fn(i, shard) on every shard, each on its own device and host thread."""
        def run(i):
            with torch.cuda.device(self.devices[i]):
                return fn(i, self.shards[i])

        if self._pool is None:
            return [run(0)]
        return list(self._pool.map(run, range(len(self.shards))))

    # ------------------------------------------------------------- data
    def add(self, vectors: torch.Tensor, ids: Optional[torch.Tensor] = None) -> None:
        n = vectors.shape[0]
        if ids is None:
            base = self.size()
            ids = torch.arange(base, base + n, dtype=torch.long, device=vectors.device)
        G = len(self.shards)

        def add_one(i, shard):
            lo, hi = shard_range(n, i, G)
            if hi > lo:
                dev = self.devices[i]
                shard.add(vectors[lo:hi].to(dev, non_blocking=True), ids[lo:hi].to(dev, non_blocking=True))

        self._map(add_one)

    def reset(self) -> None:
        for s in self.shards:
            s.reset()

    # ----------------------------------------------------------- search
    def search(self, queries: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        total = self.size()
        if total == 0:
            raise RuntimeError("index is empty")
        if not 1 <= k <= total:
            raise RuntimeError(f"k must be in [1, {total}]")
        dev0 = self.devices[0]
        Q = queries.shape[0]
        sizes = self.shard_sizes()

        def search_one(i, shard):
            dev = self.devices[i]
            q = queries.to(dev, non_blocking=True)
            kk = min(k, sizes[i])
            if kk == 0:
                d = torch.empty((Q, 0), dtype=torch.float32, device=dev)
                ix = torch.empty((Q, 0), dtype=torch.long, device=dev)
            else:
                d, ix = shard.search(q, kk)
            d, ix = pad_results(d, ix, k, self.largest)
            return d.to(dev0, non_blocking=True), ix.to(dev0, non_blocking=True)

        parts = self._map(search_one)
        if len(parts) == 1:
            return parts[0]
        from rapidadb_b200._lib import C

        with torch.cuda.device(dev0):
            vals = torch.stack([p[0] for p in parts])
            ids = torch.stack([p[1] for p in parts])
            return C().topk_merge(vals, ids, k, self.largest)

    # ---------------------------------------------------------- training
    def set_quantizer(self, centroids: torch.Tensor, codebooks: Optional[torch.Tensor] = None) -> None:
        for dev, s in zip(self.devices, self.shards):
            with torch.cuda.device(dev):
                if codebooks is None:
                    s.set_quantizer(centroids.to(dev))
                else:
                    s.set_quantizer(centroids.to(dev), codebooks.to(dev))

    def is_trained(self) -> bool:
        return all(bool(getattr(s, "is_trained", lambda: True)()) for s in self.shards)

    def close(self) -> None:
        if self._pool is not None:
            self._pool.shutdown(wait=True)
            self._pool = None

    def __len__(self) -> int:
        return self.size()
