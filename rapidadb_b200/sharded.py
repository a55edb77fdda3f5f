"""Row-sharded search over one process per GPU (torch.distributed).

The reference is single-GPU (its README.md:14 only claims multi-GPU).  Here
the database is split by rows across the ranks of a process group: every rank
holds a contiguous slice with global ids, answers the same query batch with its
local fused search, the per-rank [Q, k] candidate lists are exchanged with ONE
all-gather (NCCL over NVLink on GPUs, gloo on CPU in tests), and a final merge
kernel keeps the best k per query.  k-means centroid sums are reduced with an
all-reduce (see rapidadb_b200.kmeans).

``local_search`` and ``merge`` are injectable so the exchange logic can be
exercised on CPU ranks with the oracle standing in for the GPU parts.
"""
from __future__ import annotations

import math
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous rows [lo, hi) of rank `rank` when n rows are split evenly
    (the first n % world ranks get one extra row)."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def gather_candidates(local_d: torch.Tensor, local_i: torch.Tensor,
                      group: Optional[dist.ProcessGroup] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather [Q, k] fp32 scores and int64 ids from every rank with one
    collective.  Rank r's block of the gather buffer is [Q k scores | Q k ids]
    (32-bit words, the id block 8-byte aligned); the returned [G, Q, k] score
    and id tensors are views of the blocks (no copies), which the merge reads
    in place."""
    world = dist.get_world_size(group)
    Q, k = local_d.shape
    nv = Q * k + (Q * k) % 2  # score words, padded so the ids stay 8-byte aligned
    words = nv + 2 * Q * k
    send = torch.empty(words, dtype=torch.int32, device=local_d.device)
    send[:Q * k].view(torch.float32).copy_(local_d.reshape(-1))
    send[nv:].view(torch.int64).copy_(local_i.reshape(-1))
    out = torch.empty((world, words), dtype=torch.int32, device=local_d.device)
    dist.all_gather_into_tensor(out.view(-1), send, group=group)
    vals = out[:, :Q * k].view(torch.float32).view(world, Q, k)
    ids = out[:, nv:].view(torch.int64).view(world, Q, k)
    return vals, ids


def gpu_merge(vals: torch.Tensor, ids: torch.Tensor, k: int, largest: bool):
    from rapidadb_b200._lib import C

    return C().topk_merge(vals, ids, k, largest)


def shared_sample_plan(sizes, k: int) -> Optional[Tuple[int, int, int]]:
    """Sample plan of the shared-threshold protocol for shard sizes `sizes`:
    (rows sampled per rank, rows per group maximum, total sampled rows), or
    None when the shards are too small for a useful sample.  The total sample
    S follows the single-GPU rule (a power of two near 6 sqrt(n k), at most
    n / 4 rows, groups of up to 128 rows while >= 10 k groups remain), spread
    evenly over the ranks."""
    world, n = len(sizes), int(sum(sizes))
    S, sd = 1024, 6.0 * math.sqrt(n * k)
    while S < sd and S < 131072:
        S <<= 1
    while S > 1024 and 4 * S > n:
        S >>= 1
    while S < 8 * k:
        S <<= 1
    g = 1
    while g < 128 and S // (2 * g) >= 10 * k:
        g <<= 1
    per = (S // world) // g * g
    if per < g or 4 * per > min(sizes) or world * (per // g) < 4 * k:
        return None
    return per, g, world * per


class ShardedSearch:
    """Search one query batch against a row-sharded index.

    Args:
        index:        this rank's index object (anything with .search(q, k)
                      returning (scores [Q, k], global ids [Q, k])), or a
                      callable (q, k) -> (scores, ids).
        largest:      True for cosine / dot (descending), False for L2.
        group:        process group (default: the world).
        merge:        (vals [G,Q,k], ids [G,Q,k], k, largest) -> (vals, ids);
                      defaults to the GPU merge kernel.
    """

    def __init__(self, index, largest: bool, group: Optional[dist.ProcessGroup] = None,
                 merge: Optional[Callable] = None, shared_threshold: bool = True):
        self.search_fn = index if callable(index) and not hasattr(index, "search") else index.search
        self.largest = largest
        self.group = group
        self.merge = merge or gpu_merge
        # the extension FlatIndex (directly or inside a RapidaDB facade) with
        # fp16 / bf16 rows can share one sampled threshold across the shards
        flat = getattr(index, "index", index)
        self.flat = flat if shared_threshold and hasattr(flat, "sample_maxima") and flat.tensor_core() else None
        self._sizes = None

    def refresh_sizes(self) -> None:
        """Forget the cached shard sizes (call on every rank after adds or
        resets); the next search gathers them again."""
        self._sizes = None

    def _shared_threshold_search(self, queries: torch.Tensor, k: int):
        """Shared-threshold protocol: every rank computes group maxima of a
        strided sample of its rows (1 / world of the single-GPU sample), the
        maxima are all-gathered, the k-th best of them -- a lower bound on the
        global k-th best score -- filters every shard.  One collective per
        search (the maxima) besides the result gather; the shard sizes are
        gathered on the first search.  None (before any data collective) when
        the shards are too small."""
        world = dist.get_world_size(self.group)
        dev = queries.device
        if self._sizes is None:
            # shard sizes, gathered once (refresh_sizes() after the index changes)
            n_local = torch.tensor([self.flat.size()], dtype=torch.long, device=dev)
            sizes = torch.empty(world, dtype=torch.long, device=dev)
            dist.all_gather_into_tensor(sizes, n_local, group=self.group)
            self._sizes = sizes.tolist()
        if self._sizes[dist.get_rank(self.group)] != self.flat.size():
            raise RuntimeError("shard size changed since the sizes were gathered: call refresh_sizes() on every rank")
        plan = shared_sample_plan(self._sizes, k)
        if plan is None:
            return None
        per, g, total = plan
        maxima = self.flat.sample_maxima(queries, per, g)  # [Q, per / g]
        Q, gl = maxima.shape
        allm = torch.empty((world * Q, gl), dtype=maxima.dtype, device=dev)
        dist.all_gather_into_tensor(allm, maxima.contiguous(), group=self.group)
        allm = allm.view(world, Q, gl).permute(1, 0, 2).reshape(Q, world * gl)
        from rapidadb_b200._lib import C

        thr = C().select_threshold(allm, k, self.largest)
        expect = int(math.ceil(1.1 * self.flat.size() * k / total)) + 1
        return self.flat.search_threshold(queries, k, thr, expect)

    def search(self, queries: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return self.search_fn(queries, k)
        out = None
        if self.flat is not None:
            out = self._shared_threshold_search(queries, k)
        local_d, local_i = out if out is not None else self.search_fn(queries, k)
        vals, ids = gather_candidates(local_d, local_i, self.group)
        return self.merge(vals, ids, k, self.largest)


class ShardedIVFSearch:
    """Search a row-sharded IVF / IVF-PQ index (every rank holds the same
    trained quantizer and a slice of the rows).

    The coarse probe is split across ranks -- rank r probes its contiguous
    slice of the query batch -- and the [Q, nprobe] list table is
    all-gathered, so the replicated probe costs each GPU 1/G of the batch.
    Every rank then scans its rows of the probed lists for all queries
    (``index.search_probed``), and the per-rank [Q, k] lists are all-gathered
    and merged as in ShardedSearch."""

    def __init__(self, index, largest: bool, group: Optional[dist.ProcessGroup] = None,
                 merge: Optional[Callable] = None):
        self.index = index
        self.largest = largest
        self.group = group
        self.merge = merge or gpu_merge

    def probe(self, queries: torch.Tensor) -> torch.Tensor:
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return self.index.probe(queries)
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        Q = queries.shape[0]
        chunk = (Q + world - 1) // world
        lo, hi = min(rank * chunk, Q), min((rank + 1) * chunk, Q)
        local = self.index.probe(queries[lo:hi]) if hi > lo else None
        np_ = local.shape[1] if local is not None else self.index.probe(queries[:1]).shape[1]
        buf = torch.zeros((chunk, np_), dtype=torch.long, device=queries.device)
        if local is not None:
            buf[: hi - lo] = local
        out = torch.empty((world * chunk, np_), dtype=torch.long, device=queries.device)
        dist.all_gather_into_tensor(out, buf, group=self.group)
        return out[:Q]

    def search(self, queries: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        probe = self.probe(queries)
        local_d, local_i = self.index.search_probed(queries, probe, k)
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return local_d, local_i
        vals, ids = gather_candidates(local_d, local_i, self.group)
        return self.merge(vals, ids, k, self.largest)
