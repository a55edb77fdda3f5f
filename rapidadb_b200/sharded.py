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


def exchange_owned(local_d: torch.Tensor, local_i: torch.Tensor,
                   group: Optional[dist.ProcessGroup] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Owner exchange of [Q, k] lists: query slice r (shard_range(Q, r,
    world), contiguous rows) of every rank goes to rank r, which receives
    [G, Q_r, k] scores and ids -- 1 / G of an all-gather's bytes, no packing
    copies (one all-to-all for the scores, one for the ids)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    Q, k = local_d.shape
    sizes = [(b - a) * k for a, b in (shard_range(Q, r, world) for r in range(world))]
    n_r = sizes[rank] // k if k else 0
    vals = torch.empty(world * sizes[rank], dtype=local_d.dtype, device=local_d.device)
    ids = torch.empty(world * sizes[rank], dtype=local_i.dtype, device=local_i.device)
    dist.all_to_all_single(vals, local_d.contiguous().view(-1), [sizes[rank]] * world, sizes, group=group)
    dist.all_to_all_single(ids, local_i.contiguous().view(-1), [sizes[rank]] * world, sizes, group=group)
    return vals.view(world, n_r, k), ids.view(world, n_r, k)


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
        results:      "replicated" -- every rank returns the [Q, k] answer of
                      the whole batch (one all-gather of the per-rank lists);
                      "owner" -- rank r returns the answer of its query slice
                      owned_range(Q) only (an all-to-all carrying 1 / G of
                      the bytes, and a merge of 1 / G of the queries), the
                      shared threshold likewise selected per slice.
    """

    def __init__(self, index, largest: bool, group: Optional[dist.ProcessGroup] = None,
                 merge: Optional[Callable] = None, shared_threshold: bool = True, results: str = "replicated"):
        if results not in ("replicated", "owner"):
            raise ValueError(f"results must be 'replicated' or 'owner', got {results!r}")
        self.search_fn = index if callable(index) and not hasattr(index, "search") else index.search
        self.largest = largest
        self.group = group
        self.merge = merge or gpu_merge
        self.results = results
        # the extension FlatIndex (directly or inside a RapidaDB facade) with
        # fp16 / bf16 rows can share one sampled threshold across the shards
        flat = getattr(index, "index", index)
        self.flat = flat if shared_threshold and hasattr(flat, "sample_maxima") and flat.tensor_core() else None
        self._sizes = None

    def owned_range(self, Q: int) -> Tuple[int, int]:
        """Queries [lo, hi) of a Q-query batch whose answers this rank
        returns ([0, Q) unless results="owner" on more than one rank)."""
        if self.results != "owner" or not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return 0, Q
        return shard_range(Q, dist.get_rank(self.group), dist.get_world_size(self.group))

    def refresh_sizes(self) -> None:
        """Forget the cached shard sizes (call on every rank after adds or
        resets); the next search gathers them again."""
        self._sizes = None

    def _shared_threshold_search(self, queries: torch.Tensor, k: int):
        """Shared-threshold protocol: every rank computes group maxima of a
        strided sample of its rows (1 / world of the single-GPU sample); the
        k-th best of all ranks' maxima of a query -- a lower bound on its
        global k-th best score -- filters every shard.  results="replicated"
        all-gathers the maxima and every rank selects every query's threshold;
        results="owner" sends each rank the maxima of its query slice
        (all-to-all), selects those thresholds there and all-gathers them.
        The shard sizes are gathered on the first search.  None (before any
        data collective) when the shards are too small."""
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
        from rapidadb_b200._lib import C

        if self.results == "owner":
            # each rank selects the thresholds of its query slice from every
            # rank's maxima, then the thresholds are all-gathered
            lo, hi = self.owned_range(Q)
            sizes = [(b - a) * gl for a, b in (shard_range(Q, r, world) for r in range(world))]
            recv = torch.empty(world * (hi - lo) * gl, dtype=maxima.dtype, device=dev)
            dist.all_to_all_single(recv, maxima.contiguous().view(-1), [(hi - lo) * gl] * world, sizes,
                                   group=self.group)
            mine = recv.view(world, hi - lo, gl).permute(1, 0, 2).reshape(hi - lo, world * gl)
            cap = -(-Q // world)  # slices differ by at most one query: pad to the largest
            thr_mine = torch.zeros(cap, dtype=maxima.dtype, device=dev)
            if hi > lo:
                thr_mine[: hi - lo] = C().select_threshold(mine, k, self.largest)
            allt = torch.empty(world * cap, dtype=maxima.dtype, device=dev)
            dist.all_gather_into_tensor(allt, thr_mine, group=self.group)
            if Q % world == 0:
                thr = allt
            else:
                allt = allt.view(world, cap)
                thr = torch.cat([allt[r, : b - a] for r, (a, b) in enumerate(shard_range(Q, r, world)
                                                                              for r in range(world))])
        else:
            allm = torch.empty((world * Q, gl), dtype=maxima.dtype, device=dev)
            dist.all_gather_into_tensor(allm, maxima.contiguous(), group=self.group)
            allm = allm.view(world, Q, gl).permute(1, 0, 2).reshape(Q, world * gl)
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
        if self.results == "owner":
            vals, ids = exchange_owned(local_d, local_i, self.group)
        else:
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
    and merged as in ShardedSearch (results="owner": each rank merges and
    returns only its query slice, owned_range(Q), after an all-to-all)."""

    def __init__(self, index, largest: bool, group: Optional[dist.ProcessGroup] = None,
                 merge: Optional[Callable] = None, results: str = "replicated"):
        if results not in ("replicated", "owner"):
            raise ValueError(f"results must be 'replicated' or 'owner', got {results!r}")
        self.index = index
        self.largest = largest
        self.group = group
        self.merge = merge or gpu_merge
        self.results = results

    def owned_range(self, Q: int) -> Tuple[int, int]:
        """Queries [lo, hi) of a Q-query batch whose answers this rank returns."""
        if self.results != "owner" or not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return 0, Q
        return shard_range(Q, dist.get_rank(self.group), dist.get_world_size(self.group))

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
        if self.results == "owner":
            vals, ids = exchange_owned(local_d, local_i, self.group)
        else:
            vals, ids = gather_candidates(local_d, local_i, self.group)
        return self.merge(vals, ids, k, self.largest)
