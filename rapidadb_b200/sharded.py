"""Row-sharded search over one process per GPU (torch.distributed).

The reference is single-GPU (its README.md:14 only claims multi-GPU).  Here
the database is split by rows across the ranks of a process group: every rank
holds a contiguous slice with global ids, answers the same query batch with its
local fused search, the per-rank [Q, k] candidate lists are exchanged (GPU
ranks of one node: one exchange kernel reading the other ranks' memory over
NVLink, PeerExchange; otherwise one all-gather or all-to-all, NCCL or gloo),
and a final merge kernel keeps the best k per query.  k-means centroid sums
are reduced with an all-reduce (see rapidadb_b200.kmeans).

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


class BufferPool:
    """Device buffers kept across searches, one per (name, shape, dtype,
    device).  The tensors a search hands to NCCL are reused instead of
    allocated every search: the caching allocator cannot hand out a block that
    a collective still holds, so a host running several searches ahead of the
    GPU would otherwise grow the pool with new device allocations.  Reuse is in
    stream order: every collective here is issued blocking (the current stream
    waits for it), so a later search's writes follow the earlier reads.  One
    buffer is kept per distinct shape; nothing returned to a caller aliases
    them."""

    def __init__(self):
        self._bufs = {}

    def get(self, name: str, shape, dtype, device) -> torch.Tensor:
        key = (name, tuple(int(v) for v in shape), dtype, str(device))
        t = self._bufs.get(key)
        if t is None:
            t = torch.empty(key[1], dtype=dtype, device=device)
            self._bufs[key] = t
        return t


def pack_lists(local_d: torch.Tensor, local_i: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[Q, k] fp32 scores and int64 ids -> one [Q, W] int32 block, W = 3k
    rounded up to even: row q holds k score words, a pad word when k is odd
    (keeping the ids 8-byte aligned), then the 2k words of the ids.  One
    collective then carries both, and unpack_lists() reads them in place."""
    Q, k = local_d.shape
    parts = [local_d.contiguous().view(torch.int32)]
    if k % 2:
        parts.append(torch.zeros((Q, 1), dtype=torch.int32, device=local_d.device))
    parts.append(local_i.contiguous().view(torch.int32))
    if out is None:
        return torch.cat(parts, dim=1)
    return torch.cat(parts, dim=1, out=out)


def unpack_lists(buf: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """[..., W] packed rows -> strided views: scores [..., k] fp32, ids [..., k] int64."""
    off = k + (k % 2)
    return buf[..., :k].view(torch.float32), buf[..., off:off + 2 * k].view(torch.int64)


def _packed_width(k: int) -> int:
    return 3 * k + (k % 2)


def gather_candidates(local_d: torch.Tensor, local_i: torch.Tensor,
                      group: Optional[dist.ProcessGroup] = None,
                      pool: Optional[BufferPool] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather every rank's [Q, k] scores and ids with ONE collective of
    packed rows (pack_lists); returns [G, Q, k] score and id views of the
    receive buffer, which the merge reads in place."""
    world = dist.get_world_size(group)
    Q, k = local_d.shape
    dev = local_d.device
    W = _packed_width(k)
    send = pack_lists(local_d, local_i, pool.get("send", (Q, W), torch.int32, dev) if pool else None)
    out = (pool.get("gather", (world, Q, W), torch.int32, dev) if pool
           else torch.empty((world, Q, W), dtype=torch.int32, device=dev))
    dist.all_gather_into_tensor(out.view(-1), send.view(-1), group=group)
    return unpack_lists(out, k)


def exchange_owned(local_d: torch.Tensor, local_i: torch.Tensor,
                   group: Optional[dist.ProcessGroup] = None,
                   pool: Optional[BufferPool] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Owner exchange of [Q, k] lists: query slice r (shard_range(Q, r,
    world), contiguous rows) of every rank goes to rank r, which receives
    [G, Q_r, k] scores and ids -- 1 / G of an all-gather's bytes, in ONE
    all-to-all of packed rows (pack_lists), read in place by the merge."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    Q, k = local_d.shape
    dev = local_d.device
    W = _packed_width(k)
    send = pack_lists(local_d, local_i, pool.get("send", (Q, W), torch.int32, dev) if pool else None)
    sizes = [(b - a) * W for a, b in (shard_range(Q, r, world) for r in range(world))]
    n_r = sizes[rank] // W
    recv = (pool.get("owned", (world, n_r, W), torch.int32, dev) if pool
            else torch.empty((world, n_r, W), dtype=torch.int32, device=dev))
    dist.all_to_all_single(recv.view(-1), send.view(-1), [sizes[rank]] * world, sizes, group=group)
    return unpack_lists(recv, k)


class PeerUnavailable(RuntimeError):
    """The ranks cannot map each other's memory (not one node, no peer access)."""


class _DeviceSpan:
    """Raw device memory handed to torch.as_tensor (zero copy)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """NVLink transport of ShardedSearch for ranks on one node: every rank
    owns one exchange arena (device memory shared with the other processes as
    a CUDA IPC handle and mapped into each of them), and every exchange is ONE
    kernel (rdb_peer_gather) that signals this rank's rows ready, waits for
    the other ranks (bounded: a wait that runs out sets a device status bit
    and copies nothing) and reads the rows it needs straight out of their
    arenas with peer loads.  No collective library runs on the data path.

    Every search is one epoch; the flags hold epochs, so nothing is reset
    between searches.  Setup, growth and close() are collective (every rank
    calls them in the same order); if any rank cannot map the others'
    arenas, every rank raises PeerUnavailable."""

    FLAG_BYTES = 512  # RDB_PEER_FLAG_BYTES
    MAX_RANKS = 8     # RDB_PEER_MAX_RANKS
    SLOT_MAXIMA, SLOT_THRESHOLD, SLOT_LISTS, SLOT_PROBE = 0, 1, 2, 3
    STATUS_TIMEOUT = 1 << 6  # device status bit of a wait that ran out

    def __init__(self, group: Optional[dist.ProcessGroup], device, limit_ns: int = 2_000_000_000):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if self.world > self.MAX_RANKS:
            raise PeerUnavailable(f"at most {self.MAX_RANKS} ranks")
        self.limit_ns = int(limit_ns)
        self.nbytes = 0
        self.ptr = None
        self.bases = []
        self.buf = None
        self.epoch = 0
        self._off = {}

    def _all_ok(self, ok: bool) -> bool:
        t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.group)
        return bool(t.item())

    def reserve(self, sections: dict) -> None:
        """Lays out the named sections ({name: bytes}, the same on every rank)
        after the flags, 256-byte aligned; a layout that does not fit the
        arena grows it first (collective)."""
        off, layout = self.FLAG_BYTES, {}
        for name, n in sections.items():
            layout[name] = off
            off += (int(n) + 255) // 256 * 256
        if off > self.nbytes:
            self._map(max(off, 2 * self.nbytes))
        self._off = layout

    def _map(self, nbytes: int) -> None:
        from rapidadb_b200._lib import C

        dev = self.device.index
        if self.ptr is not None:
            self._release()
        ok, ptr, handle = True, None, bytes(64)
        try:
            ptr, handle = C().peer_arena_alloc(dev, nbytes)
        except RuntimeError:
            ok = False
        h = torch.tensor(list(handle), dtype=torch.uint8, device=self.device)
        allh = torch.empty((self.world, 64), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allh, h, group=self.group)
        allh = allh.cpu()
        bases = []
        if ok:
            try:
                for p in range(self.world):
                    bases.append(ptr if p == self.rank else C().peer_arena_open(dev, bytes(allh[p].tolist())))
            except RuntimeError:
                ok = False
        if not self._all_ok(ok):
            for p, b in enumerate(bases):
                if p != self.rank:
                    C().peer_arena_close(dev, b)
            if ptr is not None:
                C().peer_arena_free(dev, ptr)
            raise PeerUnavailable("the ranks cannot map each other's exchange arenas")
        self.ptr, self.bases, self.nbytes = ptr, bases, nbytes
        self.buf = torch.as_tensor(_DeviceSpan(ptr, nbytes), device=self.device)

    def _release(self) -> None:
        from rapidadb_b200._lib import C

        dev = self.device.index
        # no rank may still read an arena: finish local work, then agree
        torch.cuda.synchronize(self.device)
        self._all_ok(True)
        for p, b in enumerate(self.bases):
            if p != self.rank:
                C().peer_arena_close(dev, b)
        torch.cuda.synchronize(self.device)
        self._all_ok(True)
        C().peer_arena_free(dev, self.ptr)
        self.ptr, self.bases, self.buf, self.nbytes, self._off = None, [], None, 0, {}

    def close(self) -> None:
        """Unmaps and frees the arenas (collective)."""
        if self.ptr is not None:
            self._release()

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def view(self, section: str, shape, dtype) -> torch.Tensor:
        """This rank's section as a tensor of `shape` (contiguous)."""
        n = math.prod(shape) * dtype.itemsize
        off = self._off[section]
        return self.buf[off: off + n].view(dtype).view(tuple(shape))

    def gather(self, slot: int, section: str, epoch: int, *, row0, nrows, row_bytes: int, src_row_stride: int,
               dst: torch.Tensor, dst_off, dst_row_stride: int) -> None:
        """Rows row0[p] .. row0[p] + nrows[p] - 1 of `section` of every rank
        p's arena -> dst (bytes dst_off[p] + i * dst_row_stride), one kernel
        on the current stream after this rank's own section is written."""
        from rapidadb_b200._lib import C

        C().peer_gather(self.rank, slot, epoch, self.bases, self.nbytes, self._off[section], src_row_stride, row_bytes,
                        [int(v) for v in row0], [int(v) for v in nrows], dst, [int(v) for v in dst_off],
                        dst_row_stride, self.limit_ns)


class PhaseClock:
    """CUDA events recorded on the current stream at the phase boundaries of
    every search while ``enabled`` (CUDA queries only); ``summary()`` gives
    the mean device time of each phase per search and clears the log."""

    def __init__(self):
        self.enabled = False
        self._log = []
        self._cur = None

    def start(self, queries: torch.Tensor) -> None:
        self._cur = None
        if self.enabled and queries.is_cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._cur = [("start", e)]

    def mark(self, name: str) -> None:
        if self._cur is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._cur.append((name, e))

    def end(self) -> None:
        if self._cur is not None:
            self._log.append(self._cur)
        self._cur = None

    def summary(self) -> dict:
        tot, n = {}, len(self._log)
        for marks in self._log:
            marks[-1][1].synchronize()
            for (_, a), (name, b) in zip(marks, marks[1:]):
                tot[name] = tot.get(name, 0.0) + a.elapsed_time(b)
        self._log = []
        return {name: round(v / max(n, 1), 4) for name, v in tot.items()}


def gpu_merge(vals: torch.Tensor, ids: torch.Tensor, k: int, largest: bool):
    from rapidadb_b200._lib import C

    return C().topk_merge(vals, ids, k, largest)


def _rows_of(obj) -> Optional[int]:
    """Stored rows of an index object (``size`` attribute or method), or None."""
    s = getattr(obj, "size", None)
    if s is None:
        return None
    return int(s() if callable(s) else s)


def pad_results(d: torch.Tensor, i: torch.Tensor, k: int, largest: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """[Q, k'] lists (k' <= k) padded to [Q, k] with the worst score (-inf
    for cosine / dot, +inf for L2) and id -1, which a merge ranks last."""
    Q, kk = d.shape
    if kk == k:
        return d, i
    pd = torch.full((Q, k), -math.inf if largest else math.inf, dtype=d.dtype, device=d.device)
    pi = torch.full((Q, k), -1, dtype=i.dtype, device=i.device)
    pd[:, :kk] = d
    pi[:, :kk] = i
    return pd, pi


class _ShardSizes:
    """Shard sizes of every rank, gathered once (one all-gather of one int64
    per rank, on every rank's first search) and checked against k before any
    data collective, so a request that some shard cannot serve is answered
    the same way on every rank instead of raising on one rank and leaving
    the others blocked in a collective."""

    def _init_sizes(self, local_size):
        self._local_size = local_size
        self._sizes = None

    def _local_rows(self) -> Optional[int]:
        ls = self._local_size
        if ls is not None:
            return int(ls() if callable(ls) else ls)
        return _rows_of(self._size_source)

    def refresh_sizes(self) -> None:
        """Forget the cached shard sizes (call on every rank after adds or
        resets); the next search gathers them again."""
        self._sizes = None

    def shard_sizes(self, device) -> Optional[list]:
        """Every rank's stored rows (None when this rank's index does not
        report a size); collective on the first call after refresh_sizes()."""
        n_local = self._local_rows()
        if n_local is None:
            return None
        if self._sizes is None:
            world = dist.get_world_size(self.group)
            t = torch.tensor([n_local], dtype=torch.long, device=device)
            sizes = torch.empty(world, dtype=torch.long, device=device)
            dist.all_gather_into_tensor(sizes, t, group=self.group)
            self._sizes = sizes.tolist()
        if self._sizes[dist.get_rank(self.group)] != n_local:
            raise RuntimeError("shard size changed since the sizes were gathered: call refresh_sizes() on every rank")
        return self._sizes

    def _check_k(self, sizes, k: int) -> None:
        if sizes is not None and not 1 <= k <= sum(sizes):
            raise ValueError(f"k must be in [1, {sum(sizes)}] (rows stored over all shards)")

    def _padded(self, search, sizes, k: int, empty_shape):
        """search(k') on this rank's shard with k' = min(k, its rows), padded
        to k; an empty shard returns only padding."""
        if sizes is None:
            return search(k)
        n_local = sizes[dist.get_rank(self.group)]
        if n_local >= k:
            return search(k)
        Q, dev = empty_shape
        if n_local == 0:
            d = torch.empty((Q, 0), dtype=torch.float32, device=dev)
            i = torch.empty((Q, 0), dtype=torch.long, device=dev)
        else:
            d, i = search(n_local)
        return pad_results(d, i, k, self.largest)


class _PeerTransport:
    """Transport of the sharded searches' exchanges: the peer exchange
    kernel over NVLink (PeerExchange) or torch.distributed collectives."""

    def _init_transport(self, transport: str) -> None:
        if transport not in ("auto", "collective", "peer"):
            raise ValueError(f"transport must be 'auto', 'collective' or 'peer', got {transport!r}")
        self.transport = transport
        self.peer: Optional[PeerExchange] = None
        self._peer_off = transport == "collective"

    def _peer_exchange(self, device) -> Optional[PeerExchange]:
        """The peer transport (set up on the first search, collectively), or
        None for collectives.  Raises when an exchange wait on this device
        has run out since the status was last cleared (another rank fell
        behind by more than the limit or left): the results of the searches
        since then are not valid."""
        if self._peer_off:
            return None
        if self.peer is not None:
            from rapidadb_b200._lib import C

            if C().pending_status() & PeerExchange.STATUS_TIMEOUT:
                raise RuntimeError("a peer exchange wait on this device ran out (another rank fell behind or "
                                   "left); results since then are not valid. Read and clear the status with "
                                   "device_status(True) on every rank")
        if self.peer is None:
            usable = (device.type == "cuda" and "nccl" in str(dist.get_backend(self.group))
                      and dist.get_world_size(self.group) <= PeerExchange.MAX_RANKS)
            try:
                if not usable:
                    raise PeerUnavailable("the peer transport needs CUDA ranks under the NCCL backend, "
                                          f"at most {PeerExchange.MAX_RANKS}")
                ex = PeerExchange(self.group, device)
                ex.reserve({})
                self.peer = ex
            except PeerUnavailable:
                if self.transport == "peer":
                    raise
                self._peer_off = True
                return None
        return self.peer

    def close(self) -> None:
        """Frees the peer transport's arenas (collective: every rank calls it)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _exchange_lists(self, local_d, local_i, ex=None, epoch=0):
        """This rank's [Q, k] lists -> [G, Q_r, k] score and id views of the
        lists it merges (its query slice under results="owner", else all
        queries)."""
        if ex is None:
            if self.results == "owner":
                return exchange_owned(local_d, local_i, self.group, self.pool)
            return gather_candidates(local_d, local_i, self.group, self.pool)
        world = dist.get_world_size(self.group)
        Q, k = local_d.shape
        W = _packed_width(k)
        # two list sections by epoch parity: with no threshold exchange
        # between two searches, a rank may pack the next lists while another
        # still reads these
        name = "lists%d" % (epoch & 1)
        pack_lists(local_d, local_i, ex.view(name, (Q, W), torch.int32))
        lo, hi = self.owned_range(Q)
        recv = self.pool.get("peer_lists", (world, hi - lo, W), torch.int32, local_d.device)
        ex.gather(PeerExchange.SLOT_LISTS, name, epoch, row0=[lo] * world, nrows=[hi - lo] * world,
                  row_bytes=4 * W, src_row_stride=4 * W, dst=recv,
                  dst_off=[4 * W * (hi - lo) * p for p in range(world)], dst_row_stride=4 * W)
        return unpack_lists(recv, k)


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


class ShardedSearch(_ShardSizes, _PeerTransport):
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
        local_size:   this rank's stored rows (int or callable); by default
                      the index's ``size``.  With it, a shard holding fewer
                      than k rows (or none) contributes a padded list, and k
                      above the rows of all shards raises ValueError on every
                      rank before any data collective.
        transport:    "auto" -- the peer transport (PeerExchange: one
                      exchange kernel over NVLink per exchange, no
                      collective library on the data path) when the ranks
                      are CUDA ranks of one node under the NCCL backend,
                      else collectives; "collective" -- torch.distributed
                      collectives (NCCL / gloo); "peer" -- the peer
                      transport or an error.
    """

    def __init__(self, index, largest: bool, group: Optional[dist.ProcessGroup] = None,
                 merge: Optional[Callable] = None, shared_threshold: bool = True, results: str = "replicated",
                 local_size=None, transport: str = "auto"):
        if results not in ("replicated", "owner"):
            raise ValueError(f"results must be 'replicated' or 'owner', got {results!r}")
        self._init_transport(transport)
        self._size_source = index
        self._init_sizes(local_size)
        self.clock = PhaseClock()
        self.search_fn = index if callable(index) and not hasattr(index, "search") else index.search
        self.largest = largest
        self.group = group
        self.merge = merge or gpu_merge
        self.results = results
        self.pool = BufferPool()
        # the extension FlatIndex (directly or inside a RapidaDB facade) with
        # fp16 / bf16 rows can share one sampled threshold across the shards
        flat = getattr(index, "index", index)
        self.flat = flat if shared_threshold and hasattr(flat, "sample_maxima") and flat.tensor_core() else None

    def owned_range(self, Q: int) -> Tuple[int, int]:
        """Queries [lo, hi) of a Q-query batch whose answers this rank
        returns ([0, Q) unless results="owner" on more than one rank)."""
        if self.results != "owner" or not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return 0, Q
        return shard_range(Q, dist.get_rank(self.group), dist.get_world_size(self.group))

    def _shared_threshold_search(self, queries: torch.Tensor, k: int, sizes, plan, ex=None, epoch=0):
        """Shared-threshold protocol: every rank computes group maxima of a
        strided sample of its rows (1 / world of the single-GPU sample); the
        k-th best of all ranks' maxima of a query -- a lower bound on its
        global k-th best score -- filters every shard.  results="replicated"
        brings every rank every rank's maxima and every rank selects every
        query's threshold; results="owner" brings each rank the maxima of its
        query slice, selects those thresholds there and shares them.  With
        the peer transport (ex) the maxima and thresholds move through the
        exchange arenas (one exchange kernel each), else through an
        all-to-all / all-gather."""
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        dev = queries.device
        per, g, total = plan
        Q, gl = queries.shape[0], per // g
        # [Q, gl] group maxima, written straight into the exchange arena
        maxima = self.flat.sample_maxima(queries, per, g, **(
            {"out": ex.view("maxima", (Q, gl), torch.float32)} if ex is not None else {}))
        self.clock.mark("sample")
        from rapidadb_b200._lib import C

        if ex is not None:
            lo, hi = self.owned_range(Q)
            mine = self.pool.get("peer_maxima", (hi - lo, world * gl), maxima.dtype, dev)
            ex.gather(PeerExchange.SLOT_MAXIMA, "maxima", epoch, row0=[lo] * world, nrows=[hi - lo] * world,
                      row_bytes=4 * gl, src_row_stride=4 * gl, dst=mine,
                      dst_off=[4 * gl * p for p in range(world)], dst_row_stride=4 * gl * world)
            thr = ex.view("thr", (Q,), maxima.dtype)
            if hi > lo:
                C().select_threshold(mine, k, self.largest, out=thr[lo:hi])
            if self.results == "owner":
                # every rank's slice of thresholds into this rank's array (its own already in place)
                sl = [shard_range(Q, p, world) for p in range(world)]
                ex.gather(PeerExchange.SLOT_THRESHOLD, "thr", epoch, row0=[a for a, _ in sl],
                          nrows=[0 if p == rank else b - a for p, (a, b) in enumerate(sl)], row_bytes=4,
                          src_row_stride=4, dst=thr, dst_off=[4 * a for a, _ in sl], dst_row_stride=4)
        elif self.results == "owner":
            # each rank selects the thresholds of its query slice from every
            # rank's maxima, then the thresholds are all-gathered
            lo, hi = self.owned_range(Q)
            sizes = [(b - a) * gl for a, b in (shard_range(Q, r, world) for r in range(world))]
            recv = self.pool.get("maxima", (world * (hi - lo) * gl,), maxima.dtype, dev)
            dist.all_to_all_single(recv, maxima.contiguous().view(-1), [(hi - lo) * gl] * world, sizes,
                                   group=self.group)
            mine = recv.view(world, hi - lo, gl).permute(1, 0, 2).reshape(hi - lo, world * gl)
            cap = -(-Q // world)  # slices differ by at most one query: pad to the largest
            thr_mine = self.pool.get("thr_mine", (cap,), maxima.dtype, dev)  # rows past hi - lo: padding
            if hi > lo:
                thr_mine[: hi - lo] = C().select_threshold(mine, k, self.largest)
            allt = self.pool.get("thr_all", (world * cap,), maxima.dtype, dev)
            dist.all_gather_into_tensor(allt, thr_mine, group=self.group)
            if Q % world == 0:
                thr = allt
            else:
                allt = allt.view(world, cap)
                thr = torch.cat([allt[r, : b - a] for r, (a, b) in enumerate(shard_range(Q, r, world)
                                                                              for r in range(world))])
        else:
            allm = self.pool.get("maxima_all", (world * Q, gl), maxima.dtype, dev)
            dist.all_gather_into_tensor(allm, maxima.contiguous(), group=self.group)
            allm = allm.view(world, Q, gl).permute(1, 0, 2).reshape(Q, world * gl)
            thr = C().select_threshold(allm, k, self.largest)
        self.clock.mark("threshold_exchange")
        expect = int(math.ceil(1.1 * self.flat.size() * k / total)) + 1
        return self.flat.search_threshold(queries, k, thr, expect)

    def search(self, queries: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return self.search_fn(queries, k)
        sizes = self.shard_sizes(queries.device)
        self._check_k(sizes, k)
        Q = queries.shape[0]
        plan = None
        if self.flat is not None and sizes is not None and min(sizes) >= k:
            plan = shared_sample_plan(sizes, k)
        ex = self._peer_exchange(queries.device)
        epoch = 0
        if ex is not None:
            gl = plan[0] // plan[1] if plan is not None else 0
            W4 = 4 * Q * _packed_width(k)
            ex.reserve({"maxima": 4 * Q * gl, "thr": 4 * Q, "lists0": W4, "lists1": W4})
            epoch = ex.next_epoch()
        self.clock.start(queries)
        out = None
        if plan is not None:
            out = self._shared_threshold_search(queries, k, sizes, plan, ex, epoch)
        if out is None:
            out = self._padded(lambda kk: self.search_fn(queries, kk), sizes, k,
                               (queries.shape[0], queries.device))
        local_d, local_i = out
        self.clock.mark("scan")
        vals, ids = self._exchange_lists(local_d, local_i, ex, epoch)
        self.clock.mark("result_exchange")
        res = self.merge(vals, ids, k, self.largest)
        self.clock.mark("merge")
        self.clock.end()
        return res


class ShardedIVFSearch(_ShardSizes, _PeerTransport):
    """Search a row-sharded IVF / IVF-PQ index (every rank holds the same
    trained quantizer and a slice of the rows).

    The coarse probe is split across ranks -- rank r probes its contiguous
    slice of the query batch -- and the [Q, nprobe] list table is shared,
    so the replicated probe costs each GPU 1/G of the batch.  Every rank
    then scans its rows of the probed lists for all queries
    (``index.search_probed``), and the per-rank [Q, k] lists are exchanged
    and merged as in ShardedSearch (results="owner": each rank merges and
    returns only its query slice, owned_range(Q)).  Both exchanges go
    through the peer exchange kernel or collectives (``transport`` as in
    ShardedSearch).  Shards with fewer than k rows contribute padded lists
    (``local_size`` as in ShardedSearch)."""

    def __init__(self, index, largest: bool, group: Optional[dist.ProcessGroup] = None,
                 merge: Optional[Callable] = None, results: str = "replicated", local_size=None,
                 transport: str = "auto"):
        if results not in ("replicated", "owner"):
            raise ValueError(f"results must be 'replicated' or 'owner', got {results!r}")
        self._init_transport(transport)
        self._size_source = index
        self._init_sizes(local_size)
        self.clock = PhaseClock()
        self.index = index
        self.largest = largest
        self.group = group
        self.merge = merge or gpu_merge
        self.results = results
        self.pool = BufferPool()

    def owned_range(self, Q: int) -> Tuple[int, int]:
        """Queries [lo, hi) of a Q-query batch whose answers this rank returns."""
        if self.results != "owner" or not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return 0, Q
        return shard_range(Q, dist.get_rank(self.group), dist.get_world_size(self.group))

    def _probe_slice(self, queries: torch.Tensor):
        """This rank's slice of the coarse probe: (slices of every rank,
        its [hi - lo, nprobe] lists or None, nprobe)."""
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        Q = queries.shape[0]
        chunk = (Q + world - 1) // world
        sl = [(min(p * chunk, Q), min((p + 1) * chunk, Q)) for p in range(world)]
        lo, hi = sl[rank]
        local = self.index.probe(queries[lo:hi]) if hi > lo else None
        np_ = local.shape[1] if local is not None else self.index.probe(queries[:1]).shape[1]
        return sl, local, np_

    def probe(self, queries: torch.Tensor) -> torch.Tensor:
        """The [Q, nprobe] list table of the batch (collective over the
        ranks; each probes its slice), as a new tensor."""
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return self.index.probe(queries)
        world = dist.get_world_size(self.group)
        Q = queries.shape[0]
        sl, local, np_ = self._probe_slice(queries)
        chunk = (Q + world - 1) // world
        buf = self.pool.get("probe_mine", (chunk, np_), torch.long, queries.device)  # rows past hi - lo: padding
        if local is not None:
            buf[: local.shape[0]] = local
        out = self.pool.get("probe_all", (world * chunk, np_), torch.long, queries.device)
        dist.all_gather_into_tensor(out, buf, group=self.group)
        return out[:Q].clone()  # the caller may keep it; the pooled buffer is reused by the next probe

    def _probe_peer(self, queries: torch.Tensor, k: int, ex: PeerExchange) -> Tuple[torch.Tensor, int]:
        """The list table through the exchange arenas: this rank's slice in
        place, every other rank's slice read from its arena by one exchange
        kernel.  Returns the table (a view of this rank's arena, valid until
        the next search) and the search's epoch."""
        rank = dist.get_rank(self.group)
        Q = queries.shape[0]
        sl, local, np_ = self._probe_slice(queries)
        W4 = 4 * Q * _packed_width(k)
        ex.reserve({"probe": 8 * Q * np_, "lists0": W4, "lists1": W4})
        epoch = ex.next_epoch()
        table = ex.view("probe", (Q, np_), torch.long)
        lo, hi = sl[rank]
        if local is not None:
            table[lo:hi] = local
        ex.gather(PeerExchange.SLOT_PROBE, "probe", epoch, row0=[a for a, _ in sl],
                  nrows=[0 if p == rank else b - a for p, (a, b) in enumerate(sl)], row_bytes=8 * np_,
                  src_row_stride=8 * np_, dst=table, dst_off=[8 * np_ * a for a, _ in sl], dst_row_stride=8 * np_)
        return table, epoch

    def search(self, queries: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return self.index.search_probed(queries, self.probe(queries), k)
        sizes = self.shard_sizes(queries.device)
        self._check_k(sizes, k)
        ex = self._peer_exchange(queries.device)
        self.clock.start(queries)
        epoch = 0
        if ex is not None:
            probe, epoch = self._probe_peer(queries, k, ex)
        else:
            probe = self.probe(queries)
        self.clock.mark("probe")
        local_d, local_i = self._padded(lambda kk: self.index.search_probed(queries, probe, kk), sizes, k,
                                        (queries.shape[0], queries.device))
        self.clock.mark("scan")
        vals, ids = self._exchange_lists(local_d, local_i, ex, epoch)
        self.clock.mark("result_exchange")
        res = self.merge(vals, ids, k, self.largest)
        self.clock.mark("merge")
        self.clock.end()
        return res
