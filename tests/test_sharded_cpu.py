"""Row-sharded search and sharded k-means, exercised on CPU gloo ranks.

The multi-GPU path is one process per GPU: local fused search -> all-gather
of the per-rank [Q, k] lists -> merge; k-means all-reduces centroid sums and
counts.  Here two gloo ranks run the same host logic with the CPU oracle
standing in for the GPU kernels, and the result must equal the single-process
oracle answer.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from rapidadb_b200.sharded import ShardedSearch, shard_range
from rapidadb_b200.utils import sample_rows


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_merge(vals, ids, k, largest):
    v, i = oracle.topk_merge(vals.numpy(), ids.numpy(), k, largest)
    return torch.from_numpy(v), torch.from_numpy(i)


class OracleOps:
    """k-means steps on the CPU oracle (same contract as rapidadb_b200.kmeans.GpuOps)."""

    def assign(self, x, c):
        lab, _, sq = oracle.kmeans_assign(x.numpy(), c.numpy())
        return torch.from_numpy(lab), torch.from_numpy(sq)

    def update(self, x, labels, k):
        xs = x.numpy().astype(np.float64)
        lab = labels.numpy()
        sums = np.zeros((k, x.shape[1]), np.float64)
        np.add.at(sums, lab, xs)
        return torch.from_numpy(sums.astype(np.float32)), torch.from_numpy(np.bincount(lab, minlength=k).astype(np.int64))

    def finalize(self, sums, counts, c):
        out = c.clone()
        nz = counts > 0
        out[nz] = sums[nz] / counts[nz].unsqueeze(1).float()
        return out


def _worker(rank, world, port, fn, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, fn(rank, world)))
    finally:
        dist.destroy_process_group()


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def _data():
    g = np.random.default_rng(0)
    return g.standard_normal((3001, 24), dtype=np.float32), g.standard_normal((17, 24), dtype=np.float32)


def _sharded_search(rank, world):
    x, q = _data()
    lo, hi = shard_range(len(x), rank, world)

    def local(qt, k):
        d, i = oracle.flat_search("l2", qt.numpy(), x[lo:hi], k, ids=np.arange(lo, hi, dtype=np.int64))
        return torch.from_numpy(d), torch.from_numpy(i)

    d, i = ShardedSearch(local, largest=False, merge=_oracle_merge).search(torch.from_numpy(q), 10)
    return d.numpy(), i.numpy()


def test_sharded_flat_search_equals_single_process():
    out = _run(_sharded_search)
    x, q = _data()
    rd, ri = oracle.flat_search("l2", q, x, 10)
    for r in (0, 1):
        np.testing.assert_array_equal(out[r][1], ri)
        np.testing.assert_allclose(out[r][0], rd, rtol=1e-6)


def _owner_search(rank, world):
    x, q = _data()
    lo, hi = shard_range(len(x), rank, world)

    def local(qt, k):
        d, i = oracle.flat_search("l2", qt.numpy(), x[lo:hi], k, ids=np.arange(lo, hi, dtype=np.int64))
        return torch.from_numpy(d), torch.from_numpy(i)

    s = ShardedSearch(local, largest=False, merge=_oracle_merge, results="owner")
    d, i = s.search(torch.from_numpy(q), 10)
    return s.owned_range(len(q)), d.numpy(), i.numpy()


@pytest.mark.parametrize("world", [2, 3])
def test_owner_results_cover_the_batch_once(world):
    """results="owner": rank r returns the merged answers of its query slice
    (17 queries: uneven slices); together they equal the single-process
    answer, each query once."""
    out = _run(_owner_search, world)
    x, q = _data()
    rd, ri = oracle.flat_search("l2", q, x, 10)
    ranges = [out[r][0] for r in range(world)]
    assert ranges == [shard_range(len(q), r, world) for r in range(world)]
    for r in range(world):
        a, b = ranges[r]
        np.testing.assert_array_equal(out[r][2], ri[a:b])
        np.testing.assert_allclose(out[r][1], rd[a:b], rtol=1e-6)


class _OracleIVFShard:
    """One rank's slice of an IVF-Flat index on the CPU oracle: the coarse
    probe is the oracle's exact L2 search over the centroids, the list scan
    an exact search over the slice's rows whose list is probed."""

    def __init__(self, x, labels, lo, hi, cent, nprobe):
        self.x, self.labels, self.lo, self.hi = x, labels, lo, hi
        self.cent, self.nprobe = cent, nprobe

    def probe(self, qt):
        _, i = oracle.flat_search("l2", qt.numpy(), self.cent, self.nprobe)
        return torch.from_numpy(i)

    def size(self):
        return self.hi - self.lo

    def search_probed(self, qt, probe, k):
        # the GPU index rejects k above its stored rows (ivf_index.cpp check_query)
        assert 1 <= k <= self.size(), f"k={k} on a shard of {self.size()} rows"
        q = qt.numpy()
        out_d = np.full((len(q), k), np.inf, np.float32)
        out_i = np.full((len(q), k), -1, np.int64)
        lab = self.labels[self.lo:self.hi]
        for j in range(len(q)):
            rows = np.nonzero(np.isin(lab, probe[j].numpy()))[0]
            if len(rows) == 0:
                continue
            kk = min(k, len(rows))
            d, i = oracle.flat_search("l2", q[j:j + 1], self.x[self.lo + rows], kk,
                                      ids=(self.lo + rows).astype(np.int64))
            out_d[j, :kk], out_i[j, :kk] = d[0], i[0]
        return torch.from_numpy(out_d), torch.from_numpy(out_i)


def _ivf_setup():
    x, q = _data()
    cent = x[:20].copy()
    labels = oracle.kmeans_assign(x, cent)[0]
    return x, q, cent, labels


def _sharded_ivf(rank, world, results):
    from rapidadb_b200.sharded import ShardedIVFSearch

    x, q, cent, labels = _ivf_setup()
    lo, hi = shard_range(len(x), rank, world)
    s = ShardedIVFSearch(_OracleIVFShard(x, labels, lo, hi, cent, 4), largest=False, merge=_oracle_merge,
                         results=results)
    d, i = s.search(torch.from_numpy(q), 10)
    return s.owned_range(len(q)), d.numpy(), i.numpy()


def _sharded_ivf_replicated(rank, world):
    return _sharded_ivf(rank, world, "replicated")


def _sharded_ivf_owner(rank, world):
    return _sharded_ivf(rank, world, "owner")


@pytest.mark.parametrize("mode", ["replicated", "owner"])
def test_sharded_ivf_equals_single_process(mode):
    """Coarse probe split across two ranks and all-gathered, each rank
    scanning its rows of the probed lists, lists exchanged and merged: the
    same answer as the single-process oracle IVF-Flat search (each query once
    in owner mode)."""
    out = _run(_sharded_ivf_replicated if mode == "replicated" else _sharded_ivf_owner)
    x, q, cent, labels = _ivf_setup()
    order = np.argsort(labels, kind="stable")
    off = np.concatenate([[0], np.cumsum(np.bincount(labels, minlength=len(cent)))]).astype(np.int64)
    rd, ri = oracle.ivf_flat_search("l2", q, cent, off, x[order], order.astype(np.int64), 4, 10)
    covered = 0
    for r in (0, 1):
        (a, b), d, i = out[r]
        assert (a, b) == ((0, len(q)) if mode == "replicated" else shard_range(len(q), r, 2))
        np.testing.assert_array_equal(i, ri[a:b])
        np.testing.assert_allclose(d, rd[a:b], rtol=1e-5)
        covered += b - a
    assert covered == (2 if mode == "replicated" else 1) * len(q)


def _sharded_kmeans(rank, world):
    from rapidadb_b200.kmeans import kmeans

    x, _ = _data()
    lo, hi = shard_range(len(x), rank, world)
    res = kmeans(torch.from_numpy(x[lo:hi]), 12, max_iters=6, tol=0.0, seed=9, ops=OracleOps())
    return res.centroids.numpy(), res.inertia, res.labels.numpy()


def test_sharded_kmeans_equals_single_process():
    out = _run(_sharded_kmeans)
    x, _ = _data()
    init = x[sample_rows(len(x), 12, 9)]
    rc, rl, rin, _ = oracle.kmeans(x, init, 6)
    for r in (0, 1):
        np.testing.assert_allclose(out[r][0], rc, rtol=1e-5, atol=1e-6)
        assert abs(out[r][1] - rin) <= 1e-5 * rin
    np.testing.assert_array_equal(np.concatenate([out[0][2], out[1][2]]), rl)


def _failing_rank(rank, world):
    # rank 1 raises before the collective: rank 0's all-gather must fail, not hang
    import datetime

    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    x, q = _data()
    d = torch.zeros(2, 3)
    dist.monitored_barrier(timeout=datetime.timedelta(seconds=5))
    return d


def test_rank_failure_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, _failing_rank, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
    assert all(p.exitcode is not None for p in ps), "a rank hung"
    assert any(p.exitcode != 0 for p in ps)


def test_shared_sample_plan_bounds():
    """The shared-threshold sample: a power-of-two group size <= 128 dividing
    each rank's share, at most a quarter of the smallest shard sampled, and at
    least 4 k group maxima in all; None when the shards are too small."""
    from rapidadb_b200.sharded import shared_sample_plan

    assert shared_sample_plan([125_000] * 8, 100) == (8192, 64, 65536)  # 1M rows, k = 100 on 8 ranks
    for sizes, k in [([500_000, 500_001], 100), ([20_000, 15_000, 15_001], 10), ([1_000_000] * 4, 1)]:
        per, g, total = shared_sample_plan(sizes, k)
        assert g & (g - 1) == 0 and g <= 128 and per % g == 0
        assert total == len(sizes) * per and 4 * per <= min(sizes)
        assert len(sizes) * (per // g) >= 4 * k
    assert shared_sample_plan([100, 100], 10) is None


def test_results_mode_is_checked():
    from rapidadb_b200.sharded import ShardedIVFSearch

    with pytest.raises(ValueError, match="results"):
        ShardedSearch(lambda q, k: (q, q), largest=False, results="everyone")
    with pytest.raises(ValueError, match="results"):
        ShardedIVFSearch(object(), largest=False, results="")
    with pytest.raises(ValueError, match="transport"):
        ShardedSearch(lambda q, k: (q, q), largest=False, transport="nvlink")


def _transport_on_gloo(rank, world):
    """CPU ranks have no peer transport: "auto" falls back to collectives,
    "peer" raises on every rank before any data moves."""
    from rapidadb_b200.sharded import PeerUnavailable

    x, q = _data()
    lo, hi = shard_range(len(x), rank, world)

    def local(qt, k):
        d, i = oracle.flat_search("l2", qt.numpy(), x[lo:hi], k, ids=np.arange(lo, hi, dtype=np.int64))
        return torch.from_numpy(d), torch.from_numpy(i)

    s = ShardedSearch(local, largest=False, merge=_oracle_merge, results="owner")
    d, i = s.search(torch.from_numpy(q), 10)
    out = {"auto": (s.owned_range(len(q)), d.numpy(), i.numpy(), s.peer is None)}
    try:
        ShardedSearch(local, largest=False, merge=_oracle_merge, transport="peer").search(torch.from_numpy(q), 10)
        out["peer"] = None
    except PeerUnavailable as e:
        out["peer"] = str(e)
    return out


def test_peer_transport_needs_gpu_ranks():
    out = _run(_transport_on_gloo, world=2)
    x, q = _data()
    rd, ri = oracle.flat_search("l2", q, x, 10)
    for r in range(2):
        (a, b), d, i, no_peer = out[r]["auto"]
        assert no_peer
        np.testing.assert_array_equal(i, ri[a:b])
        assert "NCCL" in out[r]["peer"]


def test_shard_range_partitions():
    for n in (0, 1, 7, 1000, 1001):
        for w in (1, 2, 3, 8):
            parts = [shard_range(n, r, w) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))
            assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1


def test_sample_rows_deterministic_distinct():
    a = sample_rows(10_000, 500, 42)
    assert a == sample_rows(10_000, 500, 42)
    assert len(set(a)) == 500 and all(0 <= v < 10_000 for v in a)
    assert a != sample_rows(10_000, 500, 43)
    with pytest.raises(ValueError):
        sample_rows(5, 6, 0)


# uneven shards: rank 0 holds fewer than k rows, rank 1 none, rank 2 the rest
_UNEVEN = [(0, 6), (6, 6), (6, 3001)]


def _uneven_flat(rank, world):
    x, q = _data()
    lo, hi = _UNEVEN[rank]

    def local(qt, k):
        assert 1 <= k <= hi - lo, f"k={k} on a shard of {hi - lo} rows"  # as FlatIndex::search checks
        d, i = oracle.flat_search("l2", qt.numpy(), x[lo:hi], k, ids=np.arange(lo, hi, dtype=np.int64))
        return torch.from_numpy(d), torch.from_numpy(i)

    out = {}
    for mode in ("replicated", "owner"):
        s = ShardedSearch(local, largest=False, merge=_oracle_merge, results=mode, local_size=hi - lo)
        d, i = s.search(torch.from_numpy(q), 10)
        out[mode] = (s.owned_range(len(q)), d.numpy(), i.numpy())
    try:
        ShardedSearch(local, largest=False, merge=_oracle_merge, local_size=hi - lo).search(torch.from_numpy(q), 5000)
        out["too_large"] = None
    except ValueError as e:
        out["too_large"] = str(e)
    return out


def test_short_and_empty_shards_pad_instead_of_hanging():
    """A shard with fewer than k rows answers with a padded list, an empty
    shard with padding only, and k above the rows of all shards raises
    ValueError on every rank (before any data collective) -- no rank is left
    waiting in a collective another rank never joins."""
    out = _run(_uneven_flat, world=3)
    x, q = _data()
    rd, ri = oracle.flat_search("l2", q, x, 10)
    for r in range(3):
        for mode in ("replicated", "owner"):
            (a, b), d, i = out[r][mode]
            np.testing.assert_array_equal(i, ri[a:b])
            np.testing.assert_allclose(d, rd[a:b], rtol=1e-6)
        assert "k must be in [1, 3001]" in out[r]["too_large"]


def _uneven_ivf(rank, world):
    from rapidadb_b200.sharded import ShardedIVFSearch

    x, q, cent, labels = _ivf_setup()
    lo, hi = _UNEVEN[rank]
    s = ShardedIVFSearch(_OracleIVFShard(x, labels, lo, hi, cent, 4), largest=False, merge=_oracle_merge)
    d, i = s.search(torch.from_numpy(q), 10)
    return d.numpy(), i.numpy()


def test_sharded_ivf_short_and_empty_shards():
    out = _run(_uneven_ivf, world=3)
    x, q, cent, labels = _ivf_setup()
    order = np.argsort(labels, kind="stable")
    off = np.concatenate([[0], np.cumsum(np.bincount(labels, minlength=len(cent)))]).astype(np.int64)
    rd, ri = oracle.ivf_flat_search("l2", q, cent, off, x[order], order.astype(np.int64), 4, 10)
    for r in range(3):
        np.testing.assert_array_equal(out[r][1], ri)
        np.testing.assert_allclose(out[r][0], rd, rtol=1e-5)


def test_peer_arena_layout_on_host():
    """PeerExchange's section layout without a GPU: sections start past the
    flags, 256-byte aligned, in the order given; views have the requested
    shape and dtype; the arena is mapped again only when a layout outgrows
    it (to at least twice its size), and never for a layout that fits."""
    from rapidadb_b200.sharded import PeerExchange

    ex = PeerExchange.__new__(PeerExchange)
    ex.nbytes, ex.ptr, ex.bases, ex.buf, ex._off, ex.epoch = 0, None, [], None, {}, 0
    maps = []

    def fake_map(nbytes):
        maps.append(nbytes)
        ex.nbytes = nbytes
        ex.buf = torch.zeros(nbytes, dtype=torch.uint8)

    ex._map = fake_map
    ex.reserve({"maxima": 4 * 10 * 3, "thr": 4 * 10, "lists0": 100, "lists1": 100})
    assert ex._off == {"maxima": 512, "thr": 768, "lists0": 1024, "lists1": 1280}
    assert maps == [1536]
    m = ex.view("maxima", (10, 3), torch.float32)
    assert m.shape == (10, 3) and m.dtype == torch.float32 and m.data_ptr() == ex.buf.data_ptr() + 512
    m.fill_(1.5)
    assert ex.view("thr", (10,), torch.float32).sum().item() == 0.0  # sections do not overlap
    ex.reserve({"maxima": 120})  # fits: no new mapping
    assert maps == [1536]
    ex.reserve({"probe": 8 * 1000})
    assert maps == [1536, 8704] and ex._off == {"probe": 512}
    assert [ex.next_epoch() for _ in range(3)] == [1, 2, 3]
