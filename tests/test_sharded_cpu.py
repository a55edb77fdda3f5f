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
