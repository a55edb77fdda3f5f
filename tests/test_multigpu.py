"""Row-sharded search (Flat, IVF-Flat, IVF-PQ) and k-means over NCCL, one
process per GPU (needs >= 2 GPUs; skipped otherwise).  Each rank holds a
contiguous slice of the rows; the sharded answer must equal the single-GPU
answer on the full table."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data():
    g = np.random.default_rng(5)
    centres = g.standard_normal((40, 64)).astype(np.float32) * 3
    x = (centres[g.integers(0, 40, 30000)] + g.standard_normal((30000, 64))).astype(np.float32)
    q = (centres[g.integers(0, 40, 300)] + g.standard_normal((300, 64))).astype(np.float32)
    return x, q


def _books(dev):
    g = np.random.default_rng(9)
    return torch.from_numpy(g.standard_normal((16, 64, 4)).astype(np.float32)).to(dev)


def _worker(rank, port, out_q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import rapidadb._C as _C
        from rapidadb_b200.kmeans import kmeans
        from rapidadb_b200.sharded import ShardedIVFSearch, ShardedSearch, shard_range

        x, q = _data()
        lo, hi = shard_range(len(x), rank, WORLD)
        xt = torch.from_numpy(x[lo:hi]).to(dev)
        qt = torch.from_numpy(q).to(dev)
        res = {}
        # flat, bf16 rows on the tensor cores, cosine
        flat = _C.FlatIndex(64, _C.Metric.COSINE, _C.Precision.BF16)
        flat.add(xt, torch.arange(lo, hi, device=dev))
        d, i = ShardedSearch(flat, largest=True).search(qt, 20)
        res["flat"] = (d.cpu().numpy(), i.cpu().numpy())
        # the same with each rank answering only its query slice
        so = ShardedSearch(flat, largest=True, results="owner")
        d, i = so.search(qt, 20)
        res["flat_owner"] = (so.owned_range(len(q)), d.cpu().numpy(), i.cpu().numpy())
        # both transports explicitly: the peer exchange kernel (three searches:
        # the epochs advance, the list sections alternate) and NCCL collectives
        for mode in ("owner", "replicated"):
            for transport in ("peer", "collective"):
                for thr in (True, False):
                    s = ShardedSearch(flat, largest=True, results=mode, transport=transport, shared_threshold=thr)
                    for _ in range(3):
                        d, i = s.search(qt, 20)
                    res[f"flat_{mode}_{transport}_{thr}"] = (s.owned_range(len(q)), d.cpu().numpy(), i.cpu().numpy())
                    assert (s.peer is not None) == (transport == "peer")
                    s.close()
        assert _C.device_status(True) == 0
        # k-means over the shards (sums / counts all-reduced)
        km = kmeans(xt, 32, max_iters=5, tol=0.0, seed=3, group=dist.group.WORLD, exact_assign=True)
        res["kmeans"] = (km.centroids.cpu().numpy(), km.inertia)
        # IVF-Flat with the k-means quantizer, probe split across ranks
        ivf = _C.IVFFlatIndex(64, _C.Metric.L2, 32, 6)
        ivf.set_quantizer(km.centroids)
        ivf.add(xt, torch.arange(lo, hi, device=dev))
        d, i = ShardedIVFSearch(ivf, largest=False).search(qt, 10)
        res["ivf"] = (d.cpu().numpy(), i.cpu().numpy())
        # both transports and result modes, three searches each
        for mode in ("owner", "replicated"):
            for transport in ("peer", "collective"):
                s = ShardedIVFSearch(ivf, largest=False, results=mode, transport=transport)
                for _ in range(3):
                    d, i = s.search(qt, 10)
                res[f"ivf_{mode}_{transport}"] = (s.owned_range(len(q)), d.cpu().numpy(), i.cpu().numpy())
                assert (s.peer is not None) == (transport == "peer")
                s.close()
        # IVF-PQ (query-major search) with the same quantizer, shared codebooks
        pq = _C.IVFPQIndex(64, _C.Metric.L2, 32, 6, 16, 64)
        pq.set_quantizer(km.centroids, _books(dev))
        pq.add(xt, torch.arange(lo, hi, device=dev))
        d, i = ShardedIVFSearch(pq, largest=False).search(qt, 10)
        res["ivfpq"] = (d.cpu().numpy(), i.cpu().numpy())
        out_q.put((rank, res))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs 2 GPUs")
def test_sharded_equals_single_gpu():
    import torch.multiprocessing as mp

    import rapidadb._C as _C
    from parity import assert_topk_match
    from rapidadb_b200.kmeans import kmeans
    from rapidadb_b200.sharded import shard_range

    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, port, q_)) for r in range(WORLD)]
    for p in ps:
        p.start()
    out = dict(q_.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0

    x, q = _data()
    xt, qt = torch.from_numpy(x).cuda(), torch.from_numpy(q).cuda()
    flat = _C.FlatIndex(64, _C.Metric.COSINE, _C.Precision.BF16)
    flat.add(xt)
    d, i = flat.search(qt, 20)
    km = kmeans(xt, 32, max_iters=5, tol=0.0, seed=3, exact_assign=True)
    ivf = _C.IVFFlatIndex(64, _C.Metric.L2, 32, 6)
    ivf.set_quantizer(km.centroids)
    ivf.add(xt)
    di, ii = ivf.search(qt, 10)
    pq = _C.IVFPQIndex(64, _C.Metric.L2, 32, 6, 16, 64)
    pq.set_quantizer(km.centroids, _books(xt.device))
    pq.add(xt)
    dp, ip = pq.search(qt, 10)
    covered = 0
    for r in range(WORLD):
        assert_topk_match(d.cpu().numpy(), i.cpu().numpy(), *out[r]["flat"], rtol=1e-4, atol=1e-5)
        (a, b), do, io = out[r]["flat_owner"]
        assert (a, b) == shard_range(len(q), r, WORLD)
        assert_topk_match(d[a:b].cpu().numpy(), i[a:b].cpu().numpy(), do, io, rtol=1e-4, atol=1e-5)
        covered += b - a
        for key, ((a, b), do, io) in ((kk, v) for kk, v in out[r].items() if kk.startswith("flat_") and
                                      kk != "flat_owner"):
            assert (a, b) == (shard_range(len(q), r, WORLD) if "_owner_" in key else (0, len(q))), key
            assert_topk_match(d[a:b].cpu().numpy(), i[a:b].cpu().numpy(), do, io, rtol=1e-4, atol=1e-5)
    assert covered == len(q)
    for r in range(WORLD):
        np.testing.assert_allclose(out[r]["kmeans"][0], km.centroids.cpu().numpy(), rtol=1e-5, atol=1e-5)
        assert abs(out[r]["kmeans"][1] - km.inertia) <= 1e-5 * km.inertia
        assert_topk_match(di.cpu().numpy(), ii.cpu().numpy(), *out[r]["ivf"], rtol=1e-5, atol=1e-4)
        for key, ((a, b), do, io) in ((kk, v) for kk, v in out[r].items() if kk.startswith("ivf_")):
            assert (a, b) == (shard_range(len(q), r, WORLD) if "_owner_" in key else (0, len(q))), key
            assert_topk_match(di[a:b].cpu().numpy(), ii[a:b].cpu().numpy(), do, io, rtol=1e-5, atol=1e-4)
        assert_topk_match(dp.cpu().numpy(), ip.cpu().numpy(), *out[r]["ivfpq"], rtol=1e-5, atol=1e-3)
