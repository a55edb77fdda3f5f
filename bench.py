#!/usr/bin/env python
"""Search-QPS benchmark of RapidaDB's search hot path (one JSON line on rank 0).

Headline workload (default ``flat_cosine_bf16``): exact cosine search over
1,000,000 stored rows x 768 dims in bf16 (i.i.d. N(0,1) rows, L2-normalised,
then rounded), queries of the same distribution, k = 100.  With N GPUs
(torchrun, one process per GPU) the rows are split across the ranks and the
query batch is 1,024 x N (per-GPU work fixed: "scaling": "weak"); a step is
sample maxima -> threshold exchange -> local fused search -> exchange of the
packed [Q, k] lists by query slice -> merge kernel on the rank owning the
slice, each exchange one kernel reading the other ranks' memory over NVLink
(``--transport collective``: NCCL all-to-all / all-gather instead).

* ``value``   queries/s with queries resident in HBM, CUDA events between
              barriers, max over ranks.  The stored rows (1.5 GB) exceed L2
              (126 MB): no flush needed.
* ``e2e``     the same through the public search API with each step's query
              batch copied in from pinned host memory and its results read
              back to the host.
* ``roofline`` the dominant kernel (tcgen05 main scan): 2 Q N d FLOP per
              launch over its CUDA-event duration, against the measured dense
              bf16 peak.
* ``phases_ms`` device time per step of each phase of the search (CUDA
              events recorded on the launching stream around each phase).
* ``cpu_baseline`` the oracle (fp32 restatement of the reference's exact
              search) on every host core, on a sample of the queries.
* ``workloads`` the other hot-path workloads in the same run, each with its
              own value, roofline, cpu_baseline, e2e and clocks: IVF-PQ (one
              GPU's shard of the 100M-row table at N = 1; 100M rows split over
              the N GPUs at N > 1), IVF-Flat (10M rows), k-means (one Lloyd
              iteration over 10M x 768 bf16 points, K = 16,384).

``--impl reference`` times the reference path's CPU restatement (the oracle:
the reference has no CPU implementation of its own and its GPU kernels are
not this path) on the same workload, on every host core.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import gc
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # flat cosine search: 1,000,000 x 768 bf16 rows, 1,024 queries, k = 100 (the headline workload)
    "flat_cosine_bf16": dict(N=1_000_000, d=768, Q=1024, k=100, metric="cosine", precision="bf16",
                             normalize=True),
    # flat exact L2 search: 100,000 x 768 fp32 rows, 32 queries, k = 10 (the reference's CPU-runnable case)
    "flat_l2_fp32": dict(N=100_000, d=768, Q=32, k=10, metric="l2", precision="fp32",
                         normalize=False),
    # IVF-Flat: 10,000,000 x 128 fp32 rows from a mixture of 1,024 Gaussians
    # (centres ~N(0,4I), sigma=1); nlist=4,096 trained by 20 k-means iterations on a 1M
    # sample; 10,000 queries; nprobe=32; k=10.  N > 1 GPUs split the rows.
    "ivf_flat": dict(kind="ivf", N=10_000_000, d=128, Q=10_000, k=10, metric="l2", nlist=4096,
                     nprobe=32, ncentres=1024, spread=2.0, sigma=1.0, train=1_000_000, iters=20,
                     uint8=False),
    # IVF-PQ over 100,000,000 x 128 uint8-valued rows (stored fp32); nlist=16,384;
    # M=16 x 256; 10,000 queries; nprobe=64; k=10.  One GPU holds one 8-GPU shard
    # (12,500,000 rows); N > 1 GPUs split the full 100M rows.
    "ivf_pq": dict(kind="ivf_pq", N=100_000_000, N1=12_500_000, d=128, Q=10_000, k=10, metric="l2",
                   nlist=16384, nprobe=64, M=16, ksub=256, ncentres=1024, spread=2.0, sigma=1.0,
                   train=262_144, iters=10, uint8=True),
    # streaming add into the IVF-Flat workload's index: batches of 10,000 rows
    # appended to the 10,000,000 stored rows
    "ivf_add": dict(kind="ivf_add", N=10_000_000, d=128, batch=10_000, nlist=4096, nprobe=32,
                    ncentres=1024, spread=2.0, sigma=1.0, train=1_000_000, iters=20, uint8=False),
    # k-means: 10,000,000 x 768 bf16 points from a mixture of 16,384 Gaussians (centres
    # ~N(0,I), sigma=0.3); K=16,384; seeded random-row init; Lloyd iterations; N > 1 GPUs
    # split the rows and all-reduce centroid sums and counts
    "kmeans": dict(kind="kmeans", N=10_000_000, d=768, K=16384, iters=20, ncentres=16384,
                   spread=1.0, sigma=0.3),
}

# workloads measured inside the headline run (steps, warm-up)
SUB_WORKLOADS = [("ivf_pq", 10, 3), ("ivf_flat", 10, 3), ("kmeans", 3, 3)]

# ncu dram__bytes_read.sum + dram__bytes_write.sum of one tcgen05 main-scan
# launch of the headline search (1,000,000 rows x 768 dims, 1,024 queries:
# 1.588858 GB read + 19.74 MB written), per stored row; it scales with rows
TC_SCAN_DRAM_BYTES_PER_ROW = 1608.6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="flat_cosine_bf16", choices=sorted(WORKLOADS))
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target host time of each CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-workloads", action="store_true",
                    help="headline only: skip the IVF-PQ / IVF-Flat / k-means entries")
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--rows", type=int, default=0, help="override the workload's stored rows")
    ap.add_argument("--queries", type=int, default=0, help="override the per-GPU query batch")
    ap.add_argument("--timeline", type=int, default=0,
                    help="after the run, record the kernel timeline of this many headline searches (CUPTI via "
                         "torch.profiler) and print per-kernel durations and gaps to stderr")
    ap.add_argument("--results", default="owner", choices=["owner", "replicated"],
                    help="flat search on N > 1 GPUs: each rank returns the answers of its query slice "
                         "(owner) or of the whole batch (replicated)")
    ap.add_argument("--transport", default="auto", choices=["auto", "peer", "collective"],
                    help="sharded searches on N > 1 GPUs: exchanges through the peer exchange kernel over "
                         "NVLink (peer; auto picks it on one node) or NCCL collectives")
    return ap.parse_args()


# ------------------------------------------------------------------ data gen

def gen_rows(lo, hi, d, seed, normalize, dtype, device):
    """Rows [lo, hi) of the synthetic table: chunk c of 65,536 rows is drawn
    from a CUDA generator seeded (seed, c), so any rank regenerates exactly its
    slice of the same table."""
    import torch

    CH = 65536
    out = torch.empty((hi - lo, d), dtype=dtype, device=device)
    c0, c1 = lo // CH, (hi - 1) // CH if hi > lo else -1
    g = torch.Generator(device=device)
    for c in range(c0, c1 + 1):
        g.manual_seed(seed * 1_000_003 + c)
        a, b = c * CH, (c + 1) * CH
        blk = torch.randn((CH, d), generator=g, device=device, dtype=torch.float32)
        if normalize:
            blk = torch.nn.functional.normalize(blk, dim=1)
        s, e = max(a, lo), min(b, hi)
        out[s - lo:e - lo] = blk[s - a:e - a].to(dtype)
    return out


def gen_queries(Q, d, seed, normalize, dtype, device):
    return gen_rows(0, Q, d, seed + 7919, normalize, dtype, device)


def gen_mixture(lo, hi, d, wl, seed, dtype, device, salt=0):
    """Rows [lo, hi) of a seeded Gaussian mixture: centres ~ N(0, spread^2 I)
    (fixed by `seed`), row = centre[c] + sigma N(0, I) with c uniform; chunk c
    of 65,536 rows uses its own generator, so any rank regenerates exactly its
    slice; `salt` changes the row draws but not the centres (queries come from
    the same mixture as the stored rows).  uint8 workloads scale to 16 units
    per sigma around 128 and clip to [0, 255] (integer values stored as
    floats)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed * 7 + 1)
    centres = torch.randn((wl["ncentres"], d), generator=g, device=device) * wl["spread"]
    CH = 65536
    out = torch.empty((hi - lo, d), dtype=dtype, device=device)
    c0, c1 = lo // CH, (hi - 1) // CH if hi > lo else -1
    for c in range(c0, c1 + 1):
        g.manual_seed(seed * 1_000_003 + 17 * c + 5 + 7_919_993 * salt)
        a, b = c * CH, (c + 1) * CH
        lab = torch.randint(0, wl["ncentres"], (CH,), generator=g, device=device)
        blk = centres[lab] + wl["sigma"] * torch.randn((CH, d), generator=g, device=device)
        if wl.get("uint8"):
            blk = torch.clamp(torch.round(blk * 16.0 + 128.0), 0, 255)
        s_, e_ = max(a, lo), min(b, hi)
        out[s_ - lo:e_ - lo] = blk[s_ - a:e_ - a].to(dtype)
    return out


# ------------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    5 ms during the timed region (read-only queries; no setting is changed).
    Without NVML the record says so ("nvml unavailable") and holds no samples."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index, period_s=0.005):
        self.cuda_index = cuda_index
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def _handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.cuda_index).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid)

    def start(self):
        try:
            nv, h = self._handle()
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons

            def loop():
                while not self._stop.is_set():
                    try:
                        self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), int(get_reasons(h))))
                    except Exception:
                        pass
                    time.sleep(self.period)

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None

    def stop(self):
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        self._stop.set()
        self._thread.join(timeout=2)
        sm = [c for c, _ in self.samples]
        reasons = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvml 5 ms"}


# ------------------------------------------------------------ shared helpers

class Ctx:
    """One process per GPU: rank, world size, device; NCCL process group when
    world > 1 (short timeout so that ranks waiting on each other fail)."""

    def __init__(self):
        import datetime

        import torch
        import torch.distributed as dist

        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local_rank)
        self.dev = torch.device("cuda", self.local_rank)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)

    def barrier(self):
        import torch.distributed as dist

        if self.world > 1:
            dist.barrier()

    def device_barrier(self):
        """A one-element all-reduce on the current stream, not waited for on
        the host: work queued after it starts on every rank's GPU once all
        ranks' GPUs have reached it."""
        import torch
        import torch.distributed as dist

        if self.world > 1:
            dist.all_reduce(torch.zeros(1, device=self.dev))

    def max(self, v):
        """Max over ranks of a host float."""
        import torch
        import torch.distributed as dist

        t = torch.tensor([float(v)], device=self.dev, dtype=torch.float64)
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        import torch.distributed as dist

        if self.world > 1:
            dist.barrier()
            dist.destroy_process_group()


def kernel_lib():
    import ctypes

    lib = ctypes.CDLL(os.path.join(ROOT, "rapidadb_b200", "librdb_kernels.so"))
    lib.rdb_launch_count.restype = ctypes.c_ulonglong
    return lib


def read_tag(lib, mask):
    """(mean ms per launch, launches) of the timed launches with a tag in mask."""
    import ctypes

    tot, nl = ctypes.c_double(0.0), ctypes.c_int(0)
    lib.rdb_timing_read_tags(mask, ctypes.byref(tot), ctypes.byref(nl))
    return (tot.value / nl.value if nl.value else 0.0), nl.value


def timed(ctx, fn, steps, warmup, tag_mask, tags=None):
    """CUDA-event time of `steps` calls of fn (after `warmup` untimed calls),
    barrier + synchronize on both sides, max over ranks.  Returns a dict:
    ms (all steps), kernel_ms (mean per launch of tag_mask's first bit),
    phases (tag name -> ms per step), launches (this library's kernels in the
    timed region), clocks, out (fn's last result)."""
    import torch

    # the warm-up keeps each result alive until the next call returns, as the
    # timed loop does, so the caching allocator already holds both result
    # blocks (otherwise the second timed step makes a device allocation)
    out = None
    for _ in range(warmup):
        out = fn()
    torch.cuda.synchronize()
    ctx.barrier()
    lib = kernel_lib()
    clocks = ClockSampler(ctx.local_rank)
    clocks.start()
    all_mask = tag_mask | sum((tags or {}).values())
    lib.rdb_timing_enable(all_mask)
    torch.cuda.synchronize()
    ctx.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    # the ranks' timed regions start together on the devices (a rank whose
    # host left the barrier later would otherwise add that delay to the
    # others' first exchange and so to the max over ranks)
    ctx.device_barrier()
    n0 = lib.rdb_launch_count()
    # no garbage-collection pause inside the timed steps (as timeit does);
    # the slowest step's host time is reported, so a host stall that left
    # the GPU idle is visible in the record
    gc.collect()
    gc_was_on = gc.isenabled()
    gc.disable()
    allocs0 = torch.cuda.memory_stats().get("num_device_alloc", 0)
    host_steps = []
    e0.record()
    for _ in range(steps):
        h0 = time.perf_counter()
        out = fn()
        host_steps.append(time.perf_counter() - h0)
    e1.record()
    device_allocs = torch.cuda.memory_stats().get("num_device_alloc", 0) - allocs0
    if gc_was_on:
        gc.enable()
    host_max = max(host_steps) if host_steps else 0.0
    launches = int(lib.rdb_launch_count() - n0)
    torch.cuda.synchronize()
    ctx.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    kern_ms, _ = read_tag(lib, tag_mask)
    phases = {}
    for name, m in (tags or {}).items():
        per, n = read_tag(lib, m)
        phases[name] = round(per * n / max(steps, 1), 4)
    lib.rdb_timing_enable(0)
    clk = clocks.stop()
    return {"ms": ctx.max(ms), "kernel_ms": kern_ms, "phases": phases, "launches": launches,
            "clocks": clk, "out": out, "host_ms_max_step": round(1e3 * host_max, 3),
            "host_ms_steps": [round(1e3 * h, 3) for h in host_steps], "device_allocs": int(device_allocs)}


def peaks():
    try:
        p = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", 0.0)), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def host_threads():
    return len(os.sched_getaffinity(0))


def recall_at_k(got, ref, k):
    import numpy as np

    return float(np.mean([len(set(a.tolist()) & set(b.tolist())) / k for a, b in zip(got, ref)]))


# flat-search phase tags of the C ABI's timing hook
FLAT_TAGS = {"query_values": 32, "sample_and_threshold": 64, "main_scan": 1, "candidate_select": 128,
             "overflow_repair": 256}


# ------------------------------------------------------------------ flat

def flat_config(args, wl, world):
    """The workload's configuration (identical keys in both arms)."""
    return {"workload": args.workload, "rows": wl["N"], "dim": wl["d"], "queries_per_step": wl["Q"] * world,
            "k": wl["k"], "metric": wl["metric"], "precision": wl["precision"]}


def flat_cpu_baseline(xf, qf, wl, target_s):
    """The oracle on every host thread over a sample of the queries against
    every stored row."""
    import oracle

    nth = host_threads()
    t0 = time.perf_counter()
    oracle.flat_search(wl["metric"], qf[:2], xf, wl["k"], acc64=False, nthreads=nth)
    per_q = max((time.perf_counter() - t0) / 2, 1e-4)
    nq = int(max(2, min(len(qf), target_s / per_q)))
    t0 = time.perf_counter()
    oracle.flat_search(wl["metric"], qf[:nq], xf, wl["k"], acc64=False, nthreads=nth)
    el = time.perf_counter() - t0
    return {"value": round(nq / el, 3), "unit": "queries/s", "cores": nth, "kind": "port",
            "sample": f"{nq} queries x {xf.shape[0]:,} rows x {xf.shape[1]} dims (fp32 upcast of the "
                      f"stored values), all rows scored, {el:.1f} s"}


def run_flat(args, wl, ctx):
    import numpy as np
    import torch
    import torch.distributed as dist

    from rapidadb_b200.config import IndexConfig, Metric, Precision
    from rapidadb_b200.index import RapidaDB
    from rapidadb_b200.sharded import ShardedSearch, shard_range

    rank, world, dev = ctx.rank, ctx.world, ctx.dev
    N, d, k = wl["N"], wl["d"], wl["k"]
    Q = wl["Q"] * world
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["precision"]]
    lo, hi = shard_range(N, rank, world)
    x = gen_rows(lo, hi, d, args.seed, wl["normalize"], tdt, dev)
    q = gen_queries(Q, d, args.seed, wl["normalize"], tdt, dev)
    cfg = IndexConfig(dim=d, metric=Metric(wl["metric"]), precision=Precision(wl["precision"]))
    db = RapidaDB(config=cfg)
    db.add(x, torch.arange(lo, hi, device=dev, dtype=torch.long))
    searcher = ShardedSearch(db, wl["metric"] != "l2", results=args.results if world > 1 else "replicated",
                             transport=args.transport)
    own_lo, own_hi = searcher.owned_range(Q)

    # ---- device-resident timing: the main-scan launches carry CUDA events
    # (the roofline's kernel time); the per-phase breakdown comes from a
    # separate pass with events around every phase, so the timed region
    # holds only those two events per step
    t = timed(ctx, lambda: searcher.search(q, k), args.steps, args.warmup, 1)
    out_d, out_i = t["out"]
    tp = timed(ctx, lambda: searcher.search(q, k), min(args.steps, 10), 1, 1, FLAT_TAGS)
    phase_step_ms = tp["ms"] / min(args.steps, 10)
    exchange = None
    if world > 1:
        searcher.clock.enabled = True
        for _ in range(min(args.steps, 10)):
            searcher.search(q, k)
        searcher.clock.enabled = False
        mine = searcher.clock.summary()
        names = sorted(mine)
        vals = torch.tensor([mine[n] for n in names], device=dev, dtype=torch.float64)
        allv = torch.empty((world, len(names)), device=dev, dtype=torch.float64)
        dist.all_gather_into_tensor(allv, vals)
        allv = allv.cpu().numpy()
        exchange = {n: {"max_over_ranks": round(float(allv[:, j].max()), 4),
                        "min_over_ranks": round(float(allv[:, j].min()), 4)} for j, n in enumerate(names)}

    # ---- end to end through the public API with host buffers
    q_host = q.cpu().pin_memory()
    h2d = q_host.numel() * q_host.element_size()
    qbuf = torch.empty_like(q)
    for _ in range(max(1, args.warmup // 2)):
        qbuf.copy_(q_host, non_blocking=True)
        rd, ri = searcher.search(qbuf, k)
        rd.cpu(), ri.cpu()
    torch.cuda.synchronize()
    ctx.barrier()
    d2h = 0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        qbuf.copy_(q_host, non_blocking=True)
        rd, ri = searcher.search(qbuf, k)
        hd, hi_ = rd.cpu(), ri.cpu()
        d2h = hd.numel() * hd.element_size() + hi_.numel() * hi_.element_size()
    e2e_seq_s = ctx.max(time.perf_counter() - t0)
    e2e_s, e2e_mode = e2e_seq_s, "sequential: each step copies its batch in, searches, reads the results back"
    e2e_pipe_s = None
    if world == 1:
        # the public pipelined API (rapidadb_b200.pipeline.AsyncBatchSearcher):
        # the same host batches, staged in pinned memory, copied in, searched
        # and read back on one of two worker streams
        from rapidadb_b200.pipeline import AsyncBatchSearcher

        if q_host.dtype == torch.bfloat16:
            src = q_host.view(torch.int16).repeat(args.steps, 1).view(torch.bfloat16)
        else:
            src = q_host.repeat(args.steps, 1)
        pipe = AsyncBatchSearcher(db, num_streams=2)
        pipe.search_host(src[:2 * Q], k, batch_size=Q)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        pipe.search_host(src, k, batch_size=Q)
        e2e_pipe_s = time.perf_counter() - t0
        pipe.close()
        # both are the public API with the same host batches: the faster of
        # the two is the end-to-end figure, and the record names it
        if e2e_pipe_s < e2e_s:
            e2e_s, e2e_mode = e2e_pipe_s, "pipelined: AsyncBatchSearcher, 2 worker streams, one batch per step"

    # ---- recall against exact fp32 search over the same stored values
    nrec = min(64, own_hi - own_lo)  # rank 0 owns the first queries in every results mode
    qs = q[:nrec].float()
    xs = x.float()
    if wl["metric"] == "cosine":
        s = torch.nn.functional.normalize(qs, dim=1) @ torch.nn.functional.normalize(xs, dim=1).T
    elif wl["metric"] == "dot_product":
        s = qs @ xs.T
    else:
        s = -torch.cdist(qs, xs).pow(2)
    tv, ti = torch.topk(s, k, dim=1)
    ti = ti + lo
    if world > 1:
        gv = torch.empty((world * nrec, k), device=dev, dtype=tv.dtype)
        gi = torch.empty((world * nrec, k), device=dev, dtype=ti.dtype)
        dist.all_gather_into_tensor(gv, tv.contiguous())
        dist.all_gather_into_tensor(gi, ti.contiguous())
        gv, gi = gv.view(world, nrec, k), gi.view(world, nrec, k)
        order = torch.topk(gv.permute(1, 0, 2).reshape(nrec, -1), k, dim=1).indices
        ti = torch.gather(gi.permute(1, 0, 2).reshape(nrec, -1), 1, order)
    del s, xs
    recall = recall_at_k(out_i[:nrec].cpu().numpy(), ti.cpu().numpy(), k)

    res = None
    if rank == 0:
        hbm, bf16, bf16_sus, src = peaks()
        n_local = hi - lo
        ms = t["ms"]
        kernel_ms = t["kernel_ms"]
        qps = Q * args.steps / (ms * 1e-3)
        half = wl["precision"] != "fp32"
        if half:
            flops = 2.0 * Q * n_local * d
            ach = flops / (kernel_ms * 1e-3) / 1e12 if kernel_ms > 0 else None
            roof = {"bound": "tensor", "achieved": round(ach, 1) if ach else None, "peak": bf16,
                    "unit": "TFLOP/s", "frac": round(ach / bf16, 4) if ach else None,
                    "traffic": round(TC_SCAN_DRAM_BYTES_PER_ROW * n_local),
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the main-scan launch of "
                                      "the 1,000,000-row, 1,024-query search, per stored row x this GPU's rows",
                    "kernel": ("tc_scan_pair_kernel<FILTER> (CTA pair, main pass)" if Q > 128
                               else "tc_scan_kernel<FILTER> (main pass)"),
                    "kernel_ms": round(kernel_ms, 4), "flops_per_launch": flops,
                    "algorithmic_unit": "2 d FLOP per (query, stored row)",
                    "peak_source": f"{src} bf16 dense (burst)",
                    "step_frac": round(flops / (ms / args.steps * 1e-3) / 1e12 / bf16, 4)}
        else:
            byt = n_local * d * 4 + Q * d * 4
            ach = byt / (kernel_ms * 1e-3) / 1e9 if kernel_ms > 0 else None
            roof = {"bound": "hbm", "achieved": round(ach, 1) if ach else None, "peak": hbm, "unit": "GB/s",
                    "frac": round(ach / hbm, 4) if ach else None, "traffic": None,
                    "kernel": "simt_tma_scan_kernel<FILTER> (main pass)", "kernel_ms": round(kernel_ms, 4),
                    "bytes_per_launch": byt, "algorithmic_unit": "d x 4 B per stored row + d x 4 B per query",
                    "peak_source": f"{src} HBM copy"}
        res = {
            "metric": "search QPS (exact flat search, recall@%d)" % k,
            "value": round(qps, 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": wl["precision"],
            "data": "synthetic (seeded N(0,1) rows%s)" % (", L2-normalised" if wl["normalize"] else ""),
            "config": flat_config(args, wl, world),
            "parallelism": f"row-shard x{world}" if world > 1 else "single GPU",
            "rows_per_gpu": n_local,
            "results_mode": ("owner: rank r merges and returns the answers of its 1/%d slice of the query batch"
                             % world if args.results == "owner" else "replicated: every rank merges the whole batch")
            if world > 1 else None,
            "transport": (("peer: one exchange kernel per exchange (sample maxima, thresholds, lists) reading "
                           "the other ranks' arenas over NVLink (CUDA IPC, plain peer loads)")
                          if searcher.peer is not None else "collective: NCCL all-to-all / all-gather")
            if world > 1 else None,
            "l2_flush": "not needed: stored rows (%.2f GB per GPU) exceed L2 (126 MB)" % (
                n_local * d * (2 if half else 4) / 1e9),
            "recall_at_k_vs_fp32_exact": round(recall, 5),
            "phases_ms": dict(tp["phases"], between_phases=round(phase_step_ms - sum(tp["phases"].values()), 4),
                              step=round(phase_step_ms, 4),
                              source="separate %d-step pass with CUDA events around every phase" % min(args.steps, 10)),
            "e2e": {"value": round(Q * args.steps / e2e_s, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "mode": e2e_mode,
                    "sequential_value": round(Q * args.steps / e2e_seq_s, 1),
                    "pipelined_value": round(Q * args.steps / e2e_pipe_s, 1) if world == 1 else None},
            "gpu_launches": t["launches"],
            "roofline": roof,
            "clocks": t["clocks"],
            "host_ms_max_step": t["host_ms_max_step"],
            "device_allocs_in_timed_steps": t["device_allocs"],
        }
        if exchange is not None:
            res["exchange_phases_ms"] = exchange
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = flat_cpu_baseline(x.float().cpu().numpy(), q[:256].float().cpu().numpy(), wl,
                                                args.cpu_seconds)
    if args.timeline > 0 and world == 1:
        kernel_timeline(lambda: searcher.search(q, k), args.timeline)
    searcher.close()  # collective: every rank frees its exchange arena
    from rapidadb_b200._lib import C

    status = C().device_status(True)  # bounded device waits that ran out, any rank
    status = int(ctx.max(float(status)))
    if rank == 0:
        res["device_status"] = status
    if status:
        raise RuntimeError(f"a bounded device wait ran out during the flat workload (status {status:#x})")
    del x, q, db
    return res


def kernel_timeline(fn, n):
    """Kernels of n calls of fn as they ran back to back (CUPTI activity
    records through torch.profiler, no replay), after a 2 s pause: per kernel
    its duration and the idle gap before it, printed to stderr."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    fn()
    torch.cuda.synchronize()
    time.sleep(2.0)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            fn()
        torch.cuda.synchronize()
    ev = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA),
                key=lambda e: e.time_range.start)
    prev = None
    rows = []
    for e in ev:
        gap = None if prev is None else e.time_range.start - prev
        rows.append({"kernel": e.name[:80], "us": round(e.time_range.elapsed_us(), 1),
                     "gap_before_us": None if gap is None else round(gap, 1)})
        prev = e.time_range.end
    total = (ev[-1].time_range.end - ev[0].time_range.start) if ev else 0
    print(json.dumps({"timeline": rows, "calls": n, "us_per_call": round(total / max(n, 1), 1)}), file=sys.stderr,
          flush=True)


# ------------------------------------------------------------------ IVF

def ivf_rows(wl, world):
    """Stored rows of an IVF workload at this GPU count."""
    return wl.get("N1", wl["N"]) if world == 1 else wl["N"]


def run_ivf(args, wl, ctx, name, steps, warmup):
    """IVF-Flat / IVF-PQ search QPS.  Rows are split over the ranks (every
    rank trains the same quantizer from the same seeded sample); the coarse
    probe is split across ranks and the list table shared; each rank scans
    its rows of the probed lists; the lists of each query slice go to its
    owner, which merges them (exchanges: the peer exchange kernel, or NCCL
    with --transport collective)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from rapidadb_b200._lib import C
    from rapidadb_b200.kmeans import kmeans, train_pq
    from rapidadb_b200.sharded import ShardedIVFSearch, shard_range

    rank, world, dev = ctx.rank, ctx.world, ctx.dev
    _C = C()
    N = ivf_rows(wl, world)
    d, k, nlist, nprobe, Q = wl["d"], wl["k"], wl["nlist"], wl["nprobe"], wl["Q"]
    pq = wl["kind"] == "ivf_pq"
    t_setup = time.perf_counter()
    ntr = min(wl["train"], N)
    xtr = gen_mixture(0, ntr, d, wl, args.seed, torch.float32, dev)
    cent = kmeans(xtr, nlist, wl["iters"], 0.0, args.seed).centroids
    if pq:
        lab, _ = _C.kmeans_assign(xtr, cent, True)
        books = train_pq(xtr - cent.index_select(0, lab.long()), wl["M"], wl["ksub"], wl["iters"], args.seed)
        idx = _C.IVFPQIndex(d, _C.Metric.L2, nlist, nprobe, wl["M"], wl["ksub"])
        idx.set_quantizer(cent, books)
    else:
        idx = _C.IVFFlatIndex(d, _C.Metric.L2, nlist, nprobe, _C.Precision.FP32)
        idx.set_quantizer(cent)
    del xtr
    lo, hi = shard_range(N, rank, world)
    CH = 4_194_304
    for a in range(lo, hi, CH):
        b = min(hi, a + CH)
        xb = gen_mixture(a, b, d, wl, args.seed, torch.float32, dev)
        idx.add(xb, torch.arange(a, b, device=dev, dtype=torch.long))
        del xb
    torch.cuda.synchronize()
    t_setup = time.perf_counter() - t_setup
    q = gen_mixture(0, Q, d, wl, args.seed, torch.float32, dev, salt=1)
    searcher = ShardedIVFSearch(idx, largest=False, results="owner" if world > 1 else "replicated",
                                transport=args.transport)
    own_lo, own_hi = searcher.owned_range(Q)
    tag = 4 if pq else 2
    t = timed(ctx, lambda: searcher.search(q, k), steps, warmup, tag)
    out_d, out_i = t["out"]

    # e2e: host query batch in, results out, each step
    q_host = q.cpu().pin_memory()
    qbuf = torch.empty_like(q)
    for _ in range(2):
        qbuf.copy_(q_host, non_blocking=True)
        rd, ri = searcher.search(qbuf, k)
        rd.cpu(), ri.cpu()
    torch.cuda.synchronize()
    ctx.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        qbuf.copy_(q_host, non_blocking=True)
        rd, ri = searcher.search(qbuf, k)
        rd.cpu(), ri.cpu()
    e2e_s = ctx.max(time.perf_counter() - t0)
    searcher.close()  # collective: every rank frees its exchange arena

    # recall@k against exact search over the same rows (the first 100 queries, owned by rank 0)
    nrec = min(100, own_hi - own_lo)
    parts = []
    for a in range(lo, hi, CH):
        b = min(hi, a + CH)
        xb = gen_mixture(a, b, d, wl, args.seed, torch.float32, dev)
        xv = _C.row_values(_C.Metric.L2, xb, d)
        parts.append(_C.search_rows(_C.Metric.L2, xb, d, xv, q[:nrec], k, None, a))
        del xb
    ev = torch.cat([p[0] for p in parts], 1)
    ei = torch.cat([p[1] for p in parts], 1)
    order = torch.argsort(ev, dim=1)[:, :k]
    tv, ti = torch.gather(ev, 1, order), torch.gather(ei, 1, order)
    if world > 1:
        gv = torch.empty((world * nrec, k), device=dev)
        gi = torch.empty((world * nrec, k), device=dev, dtype=torch.long)
        dist.all_gather_into_tensor(gv, tv.contiguous())
        dist.all_gather_into_tensor(gi, ti.contiguous())
        gv = gv.view(world, nrec, k).permute(1, 0, 2).reshape(nrec, -1)
        gi = gi.view(world, nrec, k).permute(1, 0, 2).reshape(nrec, -1)
        ti = torch.gather(gi, 1, torch.argsort(gv, dim=1)[:, :k])
    recall = recall_at_k(out_i[:nrec].cpu().numpy(), ti.cpu().numpy(), k)
    sizes = idx.list_sizes().double()
    probes = searcher.probe(q)
    scanned = float(sizes[probes.flatten()].sum().item())  # rows of this rank's probed list slices
    bpr = wl["M"] if pq else d * 4
    tc = (not pq) and idx.tensor_core_search(k)
    # the tensor-core scan reads each probed list's rows once per search
    list_rows = float(sizes[torch.unique(probes.flatten())].sum().item())
    res = None
    if rank == 0:
        hbm, _, _, src = peaks()
        alg_bytes = (list_rows if tc else scanned) * bpr
        kern_ms = t["kernel_ms"]
        ach = alg_bytes / (kern_ms * 1e-3) / 1e9 if kern_ms > 0 else None
        ms = t["ms"]
        res = {
            "metric": f"search QPS ({'IVF-PQ' if pq else 'IVF-Flat'}, nprobe={nprobe}, recall@{k})",
            "value": round(Q * steps / (ms * 1e-3), 1), "unit": "queries/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(ms / steps, 4), "higher_is_better": True,
            "scaling": "strong" if world > 1 else None, "dtype": "u8" if pq else "f32",
            "data": "synthetic (seeded Gaussian mixture%s)" % (", uint8-valued" if wl.get("uint8") else ""),
            "config": {"workload": name, "rows": N, "rows_per_gpu": hi - lo, "dim": d, "queries_per_step": Q,
                       "k": k, "nlist": nlist, "nprobe": nprobe,
                       **({"pq_m": wl["M"], "pq_k": wl["ksub"]} if pq else {}),
                       "train_rows": ntr, "train_iters": wl["iters"]},
            "setup_s": round(t_setup, 1),
            "recall_at_k_vs_exact": round(recall, 4),
            "l2_flush": "not needed: stored %s (%.2f GB per GPU) exceed L2 (126 MB)" % (
                "codes" if pq else "rows", (hi - lo) * bpr / 1e9),
            "e2e": {"value": round(Q * steps / e2e_s, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(q.numel() * 4), "d2h_bytes_per_step": int((own_hi - own_lo) * k * 12),
                    "mode": "sequential: each step copies its batch in, searches, reads the results back"},
            "gpu_launches": t["launches"],
            "roofline": {"bound": "hbm", "achieved": round(ach, 1) if ach else None, "peak": hbm, "unit": "GB/s",
                         "frac": round(ach / hbm, 4) if ach else None, "traffic": None,
                         "kernel": ("ivfpq_search_kernel<%d> (query-major)" % wl["M"] if idx.query_major()
                                    else "ivfpq_scan_kernel") if pq else (
                                        "ivf_tc_scan_kernel (tcgen05)" if tc else "ivf_flat_scan_kernel"),
                         "kernel_ms": round(kern_ms, 4), "bytes_per_launch": alg_bytes,
                         "algorithmic_unit": (
                             "M code bytes per (query, probed row): sum over (query, probed list) of the list's "
                             "code bytes on this GPU; lists probed by queries running at the same time are "
                             "served from L2, so frac may exceed 1" if pq else
                             "d x 4 B per stored row of every list probed by at least one query: the tensor-core "
                             "scan reads each probed list's fp16 hi / lo planes (as many bytes as the fp32 rows) "
                             "once per 128 probing queries of the list" if tc else
                             "d x 4 B per (query, probed row): sum over (query, probed list) of the list's row "
                             "bytes on this GPU; the list-major scan reads a list once per 32-query chunk, so "
                             "frac is far above 1 and the contraction rate bounds it"),
                         "peak_source": f"{src} HBM copy"},
            "clocks": t["clocks"],
            "host_ms_max_step": t["host_ms_max_step"],
            "device_allocs_in_timed_steps": t["device_allocs"],
        }
        if not pq:
            flops = 2.0 * scanned * d
            res["roofline"]["contraction_tflops"] = round(flops / (kern_ms * 1e-3) / 1e12, 2) if kern_ms > 0 else None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = ivf_cpu_baseline(idx, pq, q, wl, args.cpu_seconds, N)
    del idx, q
    return res


def ivf_cpu_baseline(idx, pq, q, wl, target_s, N):
    """The oracle's IVF-Flat / IVF-PQ search (same centroids, codebooks and
    stored rows or codes) on every host thread over a sample of the queries."""
    import oracle

    nth = host_threads()
    off = idx.list_offsets().cpu().numpy()
    ids = idx.stored_ids().cpu().numpy()
    cent = idx.centroids().cpu().numpy()
    qf = q.cpu().numpy()
    if pq:
        data = idx.stored_codes().cpu().numpy()
        books = idx.codebooks().cpu().numpy()
        fn = lambda qq: oracle.ivfpq_search(qq, cent, off, data, ids, books, wl["nprobe"], wl["k"], nthreads=nth)
    else:
        data = idx.stored_vectors().cpu().numpy()
        fn = lambda qq: oracle.ivf_flat_search("l2", qq, cent, off, data, ids, wl["nprobe"], wl["k"], nthreads=nth)
    t0 = time.perf_counter()
    fn(qf[:32])
    per_q = max((time.perf_counter() - t0) / 32, 1e-5)
    nq = int(max(32, min(len(qf), target_s / per_q)))
    t0 = time.perf_counter()
    fn(qf[:nq])
    el = time.perf_counter() - t0
    return {"value": round(nq / el, 2), "unit": "queries/s", "cores": nth, "kind": "port",
            "sample": f"{nq} queries against all {N:,} stored rows (nprobe {wl['nprobe']}), {el:.1f} s"}


def run_ivf_add(args, wl, ctx):
    """Streaming add: rows/s of batches added to an IVF-Flat index that
    already holds wl.N rows (each rank its own shard, so per-GPU work is
    fixed).  A batch that fits every list's spare slots is written in place;
    the line reports how many did."""
    import torch

    from rapidadb_b200._lib import C
    from rapidadb_b200.kmeans import kmeans
    from rapidadb_b200.sharded import shard_range

    rank, world, dev = ctx.rank, ctx.world, ctx.dev
    _C = C()
    N, d, B, nlist = wl["N"], wl["d"], wl["batch"], wl["nlist"]
    ntr = min(wl["train"], N)
    xtr = gen_mixture(0, ntr, d, wl, args.seed, torch.float32, dev)
    cent = kmeans(xtr, nlist, wl["iters"], 0.0, args.seed).centroids
    del xtr
    idx = _C.IVFFlatIndex(d, _C.Metric.L2, nlist, wl["nprobe"], _C.Precision.FP32)
    idx.set_quantizer(cent)
    lo, hi = shard_range(N, rank, world)
    CH = 4_194_304
    for a in range(lo, hi, CH):
        b = min(hi, a + CH)
        idx.add(gen_mixture(a, b, d, wl, args.seed, torch.float32, dev), torch.arange(a, b, device=dev))
    nb = args.warmup + 2 * args.steps
    base = N + rank * nb * B
    new = gen_mixture(base, base + nb * B, d, wl, args.seed, torch.float32, dev, salt=2)
    new_ids = torch.arange(base, base + nb * B, device=dev)
    state = {"i": 0, "in_place": 0}

    def add_batch():
        i = state["i"]
        cap0 = idx.capacity()
        idx.add(new[i * B:(i + 1) * B], new_ids[i * B:(i + 1) * B])
        state["in_place"] += int(idx.capacity() == cap0)
        state["i"] = i + 1

    n0 = idx.size()
    t = timed(ctx, add_batch, args.steps, args.warmup, 8)
    host = new[state["i"] * B:].cpu().pin_memory()
    buf = torch.empty((B, d), device=dev)
    torch.cuda.synchronize()
    ctx.barrier()
    t0 = time.perf_counter()
    for j in range(args.steps):
        buf.copy_(host[j * B:(j + 1) * B], non_blocking=True)
        idx.add(buf, new_ids[(state["i"] + j) * B:(state["i"] + j + 1) * B])
    torch.cuda.synchronize()
    e2e_s = ctx.max(time.perf_counter() - t0)
    assert idx.size() == n0 + nb * B
    res = None
    if rank == 0:
        flops = 2.0 * B * nlist * d
        peak = 148 * 128 * 2 * 1.965e9 / 1e12
        kern_ms, ms = t["kernel_ms"], t["ms"]
        ach = flops / (kern_ms * 1e-3) / 1e12 if kern_ms > 0 else None
        res = {
            "metric": "IVF-Flat streaming add (rows/s)",
            "value": round(world * B * args.steps / (ms * 1e-3), 1), "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Gaussian mixture)",
            "config": {"workload": args.workload, "rows_before": N, "dim": d, "batch_rows": B, "nlist": nlist},
            "rows_per_gpu": hi - lo, "capacity_after": idx.capacity(),
            "batches_in_place": "%d of %d" % (state["in_place"], args.warmup + args.steps),
            "l2_flush": "not needed: stored rows (%.2f GB per GPU) exceed L2" % ((hi - lo) * d * 4 / 1e9),
            "e2e": {"value": round(world * B * args.steps / e2e_s, 1), "unit": "rows/s",
                    "h2d_bytes_per_step": B * d * 4, "d2h_bytes_per_step": 0},
            "gpu_launches": t["launches"],
            "roofline": {"bound": "fma", "achieved": round(ach, 2) if ach else None, "peak": round(peak, 1),
                         "unit": "TFLOP/s", "frac": round(ach / peak, 4) if ach else None, "traffic": None,
                         "kernel": "simt_tma_scan_kernel<ARGMIN, exact> (list assignment)",
                         "kernel_ms": round(kern_ms, 4), "flops_per_launch": flops,
                         "peak_source": "nominal CUDA-core fp32 (148 SMs x 128 lanes x 2 x 1.965 GHz); "
                                        "no measured CUDA-core peak"},
            "clocks": t["clocks"],
            "host_ms_max_step": t["host_ms_max_step"],
            "device_allocs_in_timed_steps": t["device_allocs"],
        }
    return res


# ---------------------------------------------------------------- k-means

def run_kmeans(args, wl, ctx, name, steps, warmup):
    """Lloyd iterations over 10M x 768 bf16 points split over the ranks
    (centroid sums / counts all-reduced each iteration: strong scaling)."""
    import torch
    import torch.distributed as dist

    from rapidadb_b200._lib import C
    from rapidadb_b200.kmeans import init_centroids, kmeans
    from rapidadb_b200.sharded import shard_range

    rank, world, dev = ctx.rank, ctx.world, ctx.dev
    _C = C()
    N, d, K = wl["N"], wl["d"], wl["K"]
    lo, hi = shard_range(N, rank, world)
    x = gen_mixture(lo, hi, d, wl, args.seed, torch.bfloat16, dev)
    group = None if world == 1 else dist.group.WORLD
    cent = init_centroids(x, K, args.seed, group)
    state = {"c": cent}

    def iteration():
        lab, sq = _C.kmeans_assign(x, state["c"], False)
        sums, counts = _C.kmeans_update(x, lab, K)
        if world > 1:
            dist.all_reduce(sums)
            dist.all_reduce(counts)
        state["c"] = _C.kmeans_finalize(sums, counts, state["c"])
        return sq

    t = timed(ctx, iteration, steps, warmup, 8, {"assign": 8, "update": 16})
    sq = t["out"]
    inertia = sq.double().sum()
    if world > 1:
        dist.all_reduce(inertia)
    # e2e: the public training call (kmeans(): Lloyd iterations + the final
    # assignment and inertia) with the centroids read back to the host
    torch.cuda.synchronize()
    ctx.barrier()
    t0 = time.perf_counter()
    r = kmeans(x, K, max_iters=steps, tol=0.0, seed=args.seed, init=state["c"], group=group)
    c_host = r.centroids.cpu()
    e2e_s = ctx.max(time.perf_counter() - t0)
    res = None
    if rank == 0:
        _, bf16, bf16_sus, src = peaks()
        pk = bf16_sus or bf16
        flops = 2.0 * (hi - lo) * K * d
        kern_ms, ms = t["kernel_ms"], t["ms"]
        ach = flops / (kern_ms * 1e-3) / 1e12 if kern_ms > 0 else None
        res = {
            "metric": "k-means Lloyd iterations/s (assign + update + all-reduce)",
            "value": round(steps / (ms * 1e-3), 3), "unit": "iterations/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(ms / steps, 3), "higher_is_better": True,
            "scaling": "strong" if world > 1 else None, "dtype": "bf16",
            "data": "synthetic (seeded Gaussian mixture, 16,384 centres ~N(0,I), sigma 0.3)",
            "config": {"workload": name, "rows": N, "rows_per_gpu": hi - lo, "dim": d, "k": K},
            "inertia_after": float(inertia.item()),
            "phases_ms": t["phases"],
            "l2_flush": "not needed: points (%.1f GB per GPU) exceed L2" % ((hi - lo) * d * 2 / 1e9),
            "e2e": {"value": round(steps / e2e_s, 3), "unit": "iterations/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": int(c_host.numel() * 4 / steps),
                    "mode": "public kmeans() call: %d iterations + final assignment, centroids read back "
                            "(points resident on the device; the one-off upload is set-up)" % steps},
            "roofline": {"bound": "tensor", "achieved": round(ach, 1) if ach else None, "peak": pk,
                         "unit": "TFLOP/s", "frac": round(ach / pk, 4) if ach else None, "traffic": None,
                         "kernel": "tc_scan_pair_kernel<ARGMIN> (assign)", "kernel_ms": round(kern_ms, 3),
                         "flops_per_launch": flops, "algorithmic_unit": "2 d FLOP per (point, centroid)",
                         "peak_source": f"{src} bf16 dense ({'sustained' if bf16_sus else 'burst'}: the assign "
                                        f"runs for a quarter second under the power cap)"},
            "gpu_launches": t["launches"],
            "clocks": t["clocks"],
            "host_ms_max_step": t["host_ms_max_step"],
            "device_allocs_in_timed_steps": t["device_allocs"],
        }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = kmeans_cpu_baseline(x, state["c"], N, args.cpu_seconds)
    del x
    return res


def kmeans_cpu_baseline(x, cent, N, target_s):
    """One Lloyd iteration of the oracle (assign + update) on every host thread
    over a subsample of the points, as iterations/s over all N points."""
    import numpy as np

    import oracle

    nth = host_threads()
    c = cent.float().cpu().numpy()
    xs = x[:256].float().cpu().numpy()
    t0 = time.perf_counter()
    oracle.kmeans_assign(xs, c, nthreads=nth)
    per_pt = max((time.perf_counter() - t0) / len(xs), 1e-7)
    n = int(max(256, min(x.shape[0], target_s / per_pt)))
    xs = x[:n].float().cpu().numpy()
    t0 = time.perf_counter()
    lab, _, _ = oracle.kmeans_assign(xs, c, nthreads=nth)
    oracle.kmeans_update(xs, lab, c)
    el = time.perf_counter() - t0
    return {"value": round(n / el / N, 6), "unit": "iterations/s", "cores": nth, "kind": "port",
            "sample": f"one Lloyd iteration (assign + update) over {n:,} of the {N:,} points x {c.shape[0]:,} "
                      f"centroids, {el:.1f} s, scaled to all points"}


# ------------------------------------------------------------ reference arm

def run_reference(args, wl):
    """The reference path's CPU restatement (the oracle) on every host core:
    each step scores a bounded sample of the query batch against every stored
    row of the same synthetic table.  Under torchrun rank 0 alone runs."""
    import torch

    import oracle

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    N, d, k = wl["N"], wl["d"], wl["k"]
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["precision"]]
    xf = gen_rows(0, N, d, args.seed, wl["normalize"], tdt, dev).float().cpu().numpy()
    qf = gen_queries(wl["Q"] * world, d, args.seed, wl["normalize"], tdt, dev).float().cpu().numpy()
    nth = host_threads()
    t0 = time.perf_counter()
    oracle.flat_search(wl["metric"], qf[:2], xf, k, acc64=False, nthreads=nth)
    per_q = max((time.perf_counter() - t0) / 2, 1e-4)
    budget = 150.0 / max(args.steps + args.warmup, 1)  # whole run within a few minutes
    nq = int(max(1, min(len(qf), budget / per_q)))
    for _ in range(args.warmup):
        oracle.flat_search(wl["metric"], qf[:nq], xf, k, acc64=False, nthreads=nth)
    times = []
    for s in range(args.steps):
        off = (s * nq) % max(1, len(qf) - nq + 1)
        t0 = time.perf_counter()
        oracle.flat_search(wl["metric"], qf[off:off + nq], xf, k, acc64=False, nthreads=nth)
        times.append(time.perf_counter() - t0)
    el = sum(times)
    v = nq * args.steps / el
    sample = f"{nq} queries per step x {N:,} rows x {d} dims (fp32), all rows scored"
    return {
        "metric": "search QPS (exact flat search, recall@%d)" % k,
        "value": round(v, 3), "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * el / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) rows%s)" % (", L2-normalised" if wl["normalize"] else ""),
        "config": flat_config(args, wl, world),
        "impl": "reference",
        "cpu_baseline": {"value": round(v, 3), "unit": "queries/s", "cores": nth, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    wl = dict(WORKLOADS[args.workload])
    if args.rows:
        wl["N"] = args.rows
        wl.pop("N1", None)
    if args.queries:
        wl["Q"] = args.queries
    kind = wl.get("kind", "flat")
    if args.impl == "reference":
        res = run_reference(args, wl) if kind == "flat" else {
            "impl": "reference", "unavailable": "the CPU baseline of this workload is timed by bench.py "
            "--workload %s in its own run (cpu_baseline)" % args.workload}
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    import torch

    ctx = Ctx()
    if kind in ("ivf", "ivf_pq"):
        res = run_ivf(args, wl, ctx, args.workload, args.steps, args.warmup)
    elif kind == "kmeans":
        res = run_kmeans(args, wl, ctx, args.workload, args.steps, args.warmup)
    elif kind == "ivf_add":
        res = run_ivf_add(args, wl, ctx)
    else:
        res = run_flat(args, wl, ctx)
        if args.workload == "flat_cosine_bf16" and not args.no_workloads:
            subs = {}
            for name, steps, warmup in SUB_WORKLOADS:
                torch.cuda.empty_cache()
                swl = dict(WORKLOADS[name])
                fn = run_kmeans if swl["kind"] == "kmeans" else run_ivf
                sub = fn(args, swl, ctx, name, steps, warmup)
                if ctx.rank == 0:
                    subs[name] = sub
            if ctx.rank == 0:
                res["workloads"] = subs
    ctx.close()
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
