#!/usr/bin/env python
"""Search-QPS benchmark of the fused flat search (one JSON line on rank 0).

Workload (default ``flat_cosine_bf16``): exact cosine search, 1,000,000 stored
rows x 768 dims in bf16 (i.i.d. N(0,1) rows, L2-normalised, then rounded),
queries of the same distribution, k = 100.  With N GPUs (torchrun, one
process per GPU) the 1,000,000 rows are split by rows across the ranks and the
query batch is 1,024 x N (per-GPU work fixed: "scaling": "weak"); each step is
local fused search -> NCCL all-to-all of the [Q, k] lists by query slice ->
merge kernel on the rank owning the slice (``--results replicated``: an
all-gather and a merge of the whole batch on every rank).

* ``value``  - queries/s with queries already resident in HBM, timed with CUDA
               events between barriers, max over ranks.  The stored rows
               (1.5 GB) exceed L2 (126 MB), so no flush is needed.
* ``e2e``    - the same through RapidaDB's public search call with the query
               batch copied from pinned host memory each step and the results
               read back to the host.
* ``roofline`` - the dominant kernel (tcgen05 main scan): 2 Q N d FLOPs per
               launch over its CUDA-event duration, against the measured bf16
               dense peak.
* ``cpu_baseline`` - the CPU oracle (fp32 restatement of the reference's
               exact search) on the host cores, on a sample of the queries.

``--impl reference`` times the reference path's CPU restatement (the oracle)
on the same workload instead (the reference has no CPU implementation of its
own; its GPU kernels are SIMT fp32 and need no tensor cores).
"""
from __future__ import annotations

import argparse
import json
import os
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
    # sample; 10,000 queries; nprobe=32; k=10
    "ivf_flat": dict(kind="ivf", N=10_000_000, d=128, Q=10_000, k=10, metric="l2", nlist=4096,
                     nprobe=32, ncentres=1024, spread=2.0, sigma=1.0, train=1_000_000, iters=20,
                     uint8=False),
    # IVF-PQ (sharded across up to 8 GPUs): 100,000,000 x 128 uint8-valued rows (stored
    # fp32); nlist=16,384; M=16 x 256; 10,000 queries; nprobe=64; k=10
    "ivf_pq": dict(kind="ivf_pq", N=100_000_000, d=128, Q=10_000, k=10, metric="l2", nlist=16384,
                   nprobe=64, M=16, ksub=256, ncentres=1024, spread=2.0, sigma=1.0, train=262_144,
                   iters=10, uint8=True),
    # streaming add into the IVF-Flat workload's index: batches of 10,000 rows
    # appended to the 10,000,000 stored rows
    "ivf_add": dict(kind="ivf_add", N=10_000_000, d=128, batch=10_000, nlist=4096, nprobe=32,
                    ncentres=1024, spread=2.0, sigma=1.0, train=1_000_000, iters=20, uint8=False),
    # k-means: 10,000,000 x 768 bf16 points from a mixture of 16,384 Gaussians (centres
    # ~N(0,I), sigma=0.3); K=16,384; seeded random-row init; 20 Lloyd iterations
    "kmeans": dict(kind="kmeans", N=10_000_000, d=768, K=16384, iters=20, ncentres=16384,
                   spread=1.0, sigma=0.3),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="flat_cosine_bf16", choices=sorted(WORKLOADS))
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target host time of the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--rows", type=int, default=0, help="override the workload's stored rows")
    ap.add_argument("--queries", type=int, default=0, help="override the per-GPU query batch")
    ap.add_argument("--results", default="owner", choices=["owner", "replicated"],
                    help="flat search on N > 1 GPUs: each rank returns the answers of its query slice "
                         "(owner) or of the whole batch (replicated)")
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
    the same mixture as the stored rows).  uint8 workloads scale to 16 units per sigma around 128 and clip to
    [0, 255] (integer values stored as floats)."""
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
        self._nvml = None

    def _handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.cuda_index).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid)

    def start(self):
        try:
            self._nvml, h = self._handle()
            nv = self._nvml
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
            self._nvml = None

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


# --------------------------------------------------------------- CPU baseline

def cpu_baseline(xf, qf, wl, target_s):
    """The oracle (fp32 restatement of the reference's exact search) on all
    host threads over a sample of the queries against every stored row."""
    import numpy as np

    import oracle

    nth = oracle.max_threads()
    t0 = time.perf_counter()
    oracle.flat_search(wl["metric"], qf[:2], xf, wl["k"], acc64=False, nthreads=nth)
    t1 = time.perf_counter() - t0
    per_q = max(t1 / 2, 1e-4)
    nq = int(max(2, min(len(qf), target_s / per_q)))
    t0 = time.perf_counter()
    oracle.flat_search(wl["metric"], qf[:nq], xf, wl["k"], acc64=False, nthreads=nth)
    el = time.perf_counter() - t0
    return {"value": nq / el, "unit": "queries/s", "cores": nth, "kind": "port",
            "sample": f"{nq} queries x {xf.shape[0]:,} rows x {xf.shape[1]} dims (fp32 upcast of the "
                      f"stored values), all rows scored, {el:.1f} s"}


# ------------------------------------------------------------------ our arm

def run_ours(args, wl):
    import numpy as np
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from rapidadb_b200._lib import C
    from rapidadb_b200.config import IndexConfig, Metric, Precision
    from rapidadb_b200.index import RapidaDB
    from rapidadb_b200.sharded import ShardedSearch, shard_range

    _C = C()
    N, d, k = wl["N"], wl["d"], wl["k"]
    Q = wl["Q"] * world
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["precision"]]
    lo, hi = shard_range(N, rank, world)
    x = gen_rows(lo, hi, d, args.seed, wl["normalize"], tdt, dev)
    q = gen_queries(Q, d, args.seed, wl["normalize"], tdt, dev)
    cfg = IndexConfig(dim=d, metric=Metric(wl["metric"]), precision=Precision(wl["precision"]))
    db = RapidaDB(config=cfg)
    db.add(x, torch.arange(lo, hi, device=dev, dtype=torch.long))
    largest = wl["metric"] != "l2"
    searcher = ShardedSearch(db, largest, results=args.results if world > 1 else "replicated")
    own_lo, own_hi = searcher.owned_range(Q)

    def step(qdev):
        return searcher.search(qdev, k)

    # ---- device-resident timing
    for _ in range(args.warmup):
        step(q)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local_rank)
    clocks.start()
    import ctypes

    lib = ctypes.CDLL(os.path.join(ROOT, "rapidadb_b200", "librdb_kernels.so"))
    lib.rdb_launch_count.restype = ctypes.c_ulonglong
    lib.rdb_timing_enable(1)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n_launch0 = lib.rdb_launch_count()
    e0.record()
    for _ in range(args.steps):
        out_d, out_i = step(q)
    e1.record()
    n_launches = int(lib.rdb_launch_count() - n_launch0)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    tot = ctypes.c_double(0.0)
    nl = ctypes.c_int(0)
    lib.rdb_timing_read(ctypes.byref(tot), ctypes.byref(nl), 1)
    lib.rdb_timing_enable(0)
    clk = clocks.stop()
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    kernel_ms = tot.value / max(nl.value, 1)

    # ---- end to end through the public API with host buffers
    q_host = q.cpu().pin_memory()
    h2d = q_host.numel() * q_host.element_size()
    qbuf = torch.empty_like(q)
    for _ in range(max(1, args.warmup // 2)):
        qbuf.copy_(q_host, non_blocking=True)
        rd, ri = step(qbuf)
        rd.cpu(), ri.cpu()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    d2h = 0
    for _ in range(args.steps):
        qbuf.copy_(q_host, non_blocking=True)
        rd, ri = step(qbuf)
        if rank == 0:
            hd, hi_ = rd.cpu(), ri.cpu()
            d2h = hd.numel() * hd.element_size() + hi_.numel() * hi_.element_size()
        else:
            torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_t.item())
    e2e_seq_s = e2e_s
    e2e_mode = "sequential: each step copies its batch in, searches, reads the results back"
    if world == 1:
        # the public pipelined API (rapidadb_b200.pipeline.AsyncBatchSearcher):
        # the same `steps` host batches, each staged in pinned memory, copied
        # in, searched and read back on one of two worker streams, so one
        # batch's copies overlap another's kernels
        from rapidadb_b200.pipeline import AsyncBatchSearcher

        q_np = q_host.view(torch.int16).numpy() if q_host.dtype == torch.bfloat16 else q_host.numpy()
        stream_in = np.concatenate([q_np] * args.steps)
        src = torch.from_numpy(stream_in).view(q_host.dtype) if q_host.dtype == torch.bfloat16 else stream_in
        pipe = AsyncBatchSearcher(db, num_streams=2)
        pipe.search_host(src[:2 * Q], k, batch_size=Q)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        pipe.search_host(src, k, batch_size=Q)
        e2e_s = time.perf_counter() - t0
        pipe.close()
        e2e_mode = "pipelined: AsyncBatchSearcher, 2 worker streams, one batch per step"

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
    got = out_i[:nrec].cpu().numpy()
    ref = ti.cpu().numpy()
    recall = float(np.mean([len(set(a) & set(b)) / k for a, b in zip(got, ref)]))

    result = None
    if rank == 0:
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
            peak, peak_src = float(peaks["bf16_tflops"]), "measured (burst)"
        except Exception:
            peak, peak_src = 1590.0, "fallback"
        n_local = hi - lo
        flops = 2.0 * Q * n_local * d
        achieved = flops / (kernel_ms * 1e-3) / 1e12 if kernel_ms > 0 else None
        qps = Q * args.steps / (ms * 1e-3)
        result = {
            "metric": "search QPS (exact flat search, recall@%d)" % k,
            "value": round(qps, 1),
            "unit": "queries/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": wl["precision"],
            "data": "synthetic (seeded N(0,1) rows%s)" % (", L2-normalised" if wl["normalize"] else ""),
            "config": {
                "workload": args.workload,
                "rows": N, "dim": d, "queries_per_step": Q, "k": k, "metric": wl["metric"],
                "precision": wl["precision"], "rows_per_gpu": n_local,
                "parallelism": f"row-shard x{world}" if world > 1 else "single GPU",
                **({"results": ("owner: rank r merges and returns the answers of its 1/%d slice of the "
                                "query batch (all-to-all of the per-rank lists)" % world)
                    if args.results == "owner" else "replicated: every rank merges the whole batch "
                                                    "(all-gather of the per-rank lists)"}
                   if world > 1 else {}),
                "l2_flush": "not needed: stored rows (%.2f GB) exceed L2 (126 MB)" % (
                    n_local * d * (2 if wl["precision"] != "fp32" else 4) / 1e9),
                "recall_at_k_vs_fp32_exact": round(recall, 5),
            },
            "e2e": {"value": round(Q * args.steps / e2e_s, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "mode": e2e_mode,
                    "sequential_value": round(Q * args.steps / e2e_seq_s, 1)},
            "gpu_launches": n_launches,
            "roofline": {
                "bound": "tensor",
                "achieved": round(achieved, 1) if achieved else None,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4) if achieved else None,
                # DRAM bytes of one main-scan launch: ncu capture of the
                # 262,144-row launch (profiles/tc_scan_flat_262kx768_full.md:
                # 408.7 MB read + 9.4 MB written = 1,595 B per row) scaled by
                # the rows of this launch; bf16 tensor-core path only
                "traffic": (round(1595.0 * n_local) if wl["precision"] != "fp32" else None),
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of a 262,144-row "
                                   "launch, scaled by rows" if wl["precision"] != "fp32" else None),
                "kernel": ("tc_scan_pair_kernel<FILTER> (CTA pair, main pass)" if Q > 128
                           else "tc_scan_kernel<FILTER> (main pass)"),
                "kernel_ms": round(kernel_ms, 4),
                "flops_per_launch": flops,
                "peak_source": peak_src,
            },
            "clocks": clk,
        }
        if wl["precision"] == "fp32":
            result["roofline"].update({"bound": "hbm", "unit": "GB/s", "kernel": "simt_scan_kernel<FILTER>"})
            byt = n_local * d * 4 + Q * d * 4
            ach = byt / (kernel_ms * 1e-3) / 1e9
            try:
                pk = float(peaks["hbm_gbs"])
            except Exception:
                pk = 6650.0
            result["roofline"].update({"achieved": round(ach, 1), "peak": pk, "frac": round(ach / pk, 4),
                                       "bytes_per_launch": byt})
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        xf = x.float().cpu().numpy()
        qf = q[:256].float().cpu().numpy()
        result["cpu_baseline"] = cpu_baseline(xf, qf, wl, args.cpu_seconds)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


# ------------------------------------------------------------ reference arm

def run_reference(args, wl):
    """The reference path's CPU restatement (the oracle) on the host cores:
    each step scores a bounded sample of the query batch against every stored
    row of the same synthetic table."""
    import numpy as np
    import torch

    import oracle

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    N, d, k = wl["N"], wl["d"], wl["k"]
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["precision"]]
    xf = gen_rows(0, N, d, args.seed, wl["normalize"], tdt, dev).float().cpu().numpy()
    qf = gen_queries(wl["Q"], d, args.seed, wl["normalize"], tdt, dev).float().cpu().numpy()
    nth = oracle.max_threads()
    t0 = time.perf_counter()
    oracle.flat_search(wl["metric"], qf[:2], xf, k, acc64=False, nthreads=nth)
    per_q = max((time.perf_counter() - t0) / 2, 1e-4)
    budget = 150.0 / max(args.steps + args.warmup, 1)  # whole run within a few minutes
    nq = int(max(1, min(wl["Q"], budget / per_q)))
    for w in range(args.warmup):
        oracle.flat_search(wl["metric"], qf[:nq], xf, k, acc64=False, nthreads=nth)
    times = []
    for s in range(args.steps):
        off = (s * nq) % max(1, wl["Q"] - nq + 1)
        t0 = time.perf_counter()
        oracle.flat_search(wl["metric"], qf[off:off + nq], xf, k, acc64=False, nthreads=nth)
        times.append(time.perf_counter() - t0)
    el = sum(times)
    v = nq * args.steps / el
    sample = f"{nq} queries per step x {N:,} rows x {d} dims (fp32), all rows scored"
    return {
        "metric": "search QPS (exact flat search, recall@%d)" % k,
        "value": round(v, 3), "unit": "queries/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * el / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) rows%s)" % (", L2-normalised" if wl["normalize"] else ""),
        "config": {"workload": args.workload, "rows": N, "dim": d, "queries_per_step": wl["Q"], "k": k,
                   "metric": wl["metric"], "precision": wl["precision"]},
        "impl": "reference",
        "cpu_baseline": {"value": round(v, 3), "unit": "queries/s", "cores": nth, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _dist_setup():
    import datetime

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    return rank, world, local_rank, dev


def _timed(fn, steps, warmup, world, tag_mask, local_rank):
    """CUDA-event time of `steps` calls (max over ranks), the tagged kernels'
    device time, and the clock record; `_timed.launches` = this library's
    kernel launches inside the timed region."""
    import ctypes

    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    lib = ctypes.CDLL(os.path.join(ROOT, "rapidadb_b200", "librdb_kernels.so"))
    lib.rdb_launch_count.restype = ctypes.c_ulonglong
    clocks = ClockSampler(local_rank)
    clocks.start()
    lib.rdb_timing_enable(tag_mask)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n_launch0 = lib.rdb_launch_count()
    e0.record()
    out = None
    for _ in range(steps):
        out = fn()
    e1.record()
    _timed.launches = int(lib.rdb_launch_count() - n_launch0)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    tot, nl = ctypes.c_double(0.0), ctypes.c_int(0)
    lib.rdb_timing_read(ctypes.byref(tot), ctypes.byref(nl), 1)
    lib.rdb_timing_enable(0)
    clk = clocks.stop()
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), tot.value / max(nl.value, 1), nl.value, clk, out


def _peaks():
    try:
        p = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def run_ivf(args, wl):
    """IVF-Flat / IVF-PQ search QPS.  Rows are sharded over the ranks (every
    rank trains the same quantizer from the same seeded sample); the query
    batch is wl.Q x N (per-GPU scan work fixed: weak scaling); the coarse probe
    is split across ranks and the list table all-gathered."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from rapidadb_b200._lib import C
    from rapidadb_b200.kmeans import kmeans, train_pq
    from rapidadb_b200.sharded import ShardedIVFSearch, shard_range

    rank, world, local_rank, dev = _dist_setup()
    _C = C()
    N, d, k, nlist, nprobe = wl["N"], wl["d"], wl["k"], wl["nlist"], wl["nprobe"]
    Q = wl["Q"] * world
    pq = wl["kind"] == "ivf_pq"
    t_setup = time.perf_counter()
    # quantizer: k-means on a seeded sample of the table (identical on every rank)
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
    searcher = ShardedIVFSearch(idx, largest=False)
    tag = 4 if pq else 2
    ms, kern_ms, nl, clk, out = _timed(lambda: searcher.search(q, k), args.steps, args.warmup, world, tag,
                                       local_rank)
    out_d, out_i = out
    # e2e: host query batch in, results out, each step
    q_host = q.cpu().pin_memory()
    qbuf = torch.empty_like(q)
    for _ in range(max(1, args.warmup // 2)):
        qbuf.copy_(q_host, non_blocking=True)
        rd, ri = searcher.search(qbuf, k)
        rd.cpu(), ri.cpu()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        qbuf.copy_(q_host, non_blocking=True)
        rd, ri = searcher.search(qbuf, k)
        rd.cpu(), ri.cpu()
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_t.item())
    # recall@k against exact search over the same rows (first 100 queries)
    nrec = min(100, Q)
    exact_rows = []
    for a in range(lo, hi, CH):
        b = min(hi, a + CH)
        xb = gen_mixture(a, b, d, wl, args.seed, torch.float32, dev)
        xv = _C.row_values(_C.Metric.L2, xb, d)
        dd, ii = _C.search_rows(_C.Metric.L2, xb, d, xv, q[:nrec], k, None, a)
        exact_rows.append((dd, ii))
        del xb
    ev = torch.cat([e[0] for e in exact_rows], 1)
    ei = torch.cat([e[1] for e in exact_rows], 1)
    order = torch.argsort(ev, dim=1)[:, :k]
    tv, ti = torch.gather(ev, 1, order), torch.gather(ei, 1, order)
    if world > 1:
        gv = torch.empty((world * nrec, k), device=dev)
        gi = torch.empty((world * nrec, k), device=dev, dtype=torch.long)
        dist.all_gather_into_tensor(gv, tv.contiguous())
        dist.all_gather_into_tensor(gi, ti.contiguous())
        gv, gi = gv.view(world, nrec, k).permute(1, 0, 2).reshape(nrec, -1), gi.view(world, nrec, k).permute(1, 0, 2).reshape(nrec, -1)
        o2 = torch.argsort(gv, dim=1)[:, :k]
        ti = torch.gather(gi, 1, o2)
    got = out_i[:nrec].cpu().numpy()
    ref = ti.cpu().numpy()
    recall = float(np.mean([len(set(a) & set(b)) / k for a, b in zip(got, ref)]))
    sizes = idx.list_sizes().double()
    probes = searcher.probe(q)
    # algorithmic bytes of the local scan: every probed list's rows (or codes) once per probing query
    scanned = float(sizes[probes.flatten()].sum().item())
    bpr = wl["M"] if pq else d * 4
    res = None
    if rank == 0:
        hbm, _, src = _peaks()
        alg_bytes = scanned * bpr
        ach = alg_bytes / (kern_ms * 1e-3) / 1e9 if kern_ms > 0 else None
        qps = Q * args.steps / (ms * 1e-3)
        res = {
            "metric": f"search QPS ({'IVF-PQ' if pq else 'IVF-Flat'}, nprobe={nprobe}, recall@{k})",
            "value": round(qps, 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8" if pq else "f32",
            "data": "synthetic (seeded Gaussian mixture%s)" % (", uint8-valued" if wl.get("uint8") else ""),
            "config": {"workload": args.workload, "rows": N, "rows_per_gpu": hi - lo, "dim": d,
                       "queries_per_step": Q, "k": k, "nlist": nlist, "nprobe": nprobe,
                       **({"pq_m": wl["M"], "pq_k": wl["ksub"]} if pq else {}),
                       "train_rows": ntr, "train_iters": wl["iters"], "setup_s": round(t_setup, 1),
                       "recall_at_k_vs_exact": round(recall, 4),
                       "l2_flush": ("not needed: stored %s (%.2f GB per GPU) exceed L2 (126 MB)" if
                                    (hi - lo) * bpr > 126e6 else
                                    "none: stored %s (%.2f GB per GPU) fit in L2 at this reduced size") % (
                           "codes" if pq else "rows", (hi - lo) * bpr / 1e9)},
            "e2e": {"value": round(Q * args.steps / e2e_s, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(q.numel() * 4), "d2h_bytes_per_step": int(Q * k * 12)},
            "gpu_launches": _timed.launches,
            "roofline": {"bound": "hbm", "achieved": round(ach, 1) if ach else None, "peak": hbm, "unit": "GB/s",
                         "frac": round(ach / hbm, 4) if ach else None, "traffic": None,
                         "kernel": ("ivfpq_search_kernel<%d> (query-major)" % wl["M"] if idx.query_major()
                                    else "ivfpq_scan_kernel") if pq else "ivf_flat_scan_kernel",
                         "kernel_ms": round(kern_ms, 4), "bytes_per_launch": alg_bytes,
                         "bytes_definition": (
                             "sum over (query, probed list) of the list's stored code bytes (query-major "
                             "count; the kernel also reads a 4-byte per-row term, not counted; lists shared by "
                             "queries running at the same time are served from L2, so frac may exceed 1)"
                             if pq else
                             "sum over (query, probed list) of the list's stored row bytes (query-major count; "
                             "the list-major scan reads each list once per 32-query chunk, so frac may exceed "
                             "1)"),
                         "peak_source": src},
            "clocks": clk,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


def run_ivf_add(args, wl):
    """Streaming add: rows/s of batches added to an IVF-Flat index that
    already holds wl.N rows (the ivf_flat workload's table; each rank its own
    shard, so per-GPU work is fixed).  A batch that fits every list's spare
    slots is written in place; the line reports how many did."""
    import torch
    import torch.distributed as dist

    from rapidadb_b200._lib import C
    from rapidadb_b200.kmeans import kmeans
    from rapidadb_b200.sharded import shard_range

    rank, world, local_rank, dev = _dist_setup()
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
    # new rows (ids past the table), generated before the timed region
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
    ms, kern_ms, nl, clk, _ = _timed(add_batch, args.steps, args.warmup, world, 8, local_rank)
    # e2e: each batch copied in from pinned host memory, then added
    host = new[state["i"] * B:].cpu().pin_memory()
    buf = torch.empty((B, d), device=dev)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for j in range(args.steps):
        buf.copy_(host[j * B:(j + 1) * B], non_blocking=True)
        idx.add(buf, new_ids[(state["i"] + j) * B:(state["i"] + j + 1) * B])
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_t.item())
    assert idx.size() == n0 + nb * B
    res = None
    if rank == 0:
        # exact list assignment of each batch: 2 B nlist d FLOP on the CUDA
        # cores (the reference's sequential fp32 arithmetic)
        flops = 2.0 * B * nlist * d
        peak = 148 * 128 * 2 * 1.965e9 / 1e12
        ach = flops / (kern_ms * 1e-3) / 1e12 if kern_ms > 0 else None
        res = {
            "metric": "IVF-Flat streaming add (rows/s)",
            "value": round(world * B * args.steps / (ms * 1e-3), 1), "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Gaussian mixture)",
            "config": {"workload": args.workload, "rows_before": N, "rows_per_gpu": hi - lo, "dim": d,
                       "batch_rows": B, "nlist": nlist, "capacity_after": idx.capacity(),
                       "batches_in_place": "%d of %d" % (state["in_place"], args.warmup + args.steps),
                       "l2_flush": "not needed: stored rows (%.2f GB per GPU) exceed L2" % ((hi - lo) * d * 4 / 1e9)},
            "e2e": {"value": round(world * B * args.steps / e2e_s, 1), "unit": "rows/s",
                    "h2d_bytes_per_step": B * d * 4, "d2h_bytes_per_step": 0},
            "gpu_launches": _timed.launches,
            "roofline": {"bound": "fma", "achieved": round(ach, 2) if ach else None, "peak": round(peak, 1),
                         "unit": "TFLOP/s", "frac": round(ach / peak, 4) if ach else None, "traffic": None,
                         "kernel": "simt_tma_scan_kernel<ARGMIN, exact> (list assignment)",
                         "kernel_ms": round(kern_ms, 4), "flops_per_launch": flops,
                         "peak_source": "nominal CUDA-core fp32 (148 SMs x 128 lanes x 2 x 1.965 GHz); "
                                        "no measured CUDA-core peak"},
            "clocks": clk,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


def run_kmeans(args, wl):
    """k-means Lloyd iterations over 10M x 768 bf16 rows sharded over the
    ranks (centroid sums / counts all-reduced each iteration: strong scaling)."""
    import torch
    import torch.distributed as dist

    from rapidadb_b200._lib import C
    from rapidadb_b200.kmeans import init_centroids
    from rapidadb_b200.sharded import shard_range

    rank, world, local_rank, dev = _dist_setup()
    _C = C()
    N, d, K = wl["N"], wl["d"], wl["K"]
    lo, hi = shard_range(N, rank, world)
    x = gen_mixture(lo, hi, d, wl, args.seed, torch.bfloat16, dev)
    cent = init_centroids(x, K, args.seed, None if world == 1 else dist.group.WORLD)
    state = {"c": cent}

    def iteration():
        lab, sq = _C.kmeans_assign(x, state["c"], False)
        sums, counts = _C.kmeans_update(x, lab, K)
        if world > 1:
            dist.all_reduce(sums)
            dist.all_reduce(counts)
        state["c"] = _C.kmeans_finalize(sums, counts, state["c"])
        return sq

    ms, kern_ms, nl, clk, sq = _timed(iteration, args.steps, args.warmup, world, 8, local_rank)
    inertia = sq.double().sum()
    if world > 1:
        dist.all_reduce(inertia)
    res = None
    if rank == 0:
        _, bf16, src = _peaks()
        flops = 2.0 * (hi - lo) * K * d
        ach = flops / (kern_ms * 1e-3) / 1e12 if kern_ms > 0 else None
        res = {
            "metric": "k-means Lloyd iterations/s (assign + update + all-reduce)",
            "value": round(args.steps / (ms * 1e-3), 3), "unit": "iterations/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded Gaussian mixture, 16,384 centres ~N(0,I), sigma 0.3)",
            "config": {"workload": args.workload, "rows": N, "rows_per_gpu": hi - lo, "dim": d, "k": K,
                       "inertia_after": float(inertia.item()),
                       "l2_flush": "not needed: rows (%.1f GB per GPU) exceed L2" % ((hi - lo) * d * 2 / 1e9)},
            "roofline": {"bound": "tensor", "achieved": round(ach, 1) if ach else None, "peak": bf16,
                         "unit": "TFLOP/s", "frac": round(ach / bf16, 4) if ach else None, "traffic": None,
                         "kernel": "tc_scan_pair_kernel<ARGMIN> (assign)", "kernel_ms": round(kern_ms, 3),
                         "flops_per_launch": flops, "peak_source": src},
            "gpu_launches": _timed.launches,
            "clocks": clk,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


def main():
    args = parse()
    wl = dict(WORKLOADS[args.workload])
    if args.rows:
        wl["N"] = args.rows
    if args.queries:
        wl["Q"] = args.queries
    kind = wl.get("kind", "flat")
    if args.impl == "reference":
        res = run_reference(args, wl) if kind == "flat" else {
            "impl": "reference", "unavailable": "the CPU baseline of this workload is timed by bench.py "
            "--workload %s in its own run (cpu_baseline)" % args.workload}
    elif kind == "ivf" or kind == "ivf_pq":
        res = run_ivf(args, wl)
    elif kind == "kmeans":
        res = run_kmeans(args, wl)
    elif kind == "ivf_add":
        res = run_ivf_add(args, wl)
    else:
        res = run_ours(args, wl)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
