#!/usr/bin/env python
"""Search-QPS benchmark of the fused flat search (one JSON line on rank 0).

Workload (default ``flat_cosine_bf16``): exact cosine search, 1,000,000 stored
rows x 768 dims in bf16 (i.i.d. N(0,1) rows, L2-normalised, then rounded),
queries of the same distribution, k = 100.  With N GPUs (torchrun, one
process per GPU) the 1,000,000 rows are split by rows across the ranks and the
query batch is 1,024 x N (per-GPU work fixed: "scaling": "weak"); each step is
local fused search -> NCCL all-gather of the [Q, k] lists -> merge kernel.

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
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # BASELINE config "Flat cosine search ... 1,000,000 x 768 bf16 ... 1,024 queries, k=100"
    "flat_cosine_bf16": dict(N=1_000_000, d=768, Q=1024, k=100, metric="cosine", precision="bf16",
                             normalize=True),
    # BASELINE config "Flat exact L2 search: fp32 base N=100,000 x 768, 32 queries, k=10"
    "flat_l2_fp32": dict(N=100_000, d=768, Q=32, k=10, metric="l2", precision="fp32",
                         normalize=False),
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


# ------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


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
    searcher = ShardedSearch(db, largest)

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
    lib.rdb_timing_enable(1)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out_d, out_i = step(q)
    e1.record()
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

    # ---- recall against exact fp32 search over the same stored values
    nrec = min(64, Q)
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
        launches_per_step = 6 if wl["precision"] != "fp32" or N >= 4096 else 4
        if world > 1:
            launches_per_step += 1
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
                "l2_flush": "not needed: stored rows (%.2f GB) exceed L2 (126 MB)" % (
                    n_local * d * (2 if wl["precision"] != "fp32" else 4) / 1e9),
                "recall_at_k_vs_fp32_exact": round(recall, 5),
            },
            "e2e": {"value": round(Q * args.steps / e2e_s, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {
                "bound": "tensor",
                "achieved": round(achieved, 1) if achieved else None,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4) if achieved else None,
                "traffic": None,
                "kernel": "tc_scan_kernel<FILTER> (main pass)",
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


def main():
    args = parse()
    wl = dict(WORKLOADS[args.workload])
    if args.rows:
        wl["N"] = args.rows
    if args.queries:
        wl["Q"] = args.queries
    res = run_reference(args, wl) if args.impl == "reference" else run_ours(args, wl)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
