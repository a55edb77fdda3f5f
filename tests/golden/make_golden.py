"""Generate golden vectors by running the reference's own code on a GPU.

Requires the reference build in oracle/_ref/ (``make -C oracle ref``) and a
CUDA device.  Writes ``ref_golden.npz`` (reference outputs only; inputs are
regenerated from the seeds in cases.py) to the directory given as argv[1]
(default: this directory).

    python tests/golden/make_golden.py /tmp/golden
"""
from __future__ import annotations

import ctypes
import importlib.machinery
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

REF = os.path.join(HERE, "..", "..", "oracle", "_ref")


def load_ref_module():
    path = os.path.join(REF, "rapidadb_ref", "_C.so")
    loader = importlib.machinery.ExtensionFileLoader("_C", path)
    spec = importlib.util.spec_from_file_location("_C", path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def main(out_dir: str) -> None:
    C = load_ref_module()
    km = ctypes.CDLL(os.path.join(REF, "libref_kmeans.so"))
    dev = torch.device("cuda")
    out = {}
    metric = {"cosine": C.Metric.COSINE, "l2": C.Metric.L2, "dot_product": C.Metric.DOT_PRODUCT}

    for name, Q, N, d, seed in cases.DISTANCE_CASES:
        q, x = cases.distance_inputs(seed, Q, N, d)
        qt, xt = torch.from_numpy(q).to(dev), torch.from_numpy(x).to(dev)
        out[f"{name}_cosine"] = C.cosine_similarity(qt, xt).cpu().numpy()
        out[f"{name}_l2"] = C.l2_distance(qt, xt).cpu().numpy()
        out[f"{name}_dot_product"] = C.dot_product(qt, xt).cpu().numpy()

    for name, B, N, seed, ks in cases.TOPK_CASES:
        m = torch.from_numpy(cases.topk_input(seed, B, N)).to(dev)
        for k in ks:
            for largest in (True, False):
                v, i = C.topk(m, k, largest)
                out[f"{name}_k{k}_{int(largest)}_v"] = v.cpu().numpy()
                out[f"{name}_k{k}_{int(largest)}_i"] = i.cpu().numpy()

    for name, met, N, Q, d, k, seed in cases.FLAT_CASES:
        q, x = cases.flat_inputs(seed, N, Q, d)
        idx = C.FlatIndex(d, metric[met])
        # two adds, exercising the torch::cat append path (flat_index.cpp:42-43)
        h = N // 2
        idx.add(torch.from_numpy(x[:h]).to(dev))
        idx.add(torch.from_numpy(x[h:]).to(dev))
        dist, ids = idx.search(torch.from_numpy(q).to(dev), k)
        out[f"{name}_d"] = dist.cpu().numpy()
        out[f"{name}_i"] = ids.cpu().numpy()

    for name, N, d, K, seed in cases.KMEANS_CASES:
        x, c0 = cases.kmeans_inputs(seed, N, d, K)
        xt = torch.from_numpy(x).to(dev)
        ct = torch.from_numpy(c0).to(dev)
        lab = torch.empty(N, dtype=torch.int32, device=dev)
        dist = torch.empty(N, dtype=torch.float32, device=dev)
        rc = km.ref_kmeans_assign(ctypes.c_void_p(xt.data_ptr()), ctypes.c_void_p(ct.data_ptr()),
                                  ctypes.c_void_p(lab.data_ptr()), ctypes.c_void_p(dist.data_ptr()),
                                  N, K, d)
        assert rc == 0, rc
        newc = ct.clone()
        counts = torch.empty(K, dtype=torch.int32, device=dev)
        rc = km.ref_kmeans_update(ctypes.c_void_p(xt.data_ptr()), ctypes.c_void_p(lab.data_ptr()),
                                  ctypes.c_void_p(newc.data_ptr()),
                                  ctypes.c_void_p(counts.data_ptr()), N, K, d)
        assert rc == 0, rc
        out[f"{name}_labels"] = lab.cpu().numpy()
        out[f"{name}_dist"] = dist.cpu().numpy()
        out[f"{name}_centroids"] = newc.cpu().numpy()
        out[f"{name}_counts"] = counts.cpu().numpy()

    for name, N, d, K, seed, iters in cases.LLOYD_CASES:
        # the reference's assign and update kernels iterated (its Lloyd
        # driver, kmeans_cuda, is declared but never defined)
        x, c0 = cases.kmeans_inputs(seed, N, d, K)
        xt = torch.from_numpy(x).to(dev)
        ct = torch.from_numpy(c0).to(dev)
        lab = torch.empty(N, dtype=torch.int32, device=dev)
        dist = torch.empty(N, dtype=torch.float32, device=dev)
        counts = torch.empty(K, dtype=torch.int32, device=dev)
        for _ in range(iters):
            assert km.ref_kmeans_assign(ctypes.c_void_p(xt.data_ptr()), ctypes.c_void_p(ct.data_ptr()),
                                        ctypes.c_void_p(lab.data_ptr()), ctypes.c_void_p(dist.data_ptr()),
                                        N, K, d) == 0
            newc = ct.clone()
            assert km.ref_kmeans_update(ctypes.c_void_p(xt.data_ptr()), ctypes.c_void_p(lab.data_ptr()),
                                        ctypes.c_void_p(newc.data_ptr()), ctypes.c_void_p(counts.data_ptr()),
                                        N, K, d) == 0
            ct = newc
        assert km.ref_kmeans_assign(ctypes.c_void_p(xt.data_ptr()), ctypes.c_void_p(ct.data_ptr()),
                                    ctypes.c_void_p(lab.data_ptr()), ctypes.c_void_p(dist.data_ptr()),
                                    N, K, d) == 0
        out[f"{name}_centroids"] = ct.cpu().numpy()
        out[f"{name}_labels"] = lab.cpu().numpy()
        out[f"{name}_dist"] = dist.cpu().numpy()

    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, "ref_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, device {torch.cuda.get_device_name()}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
