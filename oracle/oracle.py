"""ctypes front end of ``liborc.so``, the C restatement in ``cpu_oracle.c``.

TEST INFRASTRUCTURE ONLY: what the parity tests compare against, and the
timed CPU baseline.  Arrays are numpy; every function returns fresh arrays.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liborc.so")
_lib = None

METRIC = {"cosine": 0, "l2": 1, "dot_product": 2}

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64 = ctypes.c_int64
_int = ctypes.c_int


def build() -> str:
    """Compile liborc.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE, "liborc.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_max_threads.restype = _int
        L.orc_distance.argtypes = [_int, _f32p, _i64, _f32p, _i64, _int, _f32p, _int, _int]
        L.orc_topk.argtypes = [_f32p, _i64, _i64, _int, _int, _f32p, _i64p, _int]
        L.orc_flat_search.argtypes = [_int, _f32p, _i64, _f32p, _i64, _int, _int, _i64p,
                                      _f32p, _i64p, _int, _int]
        L.orc_topk_merge.argtypes = [_int, _f32p, _i64p, _int, _i64, _int, _int, _f32p, _i64p]
        L.orc_kmeans_assign.argtypes = [_f32p, _i64, _int, _f32p, _int, _i32p, _f32p, _f32p, _int]
        L.orc_kmeans_update.argtypes = [_f32p, _i64, _int, _i32p, _int, _f32p, _i64p]
        L.orc_kmeans.argtypes = [_f32p, _i64, _int, _int, _int, ctypes.c_float, _f32p, _i32p,
                                 _f64p, _int]
        L.orc_kmeans.restype = _int
        L.orc_ivf_flat_search.argtypes = [_int, _f32p, _i64, _int, _f32p, _int, _i64p, _f32p,
                                          _i64p, _int, _int, _f32p, _i64p, _int]
        L.orc_pq_encode.argtypes = [_f32p, _i64, _int, _i32p, _f32p, _f32p, _int, _int, _u8p,
                                    _int]
        L.orc_ivfpq_search.argtypes = [_f32p, _i64, _int, _f32p, _int, _i64p, _u8p, _i64p,
                                       _f32p, _int, _int, _int, _int, _f32p, _i64p, _int]
        _lib = L
    return _lib


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _p(a: np.ndarray, ptype):
    return a.ctypes.data_as(ptype)


def max_threads() -> int:
    """Host threads this process may run on (its CPU affinity).  Not
    omp_get_max_threads(), which follows OMP_NUM_THREADS (torchrun sets it to
    1); every call here passes this count explicitly."""
    return len(os.sched_getaffinity(0))


def distance(metric: str, q: np.ndarray, x: np.ndarray, acc64: bool = True,
             nthreads: int = 0) -> np.ndarray:
    q = _c(q, np.float32)
    x = _c(x, np.float32)
    out = np.empty((q.shape[0], x.shape[0]), np.float32)
    lib().orc_distance(METRIC[metric], _p(q, _f32p), q.shape[0], _p(x, _f32p), x.shape[0],
                       q.shape[1], _p(out, _f32p), int(acc64), nthreads)
    return out


def topk(dist: np.ndarray, k: int, largest: bool = True,
         nthreads: int = 0) -> Tuple[np.ndarray, np.ndarray]:
    dist = _c(dist, np.float32)
    B, N = dist.shape
    v = np.empty((B, k), np.float32)
    i = np.empty((B, k), np.int64)
    lib().orc_topk(_p(dist, _f32p), B, N, k, int(largest), _p(v, _f32p), _p(i, _i64p), nthreads)
    return v, i


def flat_search(metric: str, q: np.ndarray, x: np.ndarray, k: int,
                ids: Optional[np.ndarray] = None, acc64: bool = True,
                nthreads: int = 0) -> Tuple[np.ndarray, np.ndarray]:
    q = _c(q, np.float32)
    x = _c(x, np.float32)
    Q, d = q.shape
    out_d = np.empty((Q, k), np.float32)
    out_i = np.empty((Q, k), np.int64)
    idp = None
    if ids is not None:
        ids = _c(ids, np.int64)
        idp = _p(ids, _i64p)
    lib().orc_flat_search(METRIC[metric], _p(q, _f32p), Q, _p(x, _f32p), x.shape[0], d, k, idp,
                          _p(out_d, _f32p), _p(out_i, _i64p), int(acc64), nthreads)
    return out_d, out_i


def topk_merge(vals: np.ndarray, ids: np.ndarray, k: int,
               largest: bool) -> Tuple[np.ndarray, np.ndarray]:
    """Merge per-shard lists [G, Q, kin] into [Q, k]."""
    vals = _c(vals, np.float32)
    ids = _c(ids, np.int64)
    G, Q, kin = vals.shape
    ov = np.empty((Q, k), np.float32)
    oi = np.empty((Q, k), np.int64)
    lib().orc_topk_merge(int(largest), _p(vals, _f32p), _p(ids, _i64p), G, Q, kin, k,
                         _p(ov, _f32p), _p(oi, _i64p))
    return ov, oi


def kmeans_assign(x: np.ndarray, c: np.ndarray, nthreads: int = 0):
    """Returns (labels int32, sqrt-distance float32, squared distance float32)."""
    x = _c(x, np.float32)
    c = _c(c, np.float32)
    N, d = x.shape
    labels = np.empty(N, np.int32)
    dist = np.empty(N, np.float32)
    sq = np.empty(N, np.float32)
    lib().orc_kmeans_assign(_p(x, _f32p), N, d, _p(c, _f32p), c.shape[0], _p(labels, _i32p),
                            _p(dist, _f32p), _p(sq, _f32p), nthreads)
    return labels, dist, sq


def kmeans_update(x: np.ndarray, labels: np.ndarray, centroids: np.ndarray):
    """Returns (new centroids, counts); empty clusters keep their centroid."""
    x = _c(x, np.float32)
    labels = _c(labels, np.int32)
    cent = np.array(centroids, dtype=np.float32, copy=True, order="C")
    K = cent.shape[0]
    counts = np.empty(K, np.int64)
    lib().orc_kmeans_update(_p(x, _f32p), x.shape[0], x.shape[1], _p(labels, _i32p), K,
                            _p(cent, _f32p), _p(counts, _i64p))
    return cent, counts


def kmeans(x: np.ndarray, init_centroids: np.ndarray, max_iters: int, tol: float = 0.0,
           nthreads: int = 0):
    """Lloyd from given initial centroids -> (centroids, labels, inertia, iterations)."""
    x = _c(x, np.float32)
    cent = np.array(init_centroids, dtype=np.float32, copy=True, order="C")
    N, d = x.shape
    labels = np.empty(N, np.int32)
    inertia = ctypes.c_double(0.0)
    it = lib().orc_kmeans(_p(x, _f32p), N, d, cent.shape[0], max_iters, tol, _p(cent, _f32p),
                          _p(labels, _i32p), ctypes.byref(inertia), nthreads)
    return cent, labels, inertia.value, it


def ivf_flat_search(metric: str, q: np.ndarray, centroids: np.ndarray, list_off: np.ndarray,
                    x_sorted: np.ndarray, row_ids: np.ndarray, nprobe: int, k: int,
                    nthreads: int = 0):
    q = _c(q, np.float32)
    centroids = _c(centroids, np.float32)
    list_off = _c(list_off, np.int64)
    x_sorted = _c(x_sorted, np.float32)
    row_ids = _c(row_ids, np.int64)
    Q, d = q.shape
    out_d = np.empty((Q, k), np.float32)
    out_i = np.empty((Q, k), np.int64)
    lib().orc_ivf_flat_search(METRIC[metric], _p(q, _f32p), Q, d, _p(centroids, _f32p),
                              centroids.shape[0], _p(list_off, _i64p), _p(x_sorted, _f32p),
                              _p(row_ids, _i64p), nprobe, k, _p(out_d, _f32p),
                              _p(out_i, _i64p), nthreads)
    return out_d, out_i


def pq_encode(x: np.ndarray, labels: np.ndarray, centroids: np.ndarray,
              codebooks: np.ndarray, nthreads: int = 0) -> np.ndarray:
    x = _c(x, np.float32)
    labels = _c(labels, np.int32)
    centroids = _c(centroids, np.float32)
    codebooks = _c(codebooks, np.float32)
    M, ksub, _ = codebooks.shape
    codes = np.empty((x.shape[0], M), np.uint8)
    lib().orc_pq_encode(_p(x, _f32p), x.shape[0], x.shape[1], _p(labels, _i32p),
                        _p(centroids, _f32p), _p(codebooks, _f32p), M, ksub, _p(codes, _u8p),
                        nthreads)
    return codes


def ivfpq_search(q: np.ndarray, centroids: np.ndarray, list_off: np.ndarray,
                 codes_sorted: np.ndarray, row_ids: np.ndarray, codebooks: np.ndarray,
                 nprobe: int, k: int, nthreads: int = 0):
    q = _c(q, np.float32)
    centroids = _c(centroids, np.float32)
    list_off = _c(list_off, np.int64)
    codes_sorted = _c(codes_sorted, np.uint8)
    row_ids = _c(row_ids, np.int64)
    codebooks = _c(codebooks, np.float32)
    Q, d = q.shape
    M, ksub, _ = codebooks.shape
    out_d = np.empty((Q, k), np.float32)
    out_i = np.empty((Q, k), np.int64)
    lib().orc_ivfpq_search(_p(q, _f32p), Q, d, _p(centroids, _f32p), centroids.shape[0],
                           _p(list_off, _i64p), _p(codes_sorted, _u8p), _p(row_ids, _i64p),
                           _p(codebooks, _f32p), M, ksub, nprobe, k, _p(out_d, _f32p),
                           _p(out_i, _i64p), nthreads)
    return out_d, out_i


def sq8_encode(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """INT8 storage as this implementation defines it (the reference names
    INT8 among its precisions, csrc/include/rapidadb/core/types.h:9-14 and
    python/rapidadb/config.py:21-26, with no semantics, so parity for INT8
    is pinned by this definition only): per row, scale = max|x| / 127 (fp32
    division; 0 for a zero row), code = rint(x / scale) (fp32 division, ties
    to even) clamped to [-127, 127], 0 where scale == 0.  Returns (codes
    int8 [n, d], scales float32 [n])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    scale = (np.abs(x).max(axis=1) / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        c = np.rint(x / scale[:, None])
    c = np.where(scale[:, None] > 0, c, 0.0)
    return np.clip(c, -127, 127).astype(np.int8), scale


def sq8_decode(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """The dequantised rows fl(scale * code) (float32 products)."""
    return (np.asarray(scales, np.float32)[:, None] * np.asarray(codes).astype(np.float32)).astype(np.float32)
