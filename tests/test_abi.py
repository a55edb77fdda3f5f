"""CPU-only checks of the native boundary: the C-ABI library loads and exports
every function include/rapidadb_b200.h declares, the extension imports, and
argument errors are raised without touching a GPU."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rapidadb_b200.h")
LIB = os.path.join(ROOT, "rapidadb_b200", "librdb_kernels.so")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rdb_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("rdb_flat_search", "rdb_distance", "rdb_topk", "rdb_topk_merge", "rdb_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_abi_calls_without_gpu():
    """Pure host-side entry points work on a CPU-only machine."""
    lib = ctypes.CDLL(LIB)
    lib.rdb_version.restype = ctypes.c_int
    assert lib.rdb_version() >= 100
    lib.rdb_last_error.restype = ctypes.c_char_p
    lib.rdb_flat_search_workspace.restype = ctypes.c_size_t
    lib.rdb_flat_search_workspace.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int]
    ws = lib.rdb_flat_search_workspace(0, 2, 1024, 1_000_000, 768, 100, 0)
    assert 0 < ws < (1 << 31)
    # exhaustive workspace bounds every candidate list by its split
    ws_ex = lib.rdb_flat_search_workspace(0, 2, 1024, 1_000_000, 768, 100, 1)
    assert ws_ex >= 1024 * 1_000_000 * 8


def test_argument_errors_reported():
    lib = ctypes.CDLL(LIB)
    lib.rdb_last_error.restype = ctypes.c_char_p
    # k > n is rejected before any device work
    f = lib.rdb_flat_search
    f.restype = ctypes.c_int
    rc = f(1, 2, None, ctypes.c_int64(1), ctypes.c_int64(8), None, ctypes.c_int64(5), ctypes.c_int64(8),
           None, 8, 6, None, ctypes.c_int64(0), 0, None, None, None, ctypes.c_size_t(0), None)
    assert rc == 1
    assert b"k must be in [1, 5]" in lib.rdb_last_error()


def test_extension_imports_and_rejects_cpu_tensors():
    import rapidadb._C as _C

    with pytest.raises(RuntimeError, match="CUDA"):
        _C.l2_distance(torch.randn(2, 8), torch.randn(3, 8))
    idx = _C.FlatIndex(8, _C.Metric.L2)
    with pytest.raises(RuntimeError, match="must be on CUDA"):
        idx.add(torch.randn(3, 8))
    assert repr(idx) == "FlatIndex(dim=8, size=0)"


def test_dropin_surface():
    import rapidadb
    from rapidadb import IndexConfig, Metric, RapidaDB

    db = RapidaDB(dim=32, metric="l2")
    assert db.dim == 32 and db.metric == "l2" and len(db) == 0
    assert "index='flat'" in repr(db)
    assert IndexConfig().nlist == 4096 and Metric("dot_product") == Metric.DOT_PRODUCT
    assert rapidadb.RapidaDB is RapidaDB


def test_reference_module_paths():
    """Every module of the reference's python/rapidadb package imports under
    its own name and resolves to this implementation."""
    import rapidadb
    from rapidadb.async_search import AsyncBatchSearcher
    from rapidadb.config import IndexConfig, IndexType, Metric, Precision
    from rapidadb.index import RapidaDB
    from rapidadb.pinned_buffer import PinnedBuffer
    from rapidadb.utils import compute_recall, cuda_timer, generate_random_vectors

    from rapidadb_b200.pipeline import AsyncBatchSearcher as A, PinnedBuffer as P

    assert RapidaDB is rapidadb.RapidaDB and IndexConfig is rapidadb.IndexConfig
    assert AsyncBatchSearcher is A and PinnedBuffer is P
    assert IndexType("ivf_pq") == IndexType.IVF_PQ and Precision("bf16") == Precision.BF16
    assert Metric("cosine") == Metric.COSINE
    assert callable(compute_recall) and callable(cuda_timer) and callable(generate_random_vectors)


def test_ivf_argument_errors_reported():
    """IVF entry points reject bad shapes before any device work."""
    lib = ctypes.CDLL(LIB)
    lib.rdb_last_error.restype = ctypes.c_char_p
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    # rotated code layout only for the query-major code widths
    lib.rdb_pq_scatter_codes.argtypes = [vp, i64, ctypes.c_int, vp, vp, ctypes.c_int, vp]
    assert lib.rdb_pq_scatter_codes(None, 10, 7, None, None, 1, None) == 1
    assert b"pq_m = 7" in lib.rdb_last_error()
    assert lib.rdb_pq_scatter_codes(None, 0, 7, None, None, 0, None) == 0  # nothing to place
    # IVF scans: k above 32, unknown metric
    lib.rdb_ivf_flat_scan.argtypes = [ctypes.c_int, ctypes.c_int, vp, i64, i64, ctypes.c_int, vp, ctypes.c_int,
                                      vp, i64, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int, vp, vp, vp,
                                      ctypes.c_size_t, vp]
    rc = lib.rdb_ivf_flat_scan(1, 0, None, 4, 8, 8, None, 2, None, 8, None, None, None, 16, None, 33,
                               None, None, None, 0, None)
    assert rc == 1 and b"k in [1, 32]" in lib.rdb_last_error()
    rc = lib.rdb_ivf_flat_scan(7, 0, None, 4, 8, 8, None, 2, None, 8, None, None, None, 16, None, 10,
                               None, None, None, 0, None)
    assert rc == 1 and b"unknown metric" in lib.rdb_last_error()


def test_kmeans_init_rows_match_python_sampler():
    """_C.kmeans draws its initial rows with the same Floyd / SplitMix64
    sampler as rapidadb_b200.utils.sample_rows (host code, no GPU)."""
    import rapidadb._C as _C
    from rapidadb_b200.utils import sample_rows

    for n, k, seed in ((10, 10, 1), (1000, 37, 42), (5, 0, 3), (100000, 4096, 7)):
        assert list(_C.sample_rows(n, k, seed)) == sample_rows(n, k, seed)
    with pytest.raises(RuntimeError, match="cannot sample"):
        _C.sample_rows(3, 4, 0)


class RdbPeerGather(ctypes.Structure):
    """include/rapidadb_b200.h: RdbPeerGather (RDB_PEER_MAX_RANKS = 8)."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int), ("slot", ctypes.c_int), ("pad", ctypes.c_int),
                ("epoch", ctypes.c_ulonglong), ("base", ctypes.c_void_p * 8), ("arena_bytes", ctypes.c_longlong),
                ("src_off", ctypes.c_longlong), ("src_row_stride", ctypes.c_longlong),
                ("row_bytes", ctypes.c_longlong), ("row0", ctypes.c_longlong * 8), ("nrows", ctypes.c_longlong * 8),
                ("dst", ctypes.c_void_p), ("dst_off", ctypes.c_longlong * 8), ("dst_row_stride", ctypes.c_longlong)]


def test_peer_gather_argument_errors_without_gpu():
    """Every bad argument of the peer exchange is rejected before any device
    work (no GPU here), with a message naming it."""
    lib = ctypes.CDLL(LIB)
    lib.rdb_last_error.restype = ctypes.c_char_p
    f = lib.rdb_peer_gather
    f.argtypes = [ctypes.POINTER(RdbPeerGather), ctypes.c_ulonglong, ctypes.c_void_p]

    def args(**kw):
        a = RdbPeerGather(world=2, rank=0, slot=2, epoch=1, arena_bytes=4096, src_off=512, src_row_stride=64,
                          row_bytes=64, dst=1 << 20, dst_row_stride=64)
        a.base[0], a.base[1] = 1 << 24, 1 << 25
        a.nrows[0] = a.nrows[1] = 1
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    cases = [(dict(world=9), b"world"), (dict(rank=2), b"rank"), (dict(slot=8), b"slot"), (dict(epoch=0), b"epoch"),
             (dict(row_bytes=6), b"row_bytes"), (dict(src_off=16), b"src_off"), (dict(dst=None), b"dst"),
             (dict(arena_bytes=560), b"past the end")]
    for kw, msg in cases:
        a = args(**kw)
        assert f(ctypes.byref(a), 2_000_000_000, None) == 1, kw  # RDB_ERR_INVALID
        assert msg in lib.rdb_last_error(), (kw, lib.rdb_last_error())
    a = args()
    assert f(ctypes.byref(a), 10, None) == 1 and b"limit_ns" in lib.rdb_last_error()
