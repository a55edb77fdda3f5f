"""The allocation-free IVF-Flat scan (rdb_ivf_flat_scan_noalloc), called
through the C ABI, against the workspace entry point (rdb_ivf_flat_scan).

It serves callers that may not allocate device memory during a call (hosts
that pool all device memory themselves, serving threads that must not block
in an allocator, plug-ins whose host runtime forbids guest allocations): its
scratch is a static array inside the library.  The two entry points run the
same kernels, so their outputs must be identical; two calls in a row check
that the second call does not see stale scratch from the first.  After the
set-up call rdb_noalloc_init() (which loads the array and the scan's kernels),
a call changes neither the device's free memory nor torch's allocations.
This file is named to be collected last and must pass alone or after the
other tests.
"""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rapidadb_b200",
                   "librdb_kernels.so")
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64


def _lib():
    lib = ctypes.CDLL(LIB)
    lib.rdb_ivf_scan_workspace.restype = ctypes.c_size_t
    lib.rdb_ivf_scan_workspace.argtypes = [_i64, ctypes.c_int, ctypes.c_int]
    lib.rdb_noalloc_scratch_bytes.restype = ctypes.c_size_t
    lib.rdb_noalloc_init.restype = ctypes.c_int
    lib.rdb_last_error.restype = ctypes.c_char_p
    lib.rdb_ivf_flat_scan.argtypes = [ctypes.c_int, ctypes.c_int, _vp, _i64, _i64, ctypes.c_int, _vp, ctypes.c_int,
                                      _vp, _i64, _vp, _vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp, _vp,
                                      ctypes.c_size_t, _vp]
    lib.rdb_ivf_flat_scan_noalloc.argtypes = [ctypes.c_int, ctypes.c_int, _vp, _i64, _i64, ctypes.c_int, _vp,
                                              ctypes.c_int, _vp, _i64, _vp, _vp, _vp, ctypes.c_int, _vp, ctypes.c_int,
                                              _vp, _vp, _vp]
    return lib


def _problem(seed, nq, nprobe, nlist, n, d):
    """Rows stored list by list, per-query probe lists (distinct lists)."""
    g = torch.Generator().manual_seed(seed)
    labels = torch.randint(0, nlist, (n,), generator=g)
    order = torch.argsort(labels, stable=True)
    rows = torch.randn(n, d, generator=g)[order].contiguous()
    list_off = torch.zeros(nlist + 1, dtype=torch.long)
    list_off[1:] = torch.cumsum(torch.bincount(labels, minlength=nlist), 0)
    ids = (order * 3 + 7).long()
    probe = torch.stack([torch.randperm(nlist, generator=g)[:nprobe] for _ in range(nq)]).long()
    q = torch.randn(nq, d, generator=g)
    return [t.cuda().contiguous() for t in (q, probe, rows, list_off, ids)]


def _scan(lib, noalloc, q, probe, rows, list_off, ids, k, metric=1):
    nq, d = q.shape
    nprobe, nlist = probe.shape[1], list_off.numel() - 1
    out_v = torch.empty(nprobe, nq, k, device="cuda")
    out_i = torch.empty(nprobe, nq, k, device="cuda", dtype=torch.long)
    xv = (rows * rows).sum(1).sqrt().contiguous()
    stream = _vp(torch.cuda.current_stream().cuda_stream)
    args = [metric, 0, q.data_ptr(), nq, d, d, probe.data_ptr(), nprobe, rows.data_ptr(), d, xv.data_ptr(),
            list_off.data_ptr(), None, nlist, ids.data_ptr(), k, out_v.data_ptr(), out_i.data_ptr()]
    if noalloc:
        rc = lib.rdb_ivf_flat_scan_noalloc(*args, stream)
    else:
        wsb = lib.rdb_ivf_scan_workspace(nq, nprobe, nlist)
        ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device="cuda")
        rc = lib.rdb_ivf_flat_scan(*args, ws.data_ptr(), wsb, stream)
    assert rc == 0, lib.rdb_last_error()
    torch.cuda.synchronize()
    return out_v.cpu(), out_i.cpu()


def test_noalloc_scan_matches_workspace_scan_twice(device):
    lib = _lib()
    assert lib.rdb_noalloc_init() == 0, lib.rdb_last_error()
    for call, (seed, metric) in enumerate([(1, 1), (2, 0)]):
        prob = _problem(seed, nq=300, nprobe=6, nlist=40, n=5000 + call * 777, d=48)
        ref_v, ref_i = _scan(lib, False, *prob, k=10, metric=metric)
        got_v, got_i = _scan(lib, True, *prob, k=10, metric=metric)
        # same kernels, same inputs: identical outputs (tolerance 0)
        assert torch.equal(got_i, ref_i), f"call {call}: ids differ"
        torch.testing.assert_close(got_v, ref_v, rtol=0, atol=0)


def test_noalloc_rejects_oversized_requests(device):
    lib = _lib()
    cap = lib.rdb_noalloc_scratch_bytes()
    assert cap == 8 << 20
    nq, nprobe, nlist = 1 << 20, 64, 16384
    assert lib.rdb_ivf_scan_workspace(nq, nprobe, nlist) > cap
    z = torch.zeros(1, device="cuda")
    rc = lib.rdb_ivf_flat_scan_noalloc(1, 0, z.data_ptr(), nq, 8, 8, z.data_ptr(), nprobe, z.data_ptr(), 8,
                                       z.data_ptr(), z.data_ptr(), None, nlist, None, 10, z.data_ptr(), z.data_ptr(),
                                       _vp(torch.cuda.current_stream().cuda_stream))
    assert rc == 4  # RDB_ERR_UNSUPPORTED, raised before any device work
    assert b"static array" in lib.rdb_last_error()


def test_noalloc_call_allocates_nothing_after_init(device):
    """Set up once, then the scan itself leaves the device's free memory and
    torch's allocator untouched (inputs and outputs are allocated before)."""
    lib = _lib()
    assert lib.rdb_noalloc_init() == 0, lib.rdb_last_error()
    q, probe, rows, list_off, ids = _problem(5, nq=200, nprobe=5, nlist=30, n=4000, d=32)
    nq, d = q.shape
    k, nprobe, nlist = 8, probe.shape[1], list_off.numel() - 1
    out_v = torch.empty(nprobe, nq, k, device="cuda")
    out_i = torch.empty(nprobe, nq, k, device="cuda", dtype=torch.long)
    xv = (rows * rows).sum(1).contiguous()
    stream = _vp(torch.cuda.current_stream().cuda_stream)
    args = [1, 0, q.data_ptr(), nq, d, d, probe.data_ptr(), nprobe, rows.data_ptr(), d, xv.data_ptr(),
            list_off.data_ptr(), None, nlist, ids.data_ptr(), k, out_v.data_ptr(), out_i.data_ptr(), stream]
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    for _ in range(2):
        assert lib.rdb_ivf_flat_scan_noalloc(*args) == 0, lib.rdb_last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == alloc0
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
