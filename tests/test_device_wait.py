"""Bounded device waits: a wait that runs out is reported, not hung.

Every mbarrier wait of the tensor-core scan gives up after a time limit,
records the role in the device status word and lets the CTA exit.  Here a
probe kernel waits, through the same wait routine, on an mbarrier that no
thread ever arrives at (no TMA load or MMA in flight), with a 100 us limit:

* the C-ABI call returns RDB_ERR_TIMEOUT (3) and sets status bit 5;
* searches are asynchronous, so a timeout reaches the host through a
  mapped host word that the next search forwards; the search after that
  raises, until the status is read and cleared;
* after clearing, searches run and return correct results again.
"""
import ctypes
import os
import time

import numpy as np
import pytest
import torch

import oracle
from parity import assert_topk_match

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rapidadb_b200",
                   "librdb_kernels.so")
PROBE_BIT = 1 << 5


def test_probe_times_out_through_the_c_abi(device):
    import rapidadb._C as _C

    lib = ctypes.CDLL(LIB)
    lib.rdb_probe_bounded_wait.argtypes = [ctypes.c_ulonglong, ctypes.c_void_p]
    lib.rdb_last_error.restype = ctypes.c_char_p
    _C.device_status(True)
    t0 = time.perf_counter()
    rc = lib.rdb_probe_bounded_wait(100_000, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    elapsed = time.perf_counter() - t0
    assert rc == 3, lib.rdb_last_error()  # RDB_ERR_TIMEOUT
    assert b"ran out" in lib.rdb_last_error()
    assert elapsed < 5.0
    assert _C.device_status(True) & PROBE_BIT
    assert _C.device_status(False) == 0
    # out-of-range limits are argument errors, checked before any launch
    assert lib.rdb_probe_bounded_wait(10, None) == 1


def test_timeout_reaches_later_searches_until_cleared(device):
    import rapidadb._C as _C

    g = np.random.default_rng(3)
    x = torch.from_numpy(g.standard_normal((20000, 64), dtype=np.float32)).cuda().to(torch.bfloat16)
    q = torch.from_numpy(g.standard_normal((50, 64), dtype=np.float32)).cuda().to(torch.bfloat16)
    idx = _C.FlatIndex(64, _C.Metric.L2, _C.Precision.BF16)
    idx.add(x)
    _C.device_status(True)
    code, msg = _C.probe_bounded_wait(100_000)
    assert code == 3 and "ran out" in msg
    idx.search(q, 10)  # enqueued before the host knows; its last kernel forwards the status
    torch.cuda.synchronize()
    assert _C.pending_status() & PROBE_BIT
    with pytest.raises(RuntimeError, match="bounded device wait"):
        idx.search(q, 10)
    assert _C.device_status(True) & PROBE_BIT
    assert _C.pending_status() == 0
    dist, ids = idx.search(q, 10)
    rd, ri = oracle.flat_search("l2", q.float().cpu().numpy(), x.float().cpu().numpy(), 10)
    assert_topk_match(rd, ri, dist.cpu().numpy(), ids.cpu().numpy(), rtol=1e-4, atol=1e-5)
    torch.cuda.synchronize()
    assert _C.device_status(True) == 0
