"""The peer exchange kernel (rdb_peer_gather) on one GPU.

Two exchange arenas of this process stand for rank 0 and rank 1.  The call
runs as rank 0: it signals its slot in both arenas, waits for rank 1's
signal in its own arena and copies rank 1's rows out of rank 1's arena (and
its own out of its own).  Rank 1's signal is written into rank 0's arena
before the call, so the wait ends at once and no kernel waits on another.
Without that signal the wait runs out after its limit: the status word
reports it and nothing is copied.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PEER_BIT = 1 << 6
FLAGS = 512


def _arena(C, dev, nbytes):
    from rapidadb_b200.sharded import _DeviceSpan

    ptr, handle = C.peer_arena_alloc(dev.index, nbytes)
    assert len(handle) == 64
    return ptr, torch.as_tensor(_DeviceSpan(ptr, nbytes), device=dev)


def _signal(buf, slot, rank, epoch):
    """Rank `rank`'s signal of `slot` at `epoch`, as it would land in this arena."""
    buf[64 * slot + 8 * rank: 64 * slot + 8 * rank + 8].view(torch.int64).fill_(epoch)


@pytest.mark.parametrize("row_bytes,stride", [(512, 512), (1200, 1216), (12, 20)])
def test_gather_copies_every_ranks_rows(device, row_bytes, stride):
    import rapidadb._C as C

    dev = torch.device("cuda", torch.cuda.current_device())
    nbytes = FLAGS + 64 * stride
    (p0, a0), (p1, a1) = _arena(C, dev, nbytes), _arena(C, dev, nbytes)
    g = np.random.default_rng(row_bytes)
    for a in (a0, a1):
        a[FLAGS:] = torch.from_numpy(g.integers(0, 256, nbytes - FLAGS, dtype=np.uint8)).to(dev)
    C.device_status(True)
    _signal(a0, 2, 1, 7)
    row0, nrows = [3, 10], [20, 25]
    dst = torch.zeros(2 * 32 * row_bytes, dtype=torch.uint8, device=dev)
    C.peer_gather(0, 2, 7, [p0, p1], nbytes, FLAGS, stride, row_bytes, row0, nrows, dst, [0, 32 * row_bytes], row_bytes)
    torch.cuda.synchronize()
    assert C.device_status(True) == 0
    got = dst.view(2, 32, row_bytes).cpu().numpy()
    for r, a in enumerate((a0, a1)):
        src = a[FLAGS:].cpu().numpy()
        want = np.stack([src[(row0[r] + i) * stride: (row0[r] + i) * stride + row_bytes] for i in range(nrows[r])])
        np.testing.assert_array_equal(got[r, : nrows[r]], want)
        assert not got[r, nrows[r]:].any()
    # rank 0 signalled slot 2 at epoch 7 in both arenas
    assert a0[128:136].view(torch.int64).item() == 7
    assert a1[128:136].view(torch.int64).item() == 7
    C.peer_arena_free(dev.index, p0)
    C.peer_arena_free(dev.index, p1)


def test_later_epoch_also_releases_the_wait(device):
    import rapidadb._C as C

    dev = torch.device("cuda", torch.cuda.current_device())
    (p0, a0), (p1, a1) = _arena(C, dev, 4096), _arena(C, dev, 4096)
    a1[FLAGS: FLAGS + 64].fill_(5)
    _signal(a0, 0, 1, 9)  # rank 1 is already an epoch ahead
    dst = torch.zeros(64, dtype=torch.uint8, device=dev)
    C.device_status(True)
    C.peer_gather(0, 0, 8, [p0, p1], 4096, FLAGS, 64, 64, [0, 0], [0, 1], dst, [0, 0], 64)
    torch.cuda.synchronize()
    assert C.device_status(True) == 0
    assert (dst == 5).all()
    C.peer_arena_free(dev.index, p0)
    C.peer_arena_free(dev.index, p1)


def test_missing_signal_times_out_and_copies_nothing(device):
    import rapidadb._C as C

    dev = torch.device("cuda", torch.cuda.current_device())
    (p0, a0), (p1, a1) = _arena(C, dev, 4096), _arena(C, dev, 4096)
    a1[FLAGS: FLAGS + 64].fill_(5)
    _signal(a0, 1, 1, 3)  # an older epoch: not enough
    dst = torch.zeros(64, dtype=torch.uint8, device=dev)
    C.device_status(True)
    C.peer_gather(0, 1, 4, [p0, p1], 4096, FLAGS, 64, 64, [0, 0], [0, 1], dst, [0, 0], 64, limit_ns=100_000)
    torch.cuda.synchronize()
    assert C.pending_status() & PEER_BIT  # mirrored to host memory: the next search raises
    assert C.device_status(True) & PEER_BIT
    assert C.pending_status() == 0
    assert C.device_status(False) == 0
    assert not dst.any()
    C.peer_arena_free(dev.index, p0)
    C.peer_arena_free(dev.index, p1)


def test_argument_errors(device):
    import rapidadb._C as C

    dev = torch.device("cuda", torch.cuda.current_device())
    p0, a0 = _arena(C, dev, 4096)
    dst = torch.zeros(64, dtype=torch.uint8, device=dev)
    with pytest.raises(RuntimeError, match="src_off"):
        C.peer_gather(0, 0, 1, [p0], 4096, 16, 64, 64, [0], [1], dst, [0], 64)
    with pytest.raises(RuntimeError, match="past the end"):
        C.peer_gather(0, 0, 1, [p0], 4096, FLAGS, 64, 64, [56], [1], dst, [0], 64)
    with pytest.raises(RuntimeError, match="do not fit"):
        C.peer_gather(0, 0, 1, [p0], 4096, FLAGS, 64, 64, [0], [2], dst, [0], 64)
    with pytest.raises(RuntimeError, match="epoch"):
        C.peer_gather(0, 0, 0, [p0], 4096, FLAGS, 64, 64, [0], [1], dst, [0], 64)
    C.peer_arena_free(dev.index, p0)
