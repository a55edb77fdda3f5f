"""Host query pipeline: pinned staging buffers and multi-stream batch search.

The reference ships the same two helpers (python/rapidadb/pinned_buffer.py:11-57,
python/rapidadb/async_search.py:7-43), but its kernels run on the legacy
default stream, so its "async" searches serialise.  Here every search runs on
the caller's current stream and releases the GIL while it waits for its own
stream, so worker threads -- one CUDA stream and one set of pinned buffers
each -- really overlap: one batch's host-to-device copy and result read-back
run while another batch's kernels occupy the GPU.

* ``PinnedBuffer(max_batch_size, dim, dtype)``: ``copy_to_device(data,
  stream=None)`` as in the reference.
* ``AsyncBatchSearcher(index, num_streams=4)``: ``search_batches(batches, k)``
  (device batches, as in the reference) and ``search_host(queries, k,
  batch_size)`` (host queries in, host results out, end to end).

A sharded (multi-process) index must not be searched from several threads at
once: its collectives would interleave differently on different ranks.
"""
from __future__ import annotations

import threading
from concurrent.futures import ThreadPoolExecutor
from typing import List, Optional, Sequence, Tuple, Union

import numpy as np
import torch


class PinnedBuffer:
    """Pre-allocated page-locked host buffer for batched host-to-device copies
    (pinned_buffer.py:11-57)."""

    def __init__(self, max_batch_size: int, dim: int, dtype=torch.float32):
        self.max_batch_size = max_batch_size
        self.dim = dim
        self.dtype = dtype
        self.buffer = torch.empty(max_batch_size, dim, dtype=dtype, pin_memory=True)

    def copy_to_device(self, data, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Stage `data` ([n, dim] numpy array or CPU tensor) in the pinned
        buffer and start its copy to the current device (on `stream` if
        given).  The buffer may be refilled once that stream has passed the
        copy."""
        src = torch.from_numpy(np.ascontiguousarray(data)) if isinstance(data, np.ndarray) else data
        n = src.shape[0]
        if n > self.max_batch_size:
            raise ValueError(f"Batch size {n} exceeds buffer size {self.max_batch_size}")
        self.buffer[:n].copy_(src)
        if stream is not None:
            with torch.cuda.stream(stream):
                return self.buffer[:n].to("cuda", non_blocking=True)
        return self.buffer[:n].to("cuda")


class _Lane:
    """One worker: a CUDA stream with its pinned query / result buffers."""

    def __init__(self, device: torch.device):
        self.device = device
        self.stream = torch.cuda.Stream(device=device)
        self.qbuf: Optional[torch.Tensor] = None
        self.dbuf: Optional[torch.Tensor] = None
        self.ibuf: Optional[torch.Tensor] = None
        self.lock = threading.Lock()  # a lane's buffers serve one batch at a time

    def buffers(self, n: int, dim: int, dtype, k: int):
        if self.qbuf is None or self.qbuf.shape[0] < n or self.qbuf.shape[1] != dim or self.qbuf.dtype != dtype:
            self.qbuf = torch.empty(n, dim, dtype=dtype, pin_memory=True)
        if self.dbuf is None or self.dbuf.shape[0] < n or self.dbuf.shape[1] != k:
            self.dbuf = torch.empty(n, k, dtype=torch.float32, pin_memory=True)
            self.ibuf = torch.empty(n, k, dtype=torch.int64, pin_memory=True)
        return self.qbuf, self.dbuf, self.ibuf


class AsyncBatchSearcher:
    """Multi-stream batch search (async_search.py:7-43): batch i runs on
    worker i mod num_streams, each worker a thread with its own CUDA stream.

    Args:
        index:        anything with ``search(queries, k)`` (RapidaDB, an
                      extension index, ShardedSearch on one process).
        num_streams:  worker threads / CUDA streams.
    """

    def __init__(self, index, num_streams: int = 4, device: Optional[Union[int, torch.device]] = None):
        self.index = index
        self.num_streams = max(1, int(num_streams))
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.device = dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())
        self._lanes = [_Lane(self.device) for _ in range(self.num_streams)]
        self._pool = ThreadPoolExecutor(max_workers=self.num_streams)

    def _run(self, lane: _Lane, fn):
        torch.cuda.set_device(self.device)
        with torch.cuda.stream(lane.stream):
            out = fn(lane)
        lane.stream.synchronize()
        return out

    def search_batches(self, query_batches: Sequence[torch.Tensor], k: int) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """Search device query batches; results in batch order (each on the
        device, complete when returned)."""

        def job(q):
            return lambda lane: self.index.search(q, k)

        # each lane first waits for the caller's stream, which produced the batches
        caller = torch.cuda.current_stream(self.device)
        futures = []
        for i, q in enumerate(query_batches):
            lane = self._lanes[i % self.num_streams]
            lane.stream.wait_stream(caller)
            futures.append(self._pool.submit(self._run, lane, job(q)))
        return [f.result() for f in futures]

    def search_host(self, queries, k: int, batch_size: int = 1024,
                    dtype: Optional[torch.dtype] = None) -> Tuple[np.ndarray, np.ndarray]:
        """End to end: host queries ([n, dim] numpy array or CPU tensor) in,
        host results (distances [n, k] fp32, ids [n, k] int64) out.  Each
        batch is staged in its worker's pinned buffer, copied to the GPU,
        searched and read back into pinned result buffers on that worker's
        stream, overlapping other workers' batches."""
        src = torch.from_numpy(np.ascontiguousarray(queries)) if isinstance(queries, np.ndarray) else queries
        n, dim = src.shape
        qdtype = dtype or src.dtype
        out_d = np.empty((n, k), np.float32)
        out_i = np.empty((n, k), np.int64)

        def job(lo, hi):
            def fn(lane):
                qh, dh, ih = lane.buffers(batch_size, dim, qdtype, k)
                m = hi - lo
                qh[:m].copy_(src[lo:hi])
                qd = qh[:m].to(self.device, non_blocking=True)
                d, i = self.index.search(qd, k)
                dh[:m].copy_(d, non_blocking=True)
                ih[:m].copy_(i, non_blocking=True)
                lane.stream.synchronize()
                out_d[lo:hi] = dh[:m].numpy()
                out_i[lo:hi] = ih[:m].numpy()
                return m

            return fn

        futures = []
        for b, lo in enumerate(range(0, n, batch_size)):
            lane = self._lanes[b % self.num_streams]
            futures.append(self._pool.submit(self._run_locked, lane, job(lo, min(n, lo + batch_size))))
        for f in futures:
            f.result()
        return out_d, out_i

    def _run_locked(self, lane: _Lane, fn):
        with lane.lock:
            return self._run(lane, fn)

    def close(self) -> None:
        self._pool.shutdown(wait=True)
        for lane in self._lanes:
            lane.stream.synchronize()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

