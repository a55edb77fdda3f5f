"""High-level Python API, the drop-in for python/rapidadb/index.py.

``RapidaDB(dim, metric).add(vectors).search(queries, k)`` with torch tensors
in and out, as in the reference (index.py:24-140).  Differences:

* IVF and IVF-PQ index types are implemented (the reference raises
  NotImplementedError, index.py:64-69); they need ``train()`` (or
  ``set_quantizer``) before ``add``.
* Inputs keep their float dtype up to the index, which stores rows in
  ``config.precision`` (FP32 by default, as the reference's fp32 cast);
  FP16 / BF16 storage searches on the tcgen05 tensor cores.
* ``save(path)`` / ``RapidaDB.load(path)`` persist an index (the reference
  has no persistence): one ``torch.save`` file holding the configuration and
  the stored arrays in stored order -- rows or PQ codes, list labels, ids,
  centroids, codebooks -- so a loaded index answers exactly like the saved
  one without retraining or re-encoding.
* ``IndexConfig(devices=[0, 1, ...])`` row-shards the index over those GPUs
  of this process (rapidadb_b200.multi_device).
"""
from __future__ import annotations

import dataclasses
from typing import Optional, Tuple

import torch

from rapidadb_b200._lib import C
from rapidadb_b200.config import IndexConfig, IndexType, Metric, Precision


def _metric_to_cpp(metric: Metric):
    """Python Metric -> extension Metric (index.py:12-21)."""
    _C = C()
    return {
        Metric.COSINE: _C.Metric.COSINE,
        Metric.L2: _C.Metric.L2,
        Metric.DOT_PRODUCT: _C.Metric.DOT_PRODUCT,
    }[metric]


def _precision_to_cpp(p: Precision):
    _C = C()
    return {
        Precision.FP32: _C.Precision.FP32,
        Precision.FP16: _C.Precision.FP16,
        Precision.BF16: _C.Precision.BF16,
        Precision.INT8: _C.Precision.INT8,
    }[p]


def _as_float_cuda(t: torch.Tensor) -> torch.Tensor:
    if not t.is_cuda:
        t = t.cuda()
    if t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        t = t.float()
    return t.contiguous()


class RapidaDB:
    """GPU vector database (index.py:24-53).

    Example::

        db = RapidaDB(dim=768, metric='cosine')
        db.add(embeddings)                      # [n, 768] tensor
        distances, indices = db.search(queries, k=10)

    Args:
        dim:     Dimensionality of vectors.
        metric:  'cosine', 'l2' or 'dot_product'.
        config:  Full IndexConfig (overrides dim / metric if given).
    """

    def __init__(self, dim: int = 768, metric: str = "cosine",
                 config: Optional[IndexConfig] = None):
        if config is not None:
            self._config = config
        else:
            self._config = IndexConfig(dim=dim, metric=Metric(metric))
        self._index = self._build_index()

    def _build_index(self):
        cfg = self._config
        if cfg.devices:
            from rapidadb_b200.multi_device import MultiDeviceIndex

            return MultiDeviceIndex(lambda dev: self._build_single(), list(cfg.devices),
                                    largest=cfg.metric != Metric.L2)
        return self._build_single()

    def _build_single(self):
        _C = C()
        cfg = self._config
        if cfg.index_type == IndexType.FLAT:
            return _C.FlatIndex(cfg.dim, _metric_to_cpp(cfg.metric), _precision_to_cpp(cfg.precision))
        if cfg.index_type == IndexType.IVF and hasattr(_C, "IVFFlatIndex"):
            return _C.IVFFlatIndex(cfg.dim, _metric_to_cpp(cfg.metric), cfg.nlist, cfg.nprobe,
                                   _precision_to_cpp(cfg.precision))
        if cfg.index_type == IndexType.IVF_PQ and hasattr(_C, "IVFPQIndex"):
            return _C.IVFPQIndex(cfg.dim, _metric_to_cpp(cfg.metric), cfg.nlist, cfg.nprobe,
                                 cfg.pq_m, cfg.pq_k)
        raise NotImplementedError(
            f"Index type '{cfg.index_type.value}' is not implemented")

    # -------------------------------------------------------------- training
    def train(self, vectors: torch.Tensor, group=None) -> None:
        """Train the IVF coarse quantizer (k-means, ``config.nlist`` lists,
        ``config.kmeans_iters`` Lloyd iterations) and, for IVF-PQ, the
        per-subspace codebooks on the residuals.  ``config.train_sample`` > 0
        trains on that many seeded rows.  No-op for Flat."""
        cfg = self._config
        if cfg.index_type == IndexType.FLAT:
            return
        from rapidadb_b200.kmeans import kmeans, train_pq
        from rapidadb_b200.utils import sample_rows

        x = self._to_device(vectors)
        if 0 < cfg.train_sample < x.shape[0]:
            idx = torch.tensor(sorted(sample_rows(x.shape[0], cfg.train_sample, cfg.seed)),
                               dtype=torch.long, device=x.device)
            x = x.index_select(0, idx)
        coarse = kmeans(x, cfg.nlist, cfg.kmeans_iters, 0.0, cfg.seed, group=group).centroids
        if cfg.index_type == IndexType.IVF:
            self._index.set_quantizer(coarse)
            return
        labels, _ = C().kmeans_assign(x.float(), coarse, True)
        residuals = x.float() - coarse.index_select(0, labels.long())
        books = train_pq(residuals, cfg.pq_m, cfg.pq_k, cfg.kmeans_iters, cfg.seed, group=group)
        self._index.set_quantizer(coarse, books)

    def set_quantizer(self, centroids: torch.Tensor, codebooks: Optional[torch.Tensor] = None) -> None:
        """Install trained IVF centroids [nlist, dim] (and IVF-PQ codebooks
        [pq_m, pq_k, dim / pq_m]) directly."""
        if codebooks is None:
            self._index.set_quantizer(self._to_device(centroids).float())
        else:
            self._index.set_quantizer(self._to_device(centroids).float(), self._to_device(codebooks).float())

    @property
    def is_trained(self) -> bool:
        return bool(getattr(self._index, "is_trained", lambda: True)())

    # ------------------------------------------------------------------- data
    def add(self, vectors: torch.Tensor, ids: Optional[torch.Tensor] = None) -> None:
        """Add [n, dim] vectors (moved to CUDA if needed) with optional int64 ids
        (index.py:71-92)."""
        vectors = self._to_device(vectors)
        if ids is not None:
            ids = ids.to(vectors.device).contiguous().long()
            self._index.add(vectors, ids)
        else:
            self._index.add(vectors)

    def search(self, queries: torch.Tensor, k: int = 10) -> Tuple[torch.Tensor, torch.Tensor]:
        """k nearest neighbours of each query -> (distances [B, k] fp32,
        indices [B, k] int64), best first (index.py:94-112)."""
        queries = self._to_device(queries)
        return self._index.search(queries, k)

    def _to_device(self, t: torch.Tensor) -> torch.Tensor:
        """Float CUDA tensor on the index's (first) device."""
        if self._config.devices:
            dev = torch.device("cuda", int(self._config.devices[0]))
            if t.device != dev:
                t = t.to(dev)
        return _as_float_cuda(t)

    def reset(self) -> None:
        """Remove all vectors (index.py:114-116)."""
        self._index.reset()

    @property
    def size(self) -> int:
        return self._index.size()

    @property
    def dim(self) -> int:
        return self._config.dim

    @property
    def metric(self) -> str:
        return self._config.metric.value

    @property
    def config(self) -> IndexConfig:
        return self._config

    @property
    def index(self):
        """The underlying extension index object."""
        return self._index

    def __len__(self) -> int:
        return self.size

    # ------------------------------------------------------------ persistence
    FORMAT = "rapidadb_b200.index"
    FORMAT_VERSION = 1

    def state_dict(self) -> dict:
        """Configuration and stored arrays (host tensors) of this index; a
        multi-device index stores each shard's arrays."""
        cfg = {f.name: (getattr(self._config, f.name).value
                        if hasattr(getattr(self._config, f.name), "value") else getattr(self._config, f.name))
               for f in dataclasses.fields(self._config)}
        st = {"format": self.FORMAT, "version": self.FORMAT_VERSION, "config": cfg, "size": self.size}
        it = self._config.index_type
        if self._config.devices:
            st["shards"] = [_index_state(s, it) for s in self._index.shards]
        else:
            st.update(_index_state(self._index, it))
        return st

    def save(self, path) -> None:
        """Write the index to `path` (one torch.save file)."""
        torch.save(self.state_dict(), path)

    @classmethod
    def from_state_dict(cls, st: dict, device=None) -> "RapidaDB":
        if st.get("format") != cls.FORMAT or st.get("version") != cls.FORMAT_VERSION:
            raise ValueError("not a rapidadb_b200 index file (format %r, version %r)"
                             % (st.get("format"), st.get("version")))
        c = dict(st["config"])
        c["metric"] = Metric(c["metric"])
        c["index_type"] = IndexType(c["index_type"])
        c["precision"] = Precision(c["precision"])
        db = cls(config=IndexConfig(**c))
        it = db._config.index_type
        if db._config.devices:
            if len(st.get("shards", [])) != len(db._index.shards):
                raise ValueError("shard count in the file does not match config.devices")
            for dev, shard, sst in zip(db._index.devices, db._index.shards, st["shards"]):
                _restore_index(shard, sst, it, dev)
        else:
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            _restore_index(db._index, st, it, dev)
        return db

    @classmethod
    def load(cls, path, device=None) -> "RapidaDB":
        """Read an index written by save() onto `device` (default: the
        current CUDA device)."""
        return cls.from_state_dict(torch.load(path, map_location="cpu", weights_only=True), device)

    def __repr__(self) -> str:
        return (f"RapidaDB(dim={self.dim}, metric='{self.metric}', "
                f"index='{self._config.index_type.value}', size={self.size})")


def _index_state(ix, it: IndexType) -> dict:
    """Stored arrays of one extension index, in stored (list) order; INT8
    (SQ8) rows as their codes and scales, so a reload is exact."""
    st = {}
    if it == IndexType.FLAT:
        if ix.size():
            if ix.sq8():
                st["sq8_codes"] = ix.sq8_codes().cpu()
                st["sq8_scales"] = ix.sq8_scales().cpu()
            else:
                st["vectors"] = ix.vectors().cpu()
            st["ids"] = ix.ids().cpu()
        return st
    if ix.is_trained():
        st["centroids"] = ix.centroids().cpu()
        if it == IndexType.IVF_PQ:
            st["codebooks"] = ix.codebooks().cpu()
    if ix.size():
        st["labels"] = ix.stored_labels().cpu()
        st["ids"] = ix.stored_ids().cpu()
        if it == IndexType.IVF and ix.sq8():
            st["sq8_codes"] = ix.stored_sq8_codes().cpu()
            st["sq8_scales"] = ix.stored_sq8_scales().cpu()
        elif it == IndexType.IVF:
            st["vectors"] = ix.stored_vectors().cpu()
        else:
            st["codes"] = ix.stored_codes().cpu()
    return st


def _restore_index(ix, st: dict, it: IndexType, dev: torch.device) -> None:
    """Load arrays written by _index_state into an empty extension index on dev."""
    with torch.cuda.device(dev):
        if it == IndexType.FLAT:
            if "sq8_codes" in st:
                ix.add_sq8(st["sq8_codes"].to(dev), st["sq8_scales"].to(dev), st["ids"].to(dev))
            elif "vectors" in st:
                ix.add(st["vectors"].to(dev), st["ids"].to(dev))
            return
        if "centroids" in st:
            if it == IndexType.IVF_PQ:
                ix.set_quantizer(st["centroids"].to(dev), st["codebooks"].to(dev))
            else:
                ix.set_quantizer(st["centroids"].to(dev))
        if "sq8_codes" in st:
            ix.restore_sq8(st["sq8_codes"].to(dev), st["sq8_scales"].to(dev), st["labels"].to(dev),
                           st["ids"].to(dev))
        elif "ids" in st:
            data = st["vectors"] if it == IndexType.IVF else st["codes"]
            ix.restore(data.to(dev), st["labels"].to(dev), st["ids"].to(dev))
