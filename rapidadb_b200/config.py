"""Configuration dataclasses, the reference's python/rapidadb/config.py surface.

Same enums, fields and defaults (config.py:7-60); ``devices`` is added for
row-sharded multi-GPU indexes and ``kmeans_iters`` / ``train_sample`` for IVF
training.
"""
from dataclasses import dataclass
from enum import Enum
from typing import Optional


class Metric(str, Enum):
    """Distance metric for vector similarity search (config.py:7-11)."""
    COSINE = "cosine"
    L2 = "l2"
    DOT_PRODUCT = "dot_product"


class IndexType(str, Enum):
    """Index structure (config.py:14-18)."""
    FLAT = "flat"
    IVF = "ivf"
    IVF_PQ = "ivf_pq"


class Precision(str, Enum):
    """Storage precision (config.py:21-26).  FP32 rows search on CUDA cores,
    FP16 / BF16 rows on the tcgen05 tensor cores.  INT8 stores each row as
    SQ8 codes with a per-row scale (scale = max|x| / 127, code = rint(x /
    scale)) and searches the dequantised rows exactly, on CUDA cores, with
    fp32 queries (Flat and IVF-Flat)."""
    FP32 = "fp32"
    FP16 = "fp16"
    BF16 = "bf16"
    INT8 = "int8"


@dataclass
class IndexConfig:
    """Index configuration (config.py:29-60).

    Attributes:
        dim:            Dimensionality of vectors.
        metric:         Distance metric (cosine, l2, dot_product).
        index_type:     Index structure (flat, ivf, ivf_pq).
        precision:      Storage precision.
        nlist:          Number of IVF lists (IVF / IVF-PQ).
        nprobe:         Lists probed per query (IVF / IVF-PQ).
        pq_m:           PQ sub-quantisers (IVF-PQ).
        pq_k:           Codewords per sub-quantiser (IVF-PQ, 256 = 8-bit codes).
        num_streams:    Kept for API compatibility.
        max_batch_size: Kept for API compatibility.
        kmeans_iters:   Lloyd iterations used by train().
        train_sample:   Rows sampled for training (0 = all).
        seed:           Seed for training initialisation.
    """
    dim: int = 768
    metric: Metric = Metric.COSINE
    index_type: IndexType = IndexType.FLAT
    precision: Precision = Precision.FP32

    nlist: int = 4096
    nprobe: int = 64

    pq_m: int = 96
    pq_k: int = 256

    num_streams: int = 4
    max_batch_size: int = 128

    kmeans_iters: int = 20
    train_sample: int = 0
    seed: int = 42
    devices: Optional[list] = None
