"""rapidadb_b200 - RapidaDB's search path, rebuilt for B200 (sm_100a).

Drop-in for the reference's ``rapidadb`` package (``from rapidadb import
RapidaDB, IndexConfig, Metric``); the ``rapidadb`` alias package re-exports
this one.  Native code: ``librdb_kernels.so`` (CUDA kernels behind the C ABI
in include/rapidadb_b200.h) and ``_C.so`` (C++ host layer + bindings).
"""
from rapidadb_b200.config import IndexConfig, IndexType, Metric, Precision
from rapidadb_b200.index import RapidaDB

__version__ = "0.2.0"
__all__ = ["RapidaDB", "IndexConfig", "IndexType", "Metric", "Precision"]
