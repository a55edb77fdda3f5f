"""Drop-in alias: ``from rapidadb import RapidaDB, IndexConfig, Metric`` and
``import rapidadb._C`` resolve to rapidadb_b200 (the reference's
python/rapidadb/__init__.py:3-7 surface)."""
from rapidadb_b200 import IndexConfig, IndexType, Metric, Precision, RapidaDB  # noqa: F401
from rapidadb_b200 import __version__  # noqa: F401

__all__ = ["RapidaDB", "IndexConfig", "Metric"]
