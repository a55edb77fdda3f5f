"""``rapidadb.config`` alias (python/rapidadb/config.py)."""
from rapidadb_b200.config import IndexConfig, IndexType, Metric, Precision  # noqa: F401
