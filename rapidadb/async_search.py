"""``rapidadb.async_search`` alias (python/rapidadb/async_search.py)."""
from rapidadb_b200.pipeline import AsyncBatchSearcher  # noqa: F401
