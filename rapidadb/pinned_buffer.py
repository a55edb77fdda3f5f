"""``rapidadb.pinned_buffer`` alias (python/rapidadb/pinned_buffer.py)."""
from rapidadb_b200.pipeline import PinnedBuffer  # noqa: F401
