"""``rapidadb.utils`` alias (python/rapidadb/utils.py)."""
from rapidadb_b200.utils import compute_recall, cuda_timer, generate_random_vectors  # noqa: F401
