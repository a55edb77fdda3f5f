"""``rapidadb.index`` alias (python/rapidadb/index.py): ``from rapidadb.index
import RapidaDB`` resolves to the B200 facade."""
from rapidadb_b200.index import RapidaDB  # noqa: F401
