"""CPU oracle for the RapidaDB search hot path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package.  The product package ``rapidadb_b200`` never
does: it has no CPU fallback.
"""
from oracle.oracle import *  # noqa: F401,F403
