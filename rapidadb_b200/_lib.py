"""Loads the native extension; there is no fallback when it is missing."""
from __future__ import annotations

import torch  # noqa: F401  (libtorch must be loaded before the extension)

_C = None


def C():
    """The compiled ``rapidadb_b200._C`` module (raises if it was never built)."""
    global _C
    if _C is None:
        try:
            from rapidadb_b200 import _C as mod
        except ImportError as e:  # pragma: no cover - exercised only on broken installs
            raise ImportError(
                "rapidadb_b200 native extension is not built (rapidadb_b200/_C.so, "
                "rapidadb_b200/librdb_kernels.so); run `python -m rapidadb_b200.build`. "
                "There is no CPU fallback.") from e
        _C = mod
    return _C
