"""``rapidadb._C``: the compiled extension of rapidadb_b200 under the
reference's module name (csrc/bindings/torch_extension.cpp:16)."""
from rapidadb_b200._lib import C as _load

_mod = _load()
globals().update({k: getattr(_mod, k) for k in dir(_mod) if not k.startswith("__")})
