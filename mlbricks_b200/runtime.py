"""Backend-name policy shared by every route (reference: mlbricks/runtime.py:27-64).

Canonical names are ``auto``, ``native`` and ``pytorch``; the reference's
legacy aliases are accepted and mapped the same way.
"""
from __future__ import annotations

import warnings

VALID_BACKENDS = frozenset({"auto", "native", "pytorch"})

_ALIASES = {
    "cuda": "native", "cpp": "native", "cpp/cuda": "native",
    "torch": "pytorch", "python": "pytorch", "reference": "pytorch",
    "thunder": "auto", "flare": "pytorch", "pulse": "pytorch", "lightning": "pytorch",
}


def normalize_backend(value: str | None = "auto", *, warn_legacy: bool = False) -> str:
    """Return the canonical ``auto`` / ``native`` / ``pytorch`` name."""
    if value is None:
        return "auto"
    name = str(value).strip().lower().replace("-", "_")
    if name in VALID_BACKENDS:
        return name
    if name in _ALIASES:
        mapped = _ALIASES[name]
        if warn_legacy:
            warnings.warn(f"backend={value!r} is a legacy MLBricks backend name; "
                          f"use backend={mapped!r} instead.", DeprecationWarning, stacklevel=3)
        return mapped
    raise ValueError(f"backend must be one of: auto, native, pytorch; got {value!r}.")


def set_module_backend(module, backend: str, *, recursive: bool = True):
    """Apply ``set_backend`` to a module and (optionally) every child that has one."""
    value = normalize_backend(backend)
    targets = module.modules() if recursive and hasattr(module, "modules") else [module]
    for m in targets:
        setter = getattr(m, "set_backend", None)
        if callable(setter):
            setter(value)
    return module


__all__ = ["VALID_BACKENDS", "normalize_backend", "set_module_backend"]
