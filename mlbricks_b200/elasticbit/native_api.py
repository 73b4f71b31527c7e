"""Discovery of the native ElasticBit runtime (libebx on a CUDA device).

Same three functions as the reference's loader
(mlbricks/elasticbit/native_api.py:10-33): ``available()``, ``importError()``
and ``requireNative()``, which raises RuntimeError mentioning the CUDA runtime
when the native module could not be imported.
"""
from __future__ import annotations

import importlib

try:
    _C = importlib.import_module(f"{__package__}._native")
except Exception as exc:  # no libebx build or no CUDA device
    _C = None
    _IMPORT_ERROR: Exception | None = exc
else:
    _IMPORT_ERROR = None


def available() -> bool:
    return _C is not None


def importError() -> Exception | None:
    return _IMPORT_ERROR


def requireNative():
    if _C is None:
        raise RuntimeError(
            "ElasticBit requires its CUDA runtime: build libebx with "
            "`python mlbricks_b200/csrc/build.py` and run on a CUDA (sm_100a) device."
        ) from _IMPORT_ERROR
    return _C


__all__ = ["available", "importError", "requireNative"]
