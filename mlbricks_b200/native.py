"""``native`` route of the compressed-linear operators (reference:
mlbricks/native.py -> mlbricks/esa/native.py:49-60, 864-882).

Loads libebx, registers the dispatcher ops (custom_ops.py) and exposes thin
wrappers.  There is no CPU or PyTorch fallback here: when libebx or a CUDA
device is missing the wrappers raise RuntimeError, and ``available()`` says so.
"""
from __future__ import annotations

import os

import torch

from . import _ebx

try:
    _LIB = _ebx.load()
except ImportError as exc:
    _LIB = None
    _IMPORT_ERROR: Exception | None = exc
else:
    _IMPORT_ERROR = None

_CUSTOM_OPS_REGISTERED = False
_CUSTOM_OPS_ERROR: Exception | None = _IMPORT_ERROR
if _LIB is not None:
    try:
        from .custom_ops import register_native_custom_ops

        _CUSTOM_OPS_REGISTERED = bool(register_native_custom_ops())
    except Exception as exc:  # torch without torch.library.custom_op
        _CUSTOM_OPS_ERROR = exc


def available() -> bool:
    return _LIB is not None


def cuda_available() -> bool:
    return _LIB is not None and torch.cuda.is_available()


def import_error() -> Exception | None:
    return _IMPORT_ERROR


def custom_ops_registered() -> bool:
    return bool(_CUSTOM_OPS_REGISTERED)


def enabled_for(tensor: torch.Tensor) -> bool:
    """Native kernels apply to CUDA inference calls unless MLBRICKS_DISABLE_NATIVE=1."""
    if os.getenv("MLBRICKS_DISABLE_NATIVE", "0") == "1" or _LIB is None:
        return False
    return bool(tensor.is_cuda) and not torch.is_grad_enabled()


def _require() -> None:
    if _LIB is None:
        raise RuntimeError(f"MLBricks native extension is unavailable: {_IMPORT_ERROR}")


def elastic_linear_packed(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                          bias: torch.Tensor, bits: int, group_size: int, out_features: int,
                          in_features: int) -> torch.Tensor:
    """Packed ElasticBit CUDA linear without materialising the weight."""
    _require()
    if not x.is_cuda:
        raise RuntimeError("elastic_linear_packed requires CUDA")
    return torch.ops.mlbricks_native.elastic_linear_packed(
        x.contiguous(), packed.contiguous(), scales.contiguous(), bias.contiguous(), int(bits),
        int(group_size), int(out_features), int(in_features))


def elastic_linear(x: torch.Tensor, matrix, bias: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ W^T (+ bias) for a RuntimeMatrix (any row count) via the dispatcher op."""
    _require()
    native = getattr(matrix, "_native", matrix)
    return torch.ops.mlbricks_native.elastic_linear(x, int(native.handle), int(native.rows), bias)


__all__ = ["available", "cuda_available", "import_error", "custom_ops_registered", "enabled_for",
           "elastic_linear_packed", "elastic_linear"]
