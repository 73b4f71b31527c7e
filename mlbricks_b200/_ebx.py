"""ctypes binding of libebx (include/ebx.h), the B200 ElasticBit CUDA runtime.

This is the only module that touches the shared library.  It is loaded from
``mlbricks_b200/_lib/libebx.so`` (built in tree by ``mlbricks_b200/csrc/build.py``);
when the file is missing, ``load()`` raises ImportError -- there is no
fallback implementation.

Status codes map to Python exceptions the way the reference's pybind module
maps C++ exceptions (elasticbit_runtime.cu:26-35, 58-62): EBX_ERR_INVALID and
EBX_ERR_CODE_RANGE become ValueError, everything else RuntimeError.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import os

# EBX_LIBRARY points at an alternative build of the same ABI (e.g. a variant
# compiled with different kernel options); default: the in-tree build.
LIB_PATH = Path(os.environ.get("EBX_LIBRARY") or
                Path(__file__).resolve().parent / "_lib" / "libebx.so")

EBX_OK = 0
EBX_ERR_INVALID = 1
EBX_ERR_CUDA = 2
EBX_ERR_UNSUPPORTED = 3
EBX_ERR_WORKSPACE = 4
EBX_ERR_CODE_RANGE = 5

EXCHANGE_HANDLE_BYTES = 128  # EBX_EXCHANGE_HANDLE_BYTES

# Every symbol include/ebx.h declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64
_ST = ctypes.c_int


class MatrixInfo(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int32),
        ("cols", ctypes.c_int32),
        ("storage_bits", ctypes.c_int32),
        ("execution_width", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("payload_bytes", ctypes.c_uint64),
        ("device_bytes", ctypes.c_uint64),
    ]


SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ebx_version": (ctypes.c_char_p, []),
    "ebx_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "ebx_matrix_create_from_codes": (_ST, [_P, _P, _I32, _I32, _I32, _I32, _P, ctypes.POINTER(_P)]),
    "ebx_matrix_create_from_payload": (
        _ST, [_P, _U64, _P, _I32, _I32, _I32, _I32, _I32, _P, ctypes.POINTER(_P)]),
    "ebx_matrix_create_from_fp16": (_ST, [_P, _I32, _I32, _I32, _P, ctypes.POINTER(_P)]),
    "ebx_matrix_destroy": (_ST, [_P]),
    "ebx_matrix_query": (_ST, [_P, ctypes.POINTER(MatrixInfo)]),
    "ebx_matrix_set_execution_width": (_ST, [_P, _I32]),
    "ebx_matrix_export_payload": (_ST, [_P, _P, _U64, _P]),
    "ebx_matrix_export_scales": (_ST, [_P, _P, _P]),
    "ebx_matrix_materialize": (_ST, [_P, _P, _P]),
    "ebx_linear_workspace_bytes": (_U64, [_P, _I64]),
    "ebx_linear": (_ST, [_P, _P, _I64, _P, _P, _P, _P, _U64, _P]),
    "ebx_analyze_workspace_bytes": (_U64, [_I32, _I32]),
    "ebx_analyze": (_ST, [_P, _I32, _I32, _P, _I32, _P, _P, _P, _U64, _P]),
    "ebx_analyze_noalloc": (_ST, [_P, _I32, _I32, _P, _I32, _P, _P, _P]),
    "ebx_quantize": (_ST, [_P, _I32, _I32, _I32, _P, _P, _P]),
    "ebx_weights_to_fp16": (_ST, [_P, _I64, _P, _P]),
    "ebx_device_status": (_ST, [_I32, ctypes.POINTER(_I32), _I32]),
    "ebx_fnv1a64": (_U64, [_P, _U64]),
    "ebx_linear_swiglu": (_ST, [_P, _P, _I64, _P, _P, _P, _P]),
    "ebx_linear_multi": (_ST, [_P, _I32, _P, _I64, _P, _P, _P, _P]),
    "ebx_exchange_create": (_ST, [_I32, _I32, _I32, _I64, _I64, _P, ctypes.POINTER(_P)]),
    "ebx_exchange_connect": (_ST, [_P, _P]),
    "ebx_exchange_destroy": (_ST, [_P]),
    "ebx_linear_allreduce": (_ST, [_P, _P, _I64, _P, _P, _P, _P, _P]),
    "ebx_exchange_allreduce": (_ST, [_P, _P, _I64, _I64, _P, _P, _P, _P]),
    "ebx_exchange_set_protocol": (_ST, [_P, _I32]),
    "ebx_elastic_linear_packed": (
        _ST, [_P, _I32, _I64, _P, _P, _I32, _P, _I32, _I64, _I64, _I64, _P, _P]),
}

_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load libebx once and attach the C signatures; ImportError if absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"libebx is not built ({LIB_PATH}); run mlbricks_b200/csrc/build.py")
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        raise ImportError(f"cannot load {LIB_PATH}: {exc}") from exc
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.ebx_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(status: int) -> None:
    if status == EBX_OK:
        return
    msg = last_error() or f"libebx status {status}"
    if status in (EBX_ERR_INVALID, EBX_ERR_CODE_RANGE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def stream_ptr(stream=None, device: int | None = None) -> int:
    """cudaStream_t of the given torch stream, or of the current stream of
    `device` (default: the current device), as an integer."""
    import torch

    if stream is not None:
        return int(stream.cuda_stream)
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:  # no Stream object per call: this sits on every launch
        return int(raw(torch.cuda.current_device() if device is None else device))
    return int(torch.cuda.current_stream(device).cuda_stream)


__all__ = ["LIB_PATH", "MatrixInfo", "SIGNATURES", "load", "last_error", "check", "stream_ptr"]
