"""libebx loads and exports every symbol include/ebx.h declares; argument
validation that needs no GPU returns the documented status codes."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from mlbricks_b200 import _ebx

HEADER = Path(__file__).resolve().parents[1] / "include" / "ebx.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^EBX_API\s+[^;(]*?\b(ebx_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_bound_symbols():
    declared = declared_symbols()
    assert len(declared) >= 18
    assert declared == set(_ebx.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _ebx.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.ebx_version().decode().startswith("ebx ")


def test_fnv_entry_matches_oracle():
    from oracle import oracle as O

    lib = _ebx.load()
    data = np.random.default_rng(0).integers(0, 256, size=4099, dtype=np.uint8)
    assert lib.ebx_fnv1a64(data.ctypes.data, data.size) == O.fnv1a64(data)
    assert lib.ebx_fnv1a64(None, 0) == 1469598103934665603


def test_argument_errors_without_gpu():
    lib = _ebx.load()
    h = ctypes.c_void_p()
    # invalid width is rejected before any CUDA call
    st = lib.ebx_matrix_create_from_codes(1, 1, 4, 4, 17, 0, None, ctypes.byref(h))
    assert st == _ebx.EBX_ERR_INVALID
    assert "3..15" in _ebx.last_error()
    st = lib.ebx_matrix_create_from_payload(1, 11, 1, 4, 4, 5, 0, 0, None, ctypes.byref(h))
    assert st == _ebx.EBX_ERR_INVALID and "metadata" in _ebx.last_error()
    st = lib.ebx_elastic_linear_packed(1, 1, 1, 1, 1, 0, None, 9, 1, 1, 1, 1, None)
    assert st == _ebx.EBX_ERR_INVALID and "[2,8]" in _ebx.last_error()
    assert lib.ebx_linear(None, None, 1, None, None, None, None, 0, None) == _ebx.EBX_ERR_INVALID
    assert lib.ebx_matrix_set_execution_width(None, 8) == _ebx.EBX_ERR_INVALID
    assert lib.ebx_analyze_workspace_bytes(0, 4) == 0
    with pytest.raises(ValueError):
        _ebx.check(_ebx.EBX_ERR_INVALID)
    with pytest.raises(RuntimeError):
        _ebx.check(_ebx.EBX_ERR_CUDA)


def test_exchange_argument_errors_without_gpu():
    lib = _ebx.load()
    h = ctypes.c_void_p()
    blob = (ctypes.c_uint8 * _ebx.EXCHANGE_HANDLE_BYTES)()
    # shape and rank checks come before any CUDA call
    assert lib.ebx_exchange_create(9, 0, 0, 1, 16, blob, ctypes.byref(h)) == _ebx.EBX_ERR_INVALID
    assert "world" in _ebx.last_error()
    assert lib.ebx_exchange_create(2, 2, 0, 1, 16, blob, ctypes.byref(h)) == _ebx.EBX_ERR_INVALID
    assert lib.ebx_exchange_create(2, 0, 0, 257, 16, blob, ctypes.byref(h)) == _ebx.EBX_ERR_INVALID
    assert "max_m" in _ebx.last_error()
    assert lib.ebx_exchange_create(2, 0, 0, 1, 16, None, ctypes.byref(h)) == _ebx.EBX_ERR_INVALID
    assert lib.ebx_exchange_connect(None, blob) == _ebx.EBX_ERR_INVALID
    assert lib.ebx_exchange_destroy(None) == _ebx.EBX_OK
    assert lib.ebx_linear_allreduce(None, None, 1, None, None, None, None, None) == _ebx.EBX_ERR_INVALID
    assert lib.ebx_exchange_set_protocol(None, 0) == _ebx.EBX_ERR_INVALID
