"""Python face of the ElasticBit CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this module.  It is the checker for the CUDA product, never a fallback.

Contents
--------
* ctypes bindings of ``oracle/ebx_oracle.c`` (the C restatement of the
  reference runtime's storage, analyzer and forward arithmetic);
* MLB4 single-matrix file reader/writer restating the reference's header and
  checksum rules (elasticbit_runtime.cu:692-712, 810-871, 1024-1049);
* ``select_bits_torch``: a restatement of ``_selectBitsTorch``
  (mlbricks/elasticbit/core.py:112-195) that runs on any torch device;
* seeded generators for the BASELINE weight scheme (per-row sigma log-uniform
  in [0.005, 0.05], 0.1 % of entries x10 as outliers).
"""
from __future__ import annotations

import ctypes
import struct
from pathlib import Path

import numpy as np

from . import build as _build

_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = _build.build_oracle()
        L = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        i32, i64, u64, f32, f64 = (ctypes.c_int, ctypes.c_int64, ctypes.c_uint64,
                                   ctypes.c_float, ctypes.c_double)
        L.ebo_qmax.argtypes = [i32]; L.ebo_qmax.restype = ctypes.c_uint32
        L.ebo_packed_bytes.argtypes = [u64, i32]; L.ebo_packed_bytes.restype = u64
        L.ebo_round_fp16.argtypes = [f32]; L.ebo_round_fp16.restype = f32
        L.ebo_quantize_scalar.argtypes = [f32, f32, i32]; L.ebo_quantize_scalar.restype = i32
        L.ebo_row_scales.argtypes = [P, i32, i32, i32, P]; L.ebo_row_scales.restype = i32
        L.ebo_pack_codes.argtypes = [P, i32, i32, i32, P]; L.ebo_pack_codes.restype = i32
        L.ebo_pack_weights.argtypes = [P, i32, i32, i32, P, P]; L.ebo_pack_weights.restype = i32
        L.ebo_extract_code.argtypes = [P, u64, u64, i32]; L.ebo_extract_code.restype = ctypes.c_uint32
        L.ebo_unpack_codes.argtypes = [P, u64, i32, i32, i32, P]; L.ebo_unpack_codes.restype = i32
        L.ebo_dequantize.argtypes = [P, u64, P, i32, i32, i32, P]; L.ebo_dequantize.restype = i32
        L.ebo_dequantize_fp16.argtypes = [P, u64, P, i32, i32, i32, P]
        L.ebo_dequantize_fp16.restype = i32
        L.ebo_analyze.argtypes = [P, i32, i32, P, i32, P, P, P, P]; L.ebo_analyze.restype = i32
        L.ebo_select.argtypes = [P, f64]; L.ebo_select.restype = i32
        L.ebo_linear_full.argtypes = [P, i64, P, i32, i32, P, P]; L.ebo_linear_full.restype = None
        L.ebo_linear_hw.argtypes = [P, i64, P, P, i32, i32, P, P]; L.ebo_linear_hw.restype = None
        L.ebo_elastic_linear_packed.argtypes = [P, i64, P, P, P, i32, i64, i64, i64, P]
        L.ebo_elastic_linear_packed.restype = None
        L.ebo_fnv1a64.argtypes = [P, u64]; L.ebo_fnv1a64.restype = u64
        _LIB = L
    return _LIB


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def qmax(bits: int) -> int:
    return int(lib().ebo_qmax(bits))


def packed_bytes(count: int, bits: int) -> int:
    return int(lib().ebo_packed_bytes(count, bits))


def row_scales(w: np.ndarray, bits: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty(w.shape[0], dtype=np.float32)
    lib().ebo_row_scales(_p(w), w.shape[0], w.shape[1], bits, _p(out))
    return out


def quantize(w: np.ndarray, scales: np.ndarray, bits: int) -> np.ndarray:
    """int16 codes q = clamp(rint(w / s), +-qmax) with float32 division."""
    w = np.asarray(w, dtype=np.float32)
    s = np.asarray(scales, dtype=np.float32)[:, None]
    q = np.rint(w / s)
    m = qmax(bits)
    return np.clip(q, -m, m).astype(np.int16)


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.int16)
    rows, cols = codes.shape
    out = np.zeros(packed_bytes(rows * cols, bits), dtype=np.uint8)
    rc = lib().ebo_pack_codes(_p(codes), rows, cols, bits, _p(out))
    if rc == 1:
        raise ValueError("prequantized ElasticBit code exceeds selected bit range")
    if rc:
        raise ValueError("ElasticBit storage bits must be between 3 and 16")
    return out


def pack_weights(w: np.ndarray, bits: int, scales: np.ndarray | None = None) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if bits == 16:
        out = np.zeros(rows * cols * 2, dtype=np.uint8)
        sc = None
    else:
        out = np.zeros(packed_bytes(rows * cols, bits), dtype=np.uint8)
        sc = np.ascontiguousarray(scales if scales is not None else row_scales(w, bits),
                                  dtype=np.float32)
    rc = lib().ebo_pack_weights(_p(w), rows, cols, bits, _p(sc), _p(out))
    if rc:
        raise ValueError("ElasticBit storage bits must be between 3 and 16")
    return out


def unpack_codes(payload: np.ndarray, rows: int, cols: int, bits: int) -> np.ndarray:
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.int16)
    lib().ebo_unpack_codes(_p(payload), payload.size, rows, cols, bits, _p(out))
    return out


def dequantize(payload: np.ndarray, scales: np.ndarray | None, rows: int, cols: int,
               bits: int) -> np.ndarray:
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty((rows, cols), dtype=np.float32)
    lib().ebo_dequantize(_p(payload), payload.size, _p(sc), rows, cols, bits, _p(out))
    return out


def dequantize_fp16(payload: np.ndarray, scales: np.ndarray | None, rows: int, cols: int,
                    bits: int) -> np.ndarray:
    """fp16 dequantised weights as a float16 array (bit patterns exact)."""
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty((rows, cols), dtype=np.uint16)
    lib().ebo_dequantize_fp16(_p(payload), payload.size, _p(sc), rows, cols, bits, _p(out))
    return out.view(np.float16)


def dequantize_codes(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp16(fp32(q) * s) from int16 codes (numpy; float32 multiply, RN to fp16)."""
    prod = codes.astype(np.float32) * np.asarray(scales, dtype=np.float32)[:, None]
    return prod.astype(np.float16)


def analyze(w: np.ndarray, calib: np.ndarray, threshold: float) -> dict:
    """Host analyzer (cu:280-483): same dict layout as the reference's _C.analyze."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    c = np.ascontiguousarray(calib, dtype=np.float32)
    if w.ndim != 2 or c.ndim != 2:
        raise ValueError("weights and calibrationData must both be 2D")
    if c.shape[1] != w.shape[1]:
        raise ValueError("calibrationData width must equal weight cols")
    hw = np.zeros(14); full = np.zeros(14); err = np.zeros(14)
    storage = np.zeros(14, dtype=np.uint64)
    rc = lib().ebo_analyze(_p(w), w.shape[0], w.shape[1], _p(c), c.shape[0], _p(hw), _p(full),
                           _p(err), _p(storage))
    if rc:
        raise ValueError("weights and calibration must be non-empty")
    sel = lib().ebo_select(_p(err), float(threshold))
    if sel < 0:
        raise ValueError("threshold must be a finite non-negative value")
    original = float(w.shape[0] * w.shape[1] * 2)
    cands = []
    for i in range(14):
        cands.append({
            "bits": i + 3,
            "hardwareNativeError": float(hw[i]),
            "fullPrecisionError": float(full[i]),
            "error": float(err[i]),
            "storageBytes": int(storage[i]),
            "memoryReduction": 1.0 - float(storage[i]) / original,
            "passes": bool(err[i] <= threshold),
        })
    return {"threshold": float(threshold), "selectedBits": int(sel),
            "selectedError": float(err[sel - 3]), "candidates": cands}


def linear_full(x16: np.ndarray, w16: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """Reference fullPrecision output in float64: x16 @ w16^T (+ bias)."""
    x = np.ascontiguousarray(x16, dtype=np.float16).reshape(-1, x16.shape[-1])
    w = np.ascontiguousarray(w16, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    y = np.empty((x.shape[0], w.shape[0]), dtype=np.float64)
    lib().ebo_linear_full(_p(x.view(np.uint16)), x.shape[0], _p(w), w.shape[0], w.shape[1],
                          _p(b), _p(y))
    return y


def linear_hw(x16: np.ndarray, codes: np.ndarray, scales: np.ndarray,
              bias: np.ndarray | None = None) -> np.ndarray:
    """Reference hardwareNative (integer-dot, scale after) output in float64."""
    x = np.ascontiguousarray(x16, dtype=np.float16).reshape(-1, x16.shape[-1])
    q = np.ascontiguousarray(codes, dtype=np.int16)
    s = np.ascontiguousarray(scales, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    y = np.empty((x.shape[0], q.shape[0]), dtype=np.float64)
    lib().ebo_linear_hw(_p(x.view(np.uint16)), x.shape[0], _p(q), _p(s), q.shape[0], q.shape[1],
                        _p(b), _p(y))
    return y


def elastic_linear_packed(x: np.ndarray, packed: np.ndarray, scales: np.ndarray,
                          bias: np.ndarray | None, bits: int, group_size: int,
                          out_features: int, in_features: int) -> np.ndarray:
    xf = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, in_features)
    pk = np.ascontiguousarray(packed, dtype=np.uint8)
    sc = np.ascontiguousarray(scales, dtype=np.float32)
    b = None if bias is None or np.size(bias) == 0 else np.ascontiguousarray(bias, np.float32)
    out = np.empty((xf.shape[0], out_features), dtype=np.float32)
    lib().ebo_elastic_linear_packed(_p(xf), xf.shape[0], _p(pk), _p(sc), _p(b), bits,
                                    group_size, out_features, in_features, _p(out))
    return out


def fnv1a64(data: bytes | np.ndarray) -> int:
    arr = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    return int(lib().ebo_fnv1a64(_p(arr), arr.size))


# --------------------------------------------------------------------------
# MLB4 single-matrix files (cu:692-712 header; cu:1024-1049 writer;
# cu:810-871 reader).  Little-endian, packed, 80 bytes.
# --------------------------------------------------------------------------
MLB4_HEADER = struct.Struct("<4sHHIIB3xIQQQQQdd")
assert MLB4_HEADER.size == 80


def mlb4_bytes(rows: int, cols: int, bits: int, scales: np.ndarray | None,
               payload: np.ndarray, threshold: float, selected_error: float) -> bytes:
    sc = b"" if bits == 16 or scales is None else np.ascontiguousarray(scales, np.float32).tobytes()
    pl = np.ascontiguousarray(payload, dtype=np.uint8).tobytes()
    header = MLB4_HEADER.pack(b"MLB4", 4, 80, rows, cols, bits, len(sc) // 4, len(sc), len(pl),
                              rows * cols * 2, fnv1a64(sc), fnv1a64(pl), float(threshold),
                              float(selected_error))
    return header + sc + pl


def mlb4_parse(blob: bytes) -> dict:
    if len(blob) < 80:
        raise ValueError("invalid ElasticBit MLB4 file")
    (magic, version, hbytes, rows, cols, bits, nscale, scale_bytes, payload_bytes, orig,
     sc_sum, pl_sum, threshold, sel_err) = MLB4_HEADER.unpack_from(blob, 0)
    if magic != b"MLB4":
        raise ValueError("invalid ElasticBit MLB4 file")
    if version != 4 or hbytes != 80:
        raise ValueError("unsupported ElasticBit MLB4 version")
    if bits < 3 or bits > 16 or rows == 0 or cols == 0:
        raise ValueError("invalid ElasticBit matrix dimensions")
    count = rows * cols
    exp_payload = count * 2 if bits == 16 else packed_bytes(count, bits)
    exp_scales = 0 if bits == 16 else rows
    if (nscale != exp_scales or scale_bytes != exp_scales * 4 or payload_bytes != exp_payload
            or orig != count * 2 or len(blob) != 80 + exp_scales * 4 + exp_payload):
        raise ValueError("invalid ElasticBit MLB4 metadata")
    sc = np.frombuffer(blob, dtype=np.float32, count=exp_scales, offset=80).copy()
    pl = np.frombuffer(blob, dtype=np.uint8, count=exp_payload, offset=80 + exp_scales * 4).copy()
    if fnv1a64(sc.tobytes()) != sc_sum or fnv1a64(pl) != pl_sum:
        raise ValueError("ElasticBit MLB4 checksum mismatch")
    return {"rows": rows, "cols": cols, "bits": bits, "scales": sc, "payload": pl,
            "threshold": threshold, "selectedError": sel_err}


# --------------------------------------------------------------------------
# Model-path bit selection (core.py:112-195), device-agnostic restatement.
# --------------------------------------------------------------------------
def select_bits_torch(weight, calibration: np.ndarray, threshold: float):
    """Returns (bits, error, int16 codes | None, fp32 scales | None)."""
    import torch
    import torch.nn.functional as F

    def rel(ref, cand):
        r = ref.float(); c = cand.float()
        den = torch.linalg.vector_norm(r).clamp_min(1.0e-30)
        return float((torch.linalg.vector_norm(c - r) / den).item())

    calib = torch.from_numpy(np.ascontiguousarray(calibration, dtype=np.float32)).to(
        device=weight.device, dtype=torch.float16)
    ref = F.linear(calib, weight)
    w32 = weight.float()
    max_abs = w32.abs().amax(dim=1)
    for bits in range(3, 16):
        qm = float((1 << (bits - 1)) - 1)
        scale = torch.where(max_abs > 0.0, max_abs / qm, torch.ones_like(max_abs))
        q = torch.round(w32 / scale[:, None]).clamp(min=-qm, max=qm)
        deq = (q * scale[:, None]).to(torch.float16)
        full_err = rel(ref, F.linear(calib, deq))
        if bits <= 8:
            idot = torch.matmul(calib.float(), q.transpose(0, 1))
            hw_err = rel(ref, (idot * scale[None, :]).to(torch.float16))
        else:
            hw_err = full_err
        err = max(hw_err, full_err)
        if err <= float(threshold):
            return (bits, float(err), q.to(torch.int16).cpu().numpy(),
                    scale.float().cpu().numpy())
    return 16, 0.0, None, None


# --------------------------------------------------------------------------
# Seeded synthetic inputs with the BASELINE weight scheme.
# --------------------------------------------------------------------------
def baseline_weights(rows: int, cols: int, seed: int = 0) -> np.ndarray:
    """W[n,k] = sigma_n * N(0,1), sigma_n = exp(U(ln .005, ln .05)); 0.1 % x10."""
    rng = np.random.default_rng(seed)
    sigma = np.exp(rng.uniform(np.log(0.005), np.log(0.05), size=(rows, 1)))
    w = rng.standard_normal((rows, cols), dtype=np.float32) * sigma.astype(np.float32)
    mask = rng.random((rows, cols)) < 1.0e-3
    w[mask] *= 10.0
    return w.astype(np.float32)


def normal(shape, seed: int, scale: float = 1.0) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * scale).astype(
        np.float32)


__all__ = [name for name in dir() if not name.startswith("_")]
