"""MLB4 single-matrix file format (byte-compatible with the reference).

Layout (little-endian, packed; elasticbit_runtime.cu:692-712):

    offset size  field
    0      4     magic "MLB4"
    4      2     version = 4
    6      2     header_bytes = 80
    8      4     rows
    12     4     cols
    16     1     storage_bits (3..16)
    17     3     reserved (zero)
    20     4     scale_count (rows, or 0 for 16-bit storage)
    24     8     scale_bytes
    32     8     payload_bytes (ceil(rows*cols*bits/8), or rows*cols*2)
    40     8     original_fp16_bytes (rows*cols*2)
    48     8     scale_checksum (FNV-1a 64 of the scale bytes)
    56     8     payload_checksum (FNV-1a 64 of the payload bytes)
    64     8     threshold (f64)
    72     8     selected_error (f64)
    80     ...   scales (fp32 x scale_count), then payload

Reader checks follow cu:814-863 in the same order with the same messages.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .. import _ebx

HEADER = struct.Struct("<4sHHIIB3xIQQQQQdd")
assert HEADER.size == 80


def fnv1a64(buf: np.ndarray | bytes) -> int:
    arr = np.frombuffer(buf, dtype=np.uint8) if isinstance(buf, (bytes, bytearray)) else \
        np.ascontiguousarray(buf).reshape(-1).view(np.uint8)
    lib = _ebx.load()
    return int(lib.ebx_fnv1a64(arr.ctypes.data if arr.size else None, arr.size))


def payload_bytes_for(rows: int, cols: int, bits: int) -> int:
    count = rows * cols
    return count * 2 if bits == 16 else (count * bits + 7) // 8


@dataclass
class MLB4:
    rows: int
    cols: int
    bits: int
    scales: np.ndarray  # float32 [rows], empty for 16-bit storage
    payload: np.ndarray  # uint8
    threshold: float
    selected_error: float


def write(path: str | Path, m: MLB4) -> None:
    scales = np.ascontiguousarray(m.scales, dtype=np.float32) if m.bits != 16 else \
        np.zeros(0, dtype=np.float32)
    payload = np.ascontiguousarray(m.payload, dtype=np.uint8)
    header = HEADER.pack(
        b"MLB4", 4, HEADER.size, m.rows, m.cols, m.bits, scales.size, scales.nbytes,
        payload.nbytes, m.rows * m.cols * 2, fnv1a64(scales), fnv1a64(payload),
        float(m.threshold), float(m.selected_error))
    try:
        with open(path, "wb") as f:
            f.write(header)
            f.write(scales.tobytes())
            f.write(payload.tobytes())
    except OSError as exc:
        raise RuntimeError(f"failed to open ElasticBit output: {path}") from exc


def read(path: str | Path) -> MLB4:
    try:
        blob = Path(path).read_bytes()
    except OSError as exc:
        raise RuntimeError(f"failed to open ElasticBit file: {path}") from exc
    if len(blob) < HEADER.size or blob[:4] != b"MLB4":
        raise RuntimeError("invalid ElasticBit MLB4 file")
    (_, version, hbytes, rows, cols, bits, nscale, scale_bytes, payload_bytes, original,
     scale_sum, payload_sum, threshold, selected_error) = HEADER.unpack_from(blob, 0)
    if version != 4 or hbytes != HEADER.size:
        raise RuntimeError("unsupported ElasticBit MLB4 version")
    if bits < 3 or bits > 16:
        raise ValueError("ElasticBit storage bits must be between 3 and 16")
    if rows == 0 or cols == 0:
        raise RuntimeError("invalid ElasticBit matrix dimensions")
    count = rows * cols
    exp_payload = payload_bytes_for(rows, cols, bits)
    exp_scales = 0 if bits == 16 else rows
    if (nscale != exp_scales or scale_bytes != exp_scales * 4 or payload_bytes != exp_payload
            or original != count * 2 or len(blob) != HEADER.size + exp_scales * 4 + exp_payload):
        raise RuntimeError("invalid ElasticBit MLB4 metadata")
    scales = np.frombuffer(blob, dtype=np.float32, count=exp_scales, offset=HEADER.size).copy()
    payload = np.frombuffer(blob, dtype=np.uint8, count=exp_payload,
                            offset=HEADER.size + exp_scales * 4).copy()
    if fnv1a64(scales) != scale_sum or fnv1a64(payload) != payload_sum:
        raise RuntimeError("ElasticBit MLB4 checksum mismatch")
    return MLB4(rows, cols, bits, scales, payload, threshold, selected_error)


__all__ = ["HEADER", "MLB4", "fnv1a64", "payload_bytes_for", "read", "write"]
