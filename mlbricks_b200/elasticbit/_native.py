"""Native ElasticBit module for B200: the counterpart of the reference's pybind
extension ``mlbricks.elasticbit._C`` (elasticbit_runtime.cu:1411-1469).

Same module surface -- ``analyze``, ``backendInfo`` and class ``RuntimeMatrix``
with the same method and property names, argument meanings, defaults and error
types -- implemented over libebx's C ABI (include/ebx.h) with device buffers
from torch's allocator.  Importing this module fails (ImportError) when libebx
is not built or no CUDA device is visible; callers see that through
``native_api.available()``, exactly as a missing reference extension.
"""
from __future__ import annotations

import ctypes
import math
import threading
from pathlib import Path
from typing import Any

import numpy as np
import torch

from .. import _ebx
from . import mlb4

_LIB = _ebx.load()
if not torch.cuda.is_available():
    raise ImportError("ElasticBit B200 runtime needs a visible CUDA device")

_MIN_BITS, _MAX_BITS, _FP16_BITS = 3, 15, 16
_POLICIES = ("hardwareNative", "fullPrecision")
_DECODE_ENGINE = "FastWarp"  # public name of the M <= 16 decode route (cu:1404)


def _parse_policy(value: str) -> str:
    value = str(value)
    if value not in _POLICIES:
        raise ValueError("decodePolicy must be 'hardwareNative' or 'fullPrecision'")
    return value


def _check_threshold(value: float, name: str = "threshold") -> float:
    value = float(value)
    if not math.isfinite(value) or value < 0.0:
        if name == "threshold":
            raise ValueError("threshold must be a finite non-negative value")
        raise ValueError(f"{name} must be a finite non-negative value")
    return value


def _as_f32_2d(value: Any, what: str) -> np.ndarray:
    arr = np.ascontiguousarray(np.asarray(value, dtype=np.float32))
    if arr.ndim != 2:
        raise ValueError(what)
    return arr


def _stream() -> int:
    return _ebx.stream_ptr()


# ---------------------------------------------------------------------------
# Matrix-path analyzer (cu:438-483)
# ---------------------------------------------------------------------------
def _analyze_raw(w: np.ndarray, c: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    rows, cols = w.shape
    samples = c.shape[0]
    if rows <= 0 or cols <= 0 or samples <= 0:
        raise ValueError("weights and calibration must be non-empty")
    dev = torch.device("cuda", torch.cuda.current_device())
    wd = torch.from_numpy(w).to(dev)
    cd = torch.from_numpy(c).to(dev)
    ws_bytes = int(_LIB.ebx_analyze_workspace_bytes(rows, samples))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    hw = torch.empty(14, dtype=torch.float64, device=dev)
    full = torch.empty(14, dtype=torch.float64, device=dev)
    _ebx.check(_LIB.ebx_analyze(wd.data_ptr(), rows, cols, cd.data_ptr(), samples, hw.data_ptr(),
                                full.data_ptr(), ws.data_ptr(), ws_bytes, _stream()))
    return hw.cpu().numpy(), full.cpu().numpy()


def _candidates(rows: int, cols: int, hw: np.ndarray, full: np.ndarray, threshold: float):
    original = float(rows * cols * 2)
    out = []
    for i in range(14):
        bits = i + 3
        count = rows * cols
        storage = count * 2 if bits == 16 else (count * bits + 7) // 8 + rows * 4
        err = max(float(hw[i]), float(full[i]))
        out.append({
            "bits": bits,
            "hardwareNativeError": float(hw[i]),
            "fullPrecisionError": float(full[i]),
            "error": err,
            "storageBytes": int(storage),
            "memoryReduction": 1.0 - storage / original,
            "passes": bool(err <= threshold),
        })
    return out


def _select(cands: list[dict], threshold: float) -> dict:
    for item in cands:
        if item["bits"] <= _MAX_BITS and item["error"] <= threshold:
            return item
    return cands[-1]


def analyze(weights: Any, calibrationData: Any, threshold: float) -> dict:
    w = np.ascontiguousarray(np.asarray(weights, dtype=np.float32))
    c = np.ascontiguousarray(np.asarray(calibrationData, dtype=np.float32))
    if w.ndim != 2 or c.ndim != 2:
        raise ValueError("weights and calibrationData must both be 2D")
    if c.shape[1] != w.shape[1]:
        raise ValueError("calibrationData width must equal weight cols")
    hw, full = _analyze_raw(w, c)
    threshold = float(threshold)
    cands = _candidates(w.shape[0], w.shape[1], hw, full, threshold)
    _check_threshold(threshold)
    sel = _select(cands, threshold)
    return {"threshold": threshold, "selectedBits": sel["bits"], "selectedError": sel["error"],
            "candidates": cands}


def backendInfo() -> dict:
    dev = torch.cuda.current_device()
    props = torch.cuda.get_device_properties(dev)
    return {
        "device": props.name,
        "deviceIndex": dev,
        "architecture": f"sm{props.major}{props.minor}",
        "weightWidths": (4, 8, 16),
        "activateDType": "float16",
        "prefill": "native",
        "decodePlanner": "cudaAutoTune",
        "decodeEngine": _DECODE_ENGINE,
        "decodeStatus": "experimental",
        "decodeValidation": "unvalidated",
        "validated": False,
    }


# ---------------------------------------------------------------------------
# Execution-width planner (cu:1174-1178, 1241-1334)
# ---------------------------------------------------------------------------
_TUNE_LOCK = threading.Lock()
_TUNE_CACHE: dict[str, int] = {}


def _legal_widths(bits: int) -> tuple[int, ...]:
    """Execution widths that represent `bits`-bit codes (cu:1174-1178 on the
    reference).  4 and 8 are the reference's W4A16 / W8A16 integer-code
    semantics; 12 is the same integer-code semantics for b <= 12, which the
    B200 tensor cores execute exactly (every |q| <= 2047 is an fp16 operand);
    16 is W16A16 over fp16(q * s)."""
    if bits <= 4:
        return (4, 8, 16)
    if bits <= 8:
        return (8, 16)
    if bits <= 12:
        return (12, 16)
    return (16,)


class RuntimeMatrix:
    """One compressed matrix resident on one GPU (rows = N out, cols = K in)."""

    def __init__(self, handle: int, threshold: float, selected_error: float, policy: str,
                 device: int) -> None:
        self._h = ctypes.c_void_p(handle)
        info = _ebx.MatrixInfo()
        _ebx.check(_LIB.ebx_matrix_query(self._h, ctypes.byref(info)))
        self._rows = int(info.rows)
        self._cols = int(info.cols)
        self._bits = int(info.storage_bits)
        self._device_bytes = int(info.device_bytes)
        self._payload_bytes = int(info.payload_bytes)
        self._device = int(device)
        self._threshold = float(threshold)
        self._error = float(selected_error)
        self._policy = _parse_policy(policy)
        self._width = 16
        self._planner = "fullPrecision"
        self._host_io: tuple[torch.Tensor, torch.Tensor] | None = None
        self._configure()

    def __del__(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _LIB.ebx_matrix_destroy(h)
            except Exception:  # interpreter shutdown
                pass
            self._h = ctypes.c_void_p(0)

    # -- factories -----------------------------------------------------------
    @staticmethod
    def _device() -> int:
        return torch.cuda.current_device()

    @staticmethod
    def compress(weights: Any, calibrationData: Any, threshold: float,
                 decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        w = np.ascontiguousarray(np.asarray(weights, dtype=np.float32))
        c = np.ascontiguousarray(np.asarray(calibrationData, dtype=np.float32))
        if w.ndim != 2 or c.ndim != 2:
            raise ValueError("weights and calibrationData must both be 2D")
        if c.shape[1] != w.shape[1]:
            raise ValueError("calibrationData width must equal weight cols")
        hw, full = _analyze_raw(w, c)
        threshold = _check_threshold(threshold)
        sel = _select(_candidates(w.shape[0], w.shape[1], hw, full, threshold), threshold)
        return RuntimeMatrix._build_from_weights(w, sel["bits"], threshold, sel["error"],
                                                 _parse_policy(decodePolicy))

    @staticmethod
    def _compressSelected(weights: Any, selectedBits: int, threshold: float,
                          selectedError: float,
                          decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        w = np.ascontiguousarray(np.asarray(weights, dtype=np.float32))
        if w.ndim != 2:
            raise ValueError("weights must be 2D")
        bits = int(selectedBits)
        if bits < _MIN_BITS or bits > _FP16_BITS:
            raise ValueError("ElasticBit storage bits must be between 3 and 16")
        threshold = _check_threshold(threshold)
        err = _check_threshold(selectedError, "selectedError")
        if bits <= _MAX_BITS and err > threshold:
            raise ValueError("selected compressed width does not satisfy threshold")
        if bits == _FP16_BITS:
            err = 0.0
        return RuntimeMatrix._build_from_weights(w, bits, threshold, err,
                                                 _parse_policy(decodePolicy))

    @staticmethod
    def _build_from_weights(w: np.ndarray, bits: int, threshold: float, err: float,
                            policy: str) -> "RuntimeMatrix":
        rows, cols = w.shape
        if rows <= 0 or cols <= 0:
            raise ValueError("invalid ElasticBit matrix dimensions")
        dev = RuntimeMatrix._device()
        wd = torch.from_numpy(w).to(torch.device("cuda", dev))
        s = _stream()
        h = ctypes.c_void_p()
        if bits == _FP16_BITS:
            w16 = torch.empty((rows, cols), dtype=torch.float16, device=wd.device)
            _ebx.check(_LIB.ebx_weights_to_fp16(wd.data_ptr(), rows * cols, w16.data_ptr(), s))
            _ebx.check(_LIB.ebx_matrix_create_from_fp16(w16.data_ptr(), rows, cols, dev, s,
                                                        ctypes.byref(h)))
        else:
            codes = torch.empty((rows, cols), dtype=torch.int16, device=wd.device)
            scales = torch.empty(rows, dtype=torch.float32, device=wd.device)
            _ebx.check(_LIB.ebx_quantize(wd.data_ptr(), rows, cols, bits, codes.data_ptr(),
                                         scales.data_ptr(), s))
            _ebx.check(_LIB.ebx_matrix_create_from_codes(codes.data_ptr(), scales.data_ptr(), rows,
                                                         cols, bits, dev, s, ctypes.byref(h)))
        return RuntimeMatrix(h.value, threshold, err, policy, dev)

    @staticmethod
    def _compressSelectedCodes(codes: Any, scales: Any, selectedBits: int, threshold: float,
                               selectedError: float,
                               decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        on_device = torch.is_tensor(codes) and codes.is_cuda
        if torch.is_tensor(codes):
            q = codes.detach()
            if q.dtype != torch.int16:
                q = q.to(torch.int16)
        else:
            q = torch.from_numpy(np.ascontiguousarray(np.asarray(codes, dtype=np.int16)))
        if torch.is_tensor(scales):
            sc = scales.detach().to(torch.float32)
        else:
            sc = torch.from_numpy(np.ascontiguousarray(np.asarray(scales, dtype=np.float32)))
        if q.dim() != 2:
            raise ValueError("codes must be 2D")
        if sc.dim() != 1 or sc.shape[0] != q.shape[0]:
            raise ValueError("scales must contain one value per weight row")
        bits = int(selectedBits)
        if bits < _MIN_BITS or bits > _FP16_BITS:
            raise ValueError("ElasticBit storage bits must be between 3 and 16")
        if bits == _FP16_BITS:
            raise ValueError("prequantized codes require 3..15-bit storage")
        threshold = _check_threshold(threshold)
        err = float(selectedError)
        if not math.isfinite(err) or err < 0.0 or err > threshold:
            raise ValueError("selected compressed width does not satisfy threshold")
        rows, cols = int(q.shape[0]), int(q.shape[1])
        if rows <= 0 or cols <= 0:
            raise ValueError("invalid ElasticBit matrix dimensions")
        sc_host = sc.cpu().numpy() if (torch.is_tensor(sc) and sc.is_cuda) else sc.numpy()
        if not np.all(np.isfinite(sc_host)) or np.any(sc_host <= 0.0):
            raise ValueError("ElasticBit scales must be finite and positive")
        dev = q.device.index if on_device else RuntimeMatrix._device()
        cuda = torch.device("cuda", dev)
        qd = q.to(cuda).contiguous()
        sd = sc.to(cuda).contiguous()
        h = ctypes.c_void_p()
        with torch.cuda.device(dev):
            _ebx.check(_LIB.ebx_matrix_create_from_codes(qd.data_ptr(), sd.data_ptr(), rows, cols,
                                                         bits, dev, _stream(), ctypes.byref(h)))
        return RuntimeMatrix(h.value, threshold, err, _parse_policy(decodePolicy), dev)

    @staticmethod
    def load(path: str, decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        policy = _parse_policy(decodePolicy)
        m = mlb4.read(path)
        dev = RuntimeMatrix._device()
        h = ctypes.c_void_p()
        sc = np.ascontiguousarray(m.scales, dtype=np.float32)
        _ebx.check(_LIB.ebx_matrix_create_from_payload(
            m.payload.ctypes.data, m.payload.nbytes, sc.ctypes.data if sc.size else None,
            m.rows, m.cols, m.bits, 0, dev, _stream(), ctypes.byref(h)))
        return RuntimeMatrix(h.value, m.threshold, m.selected_error, policy, dev)

    # -- execution planning ----------------------------------------------------
    def _configure(self) -> None:
        if self._policy == "fullPrecision":
            self._set_width(16)
            self._planner = "fullPrecision"
            return
        self._set_width(self._autotune())
        self._planner = "cudaAutoTune"

    def _set_width(self, width: int) -> None:
        _ebx.check(_LIB.ebx_matrix_set_execution_width(self._h, int(width)))
        self._width = int(width)

    def _autotune(self) -> int:
        legal = _legal_widths(self._bits)
        if len(legal) == 1:
            return legal[0]
        props = torch.cuda.get_device_properties(self._device)
        bucket = 4 if self._bits <= 4 else 8 if self._bits <= 8 else 12 if self._bits <= 12 else 16
        key = f"{self._device}:{props.major}.{props.minor}:{self._rows}x{self._cols}:{bucket}"
        with _TUNE_LOCK:
            if key in _TUNE_CACHE:
                return _TUNE_CACHE[key]
        # Integer-code semantics (W4/W8) share one kernel here; W16 uses fp16(q*s).
        candidates = tuple(w for w in legal if w != 4 or self._bits <= 4)
        x = torch.tensor([((c % 29) - 14) / 14.0 for c in range(self._cols)],
                         dtype=torch.float16, device=self._cuda)
        y = torch.empty(self._rows, dtype=torch.float16, device=self._cuda)
        timings: dict[int, float] = {}
        for width in candidates:
            self._set_width(width)
            for _ in range(6):
                self._launch(x, 1, None, y, None)
            torch.cuda.synchronize(self._device)
            start = torch.cuda.Event(enable_timing=True)
            stop = torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(24):
                self._launch(x, 1, None, y, None)
            stop.record()
            stop.synchronize()
            timings[width] = start.elapsed_time(stop) / 24
        # The narrowest (integer-code) width is kept unless a wider one is more than 5 %
        # faster: these one-row timings repeat one matrix that the L2 holds, so widths
        # within a few percent of each other are a tie, and the integer-code widths leave
        # the most ALU headroom at HBM speed and larger decode batches (and skip the
        # per-weight fp16 rounding).
        fastest = min(timings.values())
        best = next(w for w in candidates if timings[w] <= 1.05 * fastest)
        with _TUNE_LOCK:
            _TUNE_CACHE[key] = best
        return best

    @property
    def _cuda(self) -> torch.device:
        return torch.device("cuda", self._device)

    # -- execution -----------------------------------------------------------
    def _launch(self, x: torch.Tensor, M: int, bias: torch.Tensor | None, y: torch.Tensor,
                y32: torch.Tensor | None) -> None:
        # libebx selects the matrix's device itself; the stream is that device's current one.
        # Decode batches (M <= 16) never need a workspace: skip the query on that hot path.
        ws_bytes = 0 if M <= 16 else int(_LIB.ebx_linear_workspace_bytes(self._h, M))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self._cuda) if ws_bytes else None
        _ebx.check(_LIB.ebx_linear(
            self._h, x.data_ptr(), M, None if bias is None else bias.data_ptr(), y.data_ptr(),
            None if y32 is None else y32.data_ptr(), None if ws is None else ws.data_ptr(),
            ws_bytes, _ebx.stream_ptr(device=self._device)))

    def linear(self, x: torch.Tensor, bias: torch.Tensor | None = None,
               out32: bool = False) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
        """y = x @ W^T (+ bias) for any number of rows; x fp16 CUDA [..., cols]."""
        if x.dtype != torch.float16 or not x.is_cuda:
            raise ValueError("linear requires FP16 CUDA activations")
        if x.shape[-1] != self._cols:
            raise ValueError(f"expected last dimension {self._cols}, got {x.shape[-1]}")
        if x.get_device() != self._device:
            raise ValueError("input CUDA device does not match RuntimeMatrix device")
        xc = x if x.is_contiguous() else x.contiguous()
        M = xc.numel() // self._cols
        y = torch.empty((*x.shape[:-1], self._rows), dtype=torch.float16, device=x.device)
        y32 = torch.empty(y.shape, dtype=torch.float32, device=x.device) if out32 else None
        b = None
        if bias is not None:
            b = bias.detach()
            if b.dtype != torch.float16 or b.device != x.device or not b.is_contiguous():
                b = b.to(device=x.device, dtype=torch.float16).contiguous()
            if b.numel() != self._rows:
                raise ValueError("bias must match output features")
        self._launch(xc, M, b, y, y32)
        return (y, y32) if out32 else y

    @staticmethod
    def linear_multi(mats: "list[RuntimeMatrix]", x: torch.Tensor,
                     biases: "list[torch.Tensor | None] | None" = None) -> list[torch.Tensor]:
        """y_i = x @ W_i^T (+ b_i) for matrices that share x, in one decode launch
        (ebx_linear_multi) when x has at most 16 rows and every width is 8..12;
        otherwise one ebx_linear launch per matrix."""
        if not mats:
            return []
        first = mats[0]
        if x.dtype != torch.float16 or not x.is_cuda or x.shape[-1] != first._cols:
            raise ValueError("linear_multi requires FP16 CUDA activations of the matrices' width")
        biases = list(biases) if biases is not None else [None] * len(mats)
        xc = x if x.is_contiguous() else x.contiguous()
        M = xc.numel() // first._cols
        if 0 < M <= 16 and len(mats) <= 8 and all(m._cols == first._cols and
                                                  m._device == first._device for m in mats):
            ys = [torch.empty((*x.shape[:-1], m._rows), dtype=torch.float16, device=x.device)
                  for m in mats]
            bs = []
            for m, b in zip(mats, biases):
                if b is not None:
                    b = b.detach().to(device=x.device, dtype=torch.float16).contiguous()
                    if b.numel() != m._rows:
                        raise ValueError("bias must match output features")
                bs.append(b)
            n = len(mats)
            hs = (ctypes.c_void_p * n)(*[m._h.value for m in mats])
            yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
            bp = (ctypes.c_void_p * n)(*[None if b is None else b.data_ptr() for b in bs])
            st = _LIB.ebx_linear_multi(hs, n, xc.data_ptr(), M, bp, yp, None,
                                       _ebx.stream_ptr(device=first._device))
            if st == _ebx.EBX_OK:
                return ys
            if st != _ebx.EBX_ERR_UNSUPPORTED:
                _ebx.check(st)
        return [m.linear(xc, b) for m, b in zip(mats, biases)]

    def linear_swiglu(self, x: torch.Tensor, bias: torch.Tensor | None = None,
                      out32: bool = False):
        """fp16(silu(g) * u) for a matrix whose gate/up rows are interleaved in blocks of 8
        (ebx_linear_swiglu); x fp16 CUDA [..., cols] with at most 16 rows."""
        if x.dtype != torch.float16 or not x.is_cuda:
            raise ValueError("linear_swiglu requires FP16 CUDA activations")
        if x.shape[-1] != self._cols:
            raise ValueError(f"expected last dimension {self._cols}, got {x.shape[-1]}")
        if x.get_device() != self._device:
            raise ValueError("input CUDA device does not match RuntimeMatrix device")
        xc = x if x.is_contiguous() else x.contiguous()
        M = xc.numel() // self._cols
        y = torch.empty((*x.shape[:-1], self._rows // 2), dtype=torch.float16, device=x.device)
        y32 = torch.empty(y.shape, dtype=torch.float32, device=x.device) if out32 else None
        b = None
        if bias is not None:
            b = bias.detach().to(device=x.device, dtype=torch.float16).contiguous()
            if b.numel() != self._rows:
                raise ValueError("bias must match the interleaved rows")
        _ebx.check(_LIB.ebx_linear_swiglu(
            self._h, xc.data_ptr(), M, None if b is None else b.data_ptr(), y.data_ptr(),
            None if y32 is None else y32.data_ptr(), _ebx.stream_ptr(device=self._device)))
        return (y, y32) if out32 else y

    def linear_allreduce(self, x: torch.Tensor, exchange, bias: torch.Tensor | None = None,
                         out32: bool = False):
        """Row-parallel shard + all-reduce in one libebx call (ebx_linear_allreduce):
        y = fp16(sum over ranks of x_r @ W_r^T + bias); x is this rank's K slice."""
        if not x.is_cuda or x.dtype != torch.float16:
            raise ValueError("linear_allreduce requires FP16 CUDA activations")
        if x.shape[-1] != self._cols:
            raise ValueError(f"expected last dimension {self._cols}, got {x.shape[-1]}")
        if x.get_device() != self._device:
            raise ValueError("input CUDA device does not match RuntimeMatrix device")
        xc = x if x.is_contiguous() else x.contiguous()
        M = xc.numel() // self._cols
        y = torch.empty((*x.shape[:-1], self._rows), dtype=torch.float16, device=x.device)
        y32 = torch.empty(y.shape, dtype=torch.float32, device=x.device) if out32 else None
        b = None
        if bias is not None:
            b = bias.detach().to(device=x.device, dtype=torch.float16).contiguous()
            if b.numel() != self._rows:
                raise ValueError("bias must match output features")
        _ebx.check(_LIB.ebx_linear_allreduce(
            self._h, xc.data_ptr(), M, None if b is None else b.data_ptr(), y.data_ptr(),
            None if y32 is None else y32.data_ptr(), exchange.handle,
            _ebx.stream_ptr(device=self._device)))
        return (y, y32) if out32 else y

    def forwardTorch(self, input: torch.Tensor) -> torch.Tensor:
        if not input.is_cuda:
            raise ValueError("forwardTorch requires a CUDA tensor")
        if input.dtype != torch.float16:
            raise ValueError("forwardTorch requires FP16 activations")
        if input.dim() < 1 or input.shape[-1] != self._cols or input.numel() != self._cols:
            raise ValueError("forwardTorch supports exactly one M=1 activation row")
        if input.get_device() != self._device:
            raise ValueError("input CUDA device does not match RuntimeMatrix device")
        return self.linear(input)

    def forward(self, input: Any) -> np.ndarray:
        x = np.asarray(input, dtype=np.float32)
        if x.ndim != 1 or x.shape[0] != self._cols:
            raise ValueError("input must have shape [cols]")
        xt = torch.from_numpy(np.ascontiguousarray(x)).to(self._cuda).to(torch.float16)
        y = self.linear(xt)
        return y.float().cpu().numpy()

    def benchmark(self, input: Any, iterations: int = 500) -> float:
        iterations = int(iterations)
        if iterations <= 0:
            raise ValueError("iterations must be positive")
        x = np.asarray(input, dtype=np.float32)
        if x.ndim != 1 or x.shape[0] != self._cols:
            raise ValueError("input must have shape [cols]")
        xt = torch.from_numpy(np.ascontiguousarray(x)).to(self._cuda).to(torch.float16)
        y = torch.empty(self._rows, dtype=torch.float16, device=self._cuda)
        with torch.cuda.device(self._device):
            for _ in range(20):
                self._launch(xt, 1, None, y, None)
            torch.cuda.synchronize(self._device)
            start = torch.cuda.Event(enable_timing=True)
            stop = torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(iterations):
                self._launch(xt, 1, None, y, None)
            stop.record()
            stop.synchronize()
        return float(start.elapsed_time(stop)) / iterations

    def _materializeTorch(self) -> torch.Tensor:
        out = torch.empty((self._rows, self._cols), dtype=torch.float16, device=self._cuda)
        with torch.cuda.device(self._device):
            _ebx.check(_LIB.ebx_matrix_materialize(self._h, out.data_ptr(), _stream()))
        return out

    def dequantize(self) -> np.ndarray:
        return self._materializeTorch().float().cpu().numpy()

    def _export_payload(self) -> np.ndarray:
        buf = torch.empty(self._payload_bytes, dtype=torch.uint8, device=self._cuda)
        with torch.cuda.device(self._device):
            _ebx.check(_LIB.ebx_matrix_export_payload(self._h, buf.data_ptr(), buf.numel(),
                                                      _stream()))
        return buf.cpu().numpy()

    def _export_scales(self) -> np.ndarray:
        if self._bits == _FP16_BITS:
            return np.zeros(0, dtype=np.float32)
        buf = torch.empty(self._rows, dtype=torch.float32, device=self._cuda)
        with torch.cuda.device(self._device):
            _ebx.check(_LIB.ebx_matrix_export_scales(self._h, buf.data_ptr(), _stream()))
        return buf.cpu().numpy()

    def save(self, path: str) -> None:
        mlb4.write(path, mlb4.MLB4(self._rows, self._cols, self._bits, self._export_scales(),
                                   self._export_payload(), self._threshold, self._error))

    def _pin_width(self, width: int, planner: str = "pinned") -> None:
        """Execute at `width` (legal for the storage width) without timing the
        candidates: tensor-parallel shards pin one width so that every rank runs
        the same arithmetic whatever its own timing would pick."""
        if int(width) not in _legal_widths(self._bits):
            raise ValueError(f"execution width {width} cannot represent {self._bits}-bit codes")
        self._policy = "fullPrecision" if int(width) == 16 else "hardwareNative"
        self._set_width(int(width))
        self._planner = planner

    def setDecodePolicy(self, value: str) -> None:
        policy = _parse_policy(value)
        if policy == self._policy:
            return
        self._policy = policy
        self._configure()

    # -- properties (cu:1051-1066) -------------------------------------------
    @property
    def handle(self) -> int:
        return int(self._h.value or 0)

    @property
    def device(self) -> int:
        return self._device

    rows = property(lambda self: self._rows)
    cols = property(lambda self: self._cols)
    shape = property(lambda self: (self._rows, self._cols))
    storageBits = property(lambda self: self._bits)
    executionWidth = property(lambda self: self._width)
    executionPlanner = property(lambda self: self._planner)
    decodePolicy = property(lambda self: self._policy)
    activateDType = property(lambda self: "float16")
    storageBytes = property(lambda self: self._payload_bytes +
                            (0 if self._bits == _FP16_BITS else 4 * self._rows))
    executionBytes = property(lambda self: self._device_bytes)
    originalBytes = property(lambda self: self._rows * self._cols * 2)
    memoryReduction = property(lambda self: 1.0 - self.storageBytes / float(self.originalBytes))
    threshold = property(lambda self: self._threshold)
    error = property(lambda self: self._error)


__all__ = ["analyze", "backendInfo", "RuntimeMatrix"]
