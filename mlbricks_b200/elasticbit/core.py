"""ElasticBit public API on the B200 runtime.

Drop-in for ``mlbricks.elasticbit.core`` (reference file
mlbricks/elasticbit/core.py): the same names, signatures, defaults, error types
and artifact formats, so code written against ``mlb.ElasticBit`` runs
unchanged.  What differs is underneath:

* compressed weights live on the GPU only as their exact-width codes in the
  tile layout of libebx (no FP16/INT8 execution copy, no host payload copy);
* ``_ElasticLinear`` sends every row count (decode M <= 16 and prefill) to
  libebx's sm_100a kernels on the ``native`` route; the ``pytorch`` route is
  the reference's own M > 1 route, F.linear on the exactly dequantised weight;
  ``auto`` asks the library planner (mlbricks_b200/planner.py), which checks
  parity once against ``pytorch`` and keeps the faster route;
* packing and the matrix-path analyzer run on the device.

Bit selection on the model path (`_selectBitsTorch`) keeps the reference's
arithmetic operation for operation (core.py:112-195), so the chosen widths,
codes and scales are the reference's on the same GPU.
"""
from __future__ import annotations

import gc
import io
import json
import os
import tempfile
import zipfile
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Iterable, Mapping, Sequence

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from ..runtime import normalize_backend
from .native_api import available as _nativeAvailable
from .native_api import importError as _nativeImportError
from .native_api import requireNative as _requireNative

_POLICIES = ("hardwareNative", "fullPrecision")
_ARTIFACT_FORMAT = "ElasticBitModel"
_ARTIFACT_VERSION = 1
_CALIBRATION_ROWS = 32  # rows kept per Linear during calibration (core.py:734)


def _checkPolicy(value: str) -> str:
    """The decode policy name, validated (ValueError with the reference's message)."""
    if value not in _POLICIES:
        raise ValueError("decodePolicy must be 'hardwareNative' or 'fullPrecision'")
    return str(value)


def _as_f32_matrix(value: Any, name: str) -> np.ndarray:
    """A host float32 C-contiguous 2-D array from a tensor, array or nested list."""
    if torch.is_tensor(value):
        arr = value.detach().to(device="cpu", dtype=torch.float32).numpy()
    else:
        arr = np.asarray(value, dtype=np.float32)
    if arr.ndim != 2:
        raise ValueError(f"{name} must be a 2D matrix")
    return np.require(arr, dtype=np.float32, requirements="C")


class _CalibrationFeed:
    """ElasticBit.compress's calibrationData as a list of model calls.

    One tensor or mapping is one call; any other iterable is a sequence of calls
    (tuple entries are positional arguments, mappings keyword arguments).
    """

    def __init__(self, data: Any) -> None:
        if torch.is_tensor(data) or isinstance(data, Mapping):
            self.batches = [data]
            return
        if isinstance(data, (str, bytes)):
            raise TypeError("calibrationData must contain model inputs, not text")
        try:
            self.batches = list(data)
        except TypeError as exc:
            raise TypeError(
                "calibrationData must be a model input or an iterable of model inputs") from exc
        if not self.batches:
            raise ValueError("calibrationData cannot be empty")

    @classmethod
    def _on(cls, obj: Any, device: torch.device) -> Any:
        if torch.is_tensor(obj):
            return obj.to(device)
        if isinstance(obj, Mapping):
            return {key: cls._on(val, device) for key, val in obj.items()}
        if isinstance(obj, list):
            return [cls._on(val, device) for val in obj]
        if isinstance(obj, tuple):
            return tuple(cls._on(val, device) for val in obj)
        return obj

    def replay(self, model: nn.Module, device: torch.device) -> None:
        with torch.inference_mode():
            for batch in self.batches:
                args = self._on(batch, device)
                if isinstance(args, Mapping):
                    model(**args)
                elif isinstance(args, tuple):
                    model(*args)
                else:
                    model(args)


def _relativeL2Torch(reference: torch.Tensor, candidate: torch.Tensor) -> float:
    """||candidate - reference|| / max(||reference||, 1e-30) in fp32 (the reference
    analyzer's error measure, same operations so the same bits)."""
    r, c = reference.float(), candidate.float()
    return float((torch.linalg.vector_norm(c - r)
                  / torch.linalg.vector_norm(r).clamp_min(1.0e-30)).item())


@torch.inference_mode()
def _selectBitsTorch(weight: torch.Tensor, calibration: np.ndarray, threshold: float):
    """Smallest width 3..15 whose hardwareNative and fullPrecision calibration
    errors are both within `threshold`; else 16 (FP16 kept as is).

    Operation-for-operation restatement of core.py:112-195 on the model's GPU:
    reference = F.linear on FP16 calibration rows and the FP16 weight; per width
    scale = max|w_row| / qmax (1 for a zero row), q = round(w / s) clamped to
    +-qmax, fullPrecision output = F.linear with fp16(q * s), hardwareNative
    output (b <= 8) = fp16((x @ q^T) * s).  Returns (bits, error, codes, scales)
    with int16 codes and fp32 scales left on the device.
    """
    if weight.device.type != "cuda":
        raise RuntimeError("ElasticBit GPU analyzer requires CUDA weights")
    if weight.dtype != torch.float16:
        raise RuntimeError("ElasticBit GPU analyzer requires FP16 weights")
    if not np.isfinite(threshold) or float(threshold) < 0.0:
        raise ValueError("threshold must be a finite non-negative value")
    calib16 = torch.from_numpy(np.ascontiguousarray(calibration, dtype=np.float32)).to(
        device=weight.device, dtype=torch.float16)
    reference = F.linear(calib16, weight).detach()
    w32 = weight.detach().float()
    row_max = w32.abs().amax(dim=1)
    limit = float(threshold)
    for bits in range(3, 16):
        qmax = float((1 << (bits - 1)) - 1)
        scale = torch.where(row_max > 0.0, row_max / qmax, torch.ones_like(row_max))
        q = torch.round(w32 / scale[:, None]).clamp(min=-qmax, max=qmax)
        full_err = _relativeL2Torch(reference, F.linear(calib16, (q * scale[:, None]).to(torch.float16)))
        if bits <= 8:
            hw_out = (torch.matmul(calib16.float(), q.transpose(0, 1)) * scale[None, :]).to(
                torch.float16)
            hw_err = _relativeL2Torch(reference, hw_out)
        else:
            hw_err = full_err
        err = max(hw_err, full_err)
        if err <= limit:
            return bits, float(err), q.to(torch.int16), scale.float()
    return 16, 0.0, None, None


def _moduleDevice(module: nn.Module) -> torch.device:
    """Device of the module's first parameter (else first buffer, else CPU)."""
    first = next(module.parameters(), None)
    if first is None:
        first = next(module.buffers(), None)
    return first.device if first is not None else torch.device("cpu")


def _swap_module(root: nn.Module, name: str, replacement: nn.Module) -> None:
    """Put `replacement` at dotted path `name` inside `root`."""
    parent_name, _, leaf = name.rpartition(".")
    if not leaf:
        raise ValueError("ElasticBit cannot replace the root module")
    parent = root.get_submodule(parent_name) if parent_name else root
    parent._modules[leaf] = replacement


@dataclass(frozen=True)
class BitCandidate:
    bits: int
    hardwareNativeError: float
    fullPrecisionError: float
    error: float
    storageBytes: int
    memoryReduction: float
    passes: bool


@dataclass(frozen=True)
class BitAnalysis:
    threshold: float
    selectedBits: int
    selectedError: float
    candidates: tuple[BitCandidate, ...]


@dataclass(frozen=True)
class BackendInfo:
    available: bool
    device: str | None
    deviceIndex: int | None
    architecture: str | None
    weightWidths: tuple[int, ...]
    activateDType: str | None
    prefill: str | None
    decodePlanner: str | None
    validated: bool
    error: str | None = None
    decodeEngine: str | None = None
    decodeStatus: str | None = None
    decodeValidation: str | None = None

    def __str__(self) -> str:
        if not self.available:
            return f"ElasticBitBackend(unavailable, error={self.error!r})"
        return ("ElasticBitBackend("
                f"device={self.device!r}, architecture={self.architecture!r}, "
                f"weightWidths={self.weightWidths}, activateDType={self.activateDType!r}, "
                f"prefill={self.prefill!r}, decodePlanner={self.decodePlanner!r}, "
                f"decodeEngine={self.decodeEngine!r}, decodeStatus={self.decodeStatus!r}, "
                f"decodeValidation={self.decodeValidation!r}, validated={self.validated})")


class RuntimeMatrix:
    """Advanced single-matrix ElasticBit runtime.

    Built only through :meth:`compress` / :meth:`load` (and the internal
    analyzer hooks); there is no constructor taking a user-chosen width.
    """

    def __init__(self, native: Any) -> None:
        self._native = native

    @classmethod
    def compress(cls, weights: Any, calibrationData: Any, threshold: float,
                 decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        native = _requireNative()
        policy = _checkPolicy(decodePolicy)
        w = _as_f32_matrix(weights, "weights")
        c = _as_f32_matrix(calibrationData, "calibrationData")
        return cls(native.RuntimeMatrix.compress(w, c, float(threshold), policy))

    @classmethod
    def _compressSelected(cls, weights: Any, selectedBits: int, threshold: float,
                          selectedError: float,
                          decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        native = _requireNative()
        policy = _checkPolicy(decodePolicy)
        w = _as_f32_matrix(weights, "weights")
        return cls(native.RuntimeMatrix._compressSelected(
            w, int(selectedBits), float(threshold), float(selectedError), policy))

    @classmethod
    def _compressSelectedCodes(cls, codes: Any, scales: Any, selectedBits: int,
                               threshold: float, selectedError: float,
                               decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        """Pack an analyzer result without re-quantising (codes may stay on the GPU)."""
        native = _requireNative()
        policy = _checkPolicy(decodePolicy)
        if not torch.is_tensor(codes):
            codes = np.ascontiguousarray(codes, dtype=np.int16)
        if not torch.is_tensor(scales):
            scales = np.ascontiguousarray(scales, dtype=np.float32)
        if codes.ndim != 2:
            raise ValueError("codes must be a 2D matrix")
        if scales.ndim != 1 or scales.shape[0] != codes.shape[0]:
            raise ValueError("scales must contain one value per weight row")
        return cls(native.RuntimeMatrix._compressSelectedCodes(
            codes, scales, int(selectedBits), float(threshold), float(selectedError), policy))

    @classmethod
    def load(cls, path: str | Path, decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        native = _requireNative()
        policy = _checkPolicy(decodePolicy)
        return cls(native.RuntimeMatrix.load(str(path), policy))

    def forward(self, x: Any) -> Any:
        if torch.is_tensor(x):
            if x.is_cuda and x.dtype == torch.float16 and x.numel() == self.cols:
                return self._native.forwardTorch(x.contiguous())
            flat = np.asarray(x.detach().float().cpu().numpy(), dtype=np.float32).reshape(-1)
            out = self._native.forward(np.ascontiguousarray(flat))
            return torch.from_numpy(np.asarray(out)).to(device=x.device, dtype=x.dtype)
        flat = np.asarray(x, dtype=np.float32).reshape(-1)
        return np.asarray(self._native.forward(np.ascontiguousarray(flat)))

    def linear(self, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        """B200 extension: y = x @ W^T (+ bias) for any number of FP16 rows."""
        return self._native.linear(x, bias)

    def benchmark(self, x: Any, iterations: int = 500) -> float:
        if torch.is_tensor(x):
            x = x.detach().float().cpu().numpy()
        flat = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1))
        return float(self._native.benchmark(flat, int(iterations)))

    def dequantize(self) -> np.ndarray:
        return np.asarray(self._native.dequantize(), dtype=np.float32)

    def _materializeTorch(self) -> torch.Tensor:
        return self._native._materializeTorch()

    def save(self, path: str | Path) -> None:
        self._native.save(str(path))

    def setDecodePolicy(self, decodePolicy: str) -> "RuntimeMatrix":
        self._native.setDecodePolicy(_checkPolicy(decodePolicy))
        return self

    rows = property(lambda self: int(self._native.rows))
    cols = property(lambda self: int(self._native.cols))
    shape = property(lambda self: tuple(int(v) for v in self._native.shape))
    storageBits = property(lambda self: int(self._native.storageBits))
    executionWidth = property(lambda self: int(self._native.executionWidth))
    executionPlanner = property(lambda self: str(self._native.executionPlanner))
    decodePolicy = property(lambda self: str(self._native.decodePolicy))
    activateDType = property(lambda self: str(self._native.activateDType))
    storageBytes = property(lambda self: int(self._native.storageBytes))
    executionBytes = property(lambda self: int(self._native.executionBytes))
    originalBytes = property(lambda self: int(self._native.originalBytes))
    memoryReduction = property(lambda self: float(self._native.memoryReduction))
    threshold = property(lambda self: float(self._native.threshold))
    error = property(lambda self: float(self._native.error))


def _row_regime(rows: int) -> str:
    """Row-count regime an `auto` decision is frozen for: the native kernels
    differ by regime (decode GEMV, decode-GEMM, prefill GEMM), so a race won on
    a 4096-token prefill says nothing about a one-token decode step."""
    if rows <= 16:
        return "decode"
    return "small-batch" if rows <= 256 else "prefill"


class _FusedGroup:
    """Compressed Linears that read the same input tensor (Q, K and V; gate and up).

    At decode sizes (at most 16 rows) the first member called with an input runs
    every member in ONE launch (ebx_linear_multi: each matrix keeps its own
    width, scales and semantics) and keeps the other members' outputs until they
    are asked for with that same input object (same tensor, storage and version
    -- inference tensors have no version counter, so an in-place change of one
    between two members' calls is not seen -- on the same stream).  Any other
    call runs on its own.  Used only while every member is on
    the native route for decode sizes, so the arithmetic is the one each member
    would run alone.  This replaces the reference's fused execution, which
    concatenates the groups' dequantised FP16 weights (stage2f.py:382-420).
    """

    def __init__(self, layers: Sequence["_ElasticLinear"]) -> None:
        self.layers = list(layers)
        self._key: tuple | None = None
        self._x: torch.Tensor | None = None
        self._outputs: dict[int, torch.Tensor] = {}

    def _native_decode(self, layer: "_ElasticLinear") -> bool:
        if layer.backend == "native":
            return True
        if layer.backend != "auto":
            return False
        routes = getattr(layer, "_mlbricks_frozen_auto_routes", None) or {}
        return routes.get(("elastic_linear", False, "decode")) == "native"

    def serves(self, x: torch.Tensor) -> bool:
        rows = x.numel() // max(1, x.shape[-1])
        return 0 < rows <= 16 and all(self._native_decode(layer) for layer in self.layers)

    @staticmethod
    def _version(x: torch.Tensor) -> int:
        try:
            return x._version
        except RuntimeError:  # inference tensors carry no version counter
            return -1

    def output(self, layer: "_ElasticLinear", x: torch.Tensor) -> torch.Tensor:
        key = (self._version(x), x.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream)
        if self._x is not x or self._key != key or id(layer) not in self._outputs:
            natives = [getattr(m.matrix, "_native", m.matrix) for m in self.layers]
            biases = [m._bias_for(x) for m in self.layers]
            x2 = x.reshape(-1, x.shape[-1])
            ys = type(natives[0]).linear_multi(natives, x2, biases)
            self._outputs = {id(m): y.view(*x.shape[:-1], m.outFeatures)
                             for m, y in zip(self.layers, ys)}
            self._x, self._key = x, key
        y = self._outputs.pop(id(layer))
        if not self._outputs:  # every member served: drop the input reference
            self._x = self._key = None
        return y


class _ElasticLinear(nn.Module):
    """Internal replacement for nn.Linear.  Not part of the public import surface.

    Routes (``backend``):
      native  -- libebx kernels for FP16 CUDA activations at every row count;
      pytorch -- F.linear on the exactly dequantised FP16 weight, the
                 reference's M > 1 route (core.py:465-471);
      auto    -- planner decision per module, parity-checked once against
                 pytorch (planner.py qualify_operator_once).
    Non-FP16 activations always take the pytorch route (the reference casts the
    weight to the activation dtype there, core.py:466-467).
    """

    def __init__(self, matrix: RuntimeMatrix, inFeatures: int, outFeatures: int,
                 bias: torch.Tensor | None, backend: str = "auto") -> None:
        super().__init__()
        self.matrix = matrix
        self.inFeatures = int(inFeatures)
        self.outFeatures = int(outFeatures)
        self.backend = normalize_backend(backend)
        self._fused: _FusedGroup | None = None  # siblings reading the same input (compress)
        if bias is None:
            self.register_parameter("bias", None)
        else:
            self.bias = nn.Parameter(bias.detach().clone(), requires_grad=False)

    def set_backend(self, backend: str) -> "_ElasticLinear":
        self.backend = normalize_backend(backend)
        for attr in ("_mlbricks_frozen_auto_routes", "_mlbricks_frozen_auto_details"):
            if hasattr(self, attr):
                delattr(self, attr)
        return self

    def _bias_for(self, x: torch.Tensor) -> torch.Tensor | None:
        b = self.bias
        if b is not None and (b.device != x.device or b.dtype != x.dtype):
            b = b.to(device=x.device, dtype=x.dtype)
        return b

    def _forward_pytorch(self, x: torch.Tensor) -> torch.Tensor:
        weight = self.matrix._materializeTorch()
        if weight.dtype != x.dtype:
            weight = weight.to(dtype=x.dtype)
        return F.linear(x, weight, self._bias_for(x))

    def _forward_native(self, x: torch.Tensor) -> torch.Tensor:
        return self.matrix.linear(x, self._bias_for(x))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.inFeatures:
            raise ValueError(
                f"ElasticBit Linear expected last dimension {self.inFeatures}, got {x.shape[-1]}")
        eligible = x.is_cuda and x.dtype == torch.float16
        if not eligible or self.backend == "pytorch":
            return self._forward_pytorch(x)
        group = self._fused
        if group is not None and group.serves(x):
            return group.output(self, x)
        if self.backend == "native":
            return self._forward_native(x)
        from ..planner import EXECUTION_PLANNER

        rows = int(x.numel() // self.inFeatures)
        route = EXECUTION_PLANNER.qualify_operator_once(
            self, "elastic_linear", x,
            {"native": lambda: self._forward_native(x), "pytorch": lambda: self._forward_pytorch(x)},
            requested_backend="auto", native_available=True, training=False,
            extra=(self.inFeatures, self.outFeatures, rows), freeze_on=(_row_regime(rows),),
        )
        return self._forward_native(x) if route == "native" else self._forward_pytorch(x)


class _ModelElasticBit:
    """Controller attached as ``model.elasticbit`` by ElasticBit.compress / load.

    Holds the artifact-level facts (threshold, policy, which Linears were
    compressed or left alone) and applies policy / backend changes to every
    compressed layer; matrices shared by several layers are switched once.
    """

    def __init__(self, model: nn.Module, threshold: float, decodePolicy: str,
                 compressedNames: Sequence[str], skippedNames: Sequence[str],
                 optimizationProfiles: Mapping[str, Any] | None = None) -> None:
        self._model = model
        self.threshold = float(threshold)
        self.decodePolicy = _checkPolicy(decodePolicy)
        self.compressedNames = tuple(compressedNames)
        self.skippedNames = tuple(skippedNames)
        self.optimizationProfiles = dict(optimizationProfiles or {})
        self.activeOptimization: dict[str, Any] | None = None

    def _compressed_layers(self) -> Iterable[tuple[str, "_ElasticLinear"]]:
        for name in self.compressedNames:
            try:
                layer = self._model.get_submodule(name)
            except AttributeError:
                continue
            if isinstance(layer, _ElasticLinear):
                yield name, layer

    def _matrices(self) -> Iterable[RuntimeMatrix]:
        seen: set[int] = set()
        for _, layer in self._compressed_layers():
            if id(layer.matrix) not in seen:
                seen.add(id(layer.matrix))
                yield layer.matrix

    def setDecodePolicy(self, decodePolicy: str) -> "_ModelElasticBit":
        policy = _checkPolicy(decodePolicy)
        for matrix in self._matrices():
            matrix.setDecodePolicy(policy)
        self.decodePolicy = policy
        return self

    def setBackend(self, backend: str) -> "_ModelElasticBit":
        for _, layer in self._compressed_layers():
            layer.set_backend(backend)
        return self

    def summary(self) -> str:
        """Print and return a per-layer table: stored width, execution width,
        planner and selected error, after the backend facts."""
        info = ElasticBit.backend()
        active = self.activeOptimization
        facts = [
            ("Threshold", self.threshold),
            ("Decode Policy", self.decodePolicy),
            ("Backend", info.architecture or "unavailable"),
            ("Prefill", info.prefill or "unknown"),
            ("Decode Engine", info.decodeEngine or "unknown"),
            ("Decode Status", info.decodeStatus or "unknown"),
            ("Decode Planner", info.decodePlanner or "unknown"),
            ("Decode Validate", info.decodeValidation or "unknown"),
            ("Activate DType", info.activateDType or "unknown"),
            ("Optimize Cache", f"{len(self.optimizationProfiles)} profile(s)"),
            ("Optimize Active", "none" if active is None else str(active.get("planner", "unknown"))),
        ]
        widths = (36, 8, 10, 14, 10)
        cells = [("Layer", "Stored", "Execute", "Planner", "Error")]
        for name, layer in self._compressed_layers():
            m = layer.matrix
            cells.append((name[:36], f"{m.storageBits}-bit", f"W{m.executionWidth}A16",
                          m.executionPlanner, f"{m.error:.6f}"))
        out = ["ElasticBit Summary", "-" * 60]
        out += [f"{label:<16s}: {value}" for label, value in facts]
        out.append("")
        out += [" ".join([row[0].ljust(widths[0])] + [c.rjust(w) for c, w in zip(row[1:], widths[1:])])
                for row in cells]
        if self.skippedNames:
            out += ["", "Uncompressed (no safe calibration path):"]
            out += ["  " + n for n in self.skippedNames]
        text = "\n".join(out)
        print(text)
        return text


def _semanticOutputWeightIds(model: nn.Module) -> set[int]:
    """Weight ids of the model's semantic output head, via get_output_embeddings().

    Architecture-agnostic (core.py:550-568): models without that method, or
    whose head is not an nn.Linear, protect nothing.
    """
    getter = getattr(model, "get_output_embeddings", None)
    if not callable(getter):
        return set()
    try:
        head = getter()
    except Exception:
        return set()
    return {id(head.weight)} if isinstance(head, nn.Linear) else set()


class _RowRecorder:
    """Forward pre-hooks that keep, per Linear name, the first `limit` input rows
    the Linear sees during the calibration pass (the reference analyzes only the
    first 32 rows of each Linear, core.py:734)."""

    def __init__(self, limit: int) -> None:
        self.limit = int(limit)
        self._rows: dict[str, list[torch.Tensor]] = {}
        self._count: dict[str, int] = {}
        self._first: dict[str, torch.Tensor] = {}  # the input object of each name's first call

    def _pre_hook(self, name: str):
        def record(_module: nn.Module, inputs: tuple[Any, ...]) -> None:
            if not inputs or not torch.is_tensor(inputs[0]):
                return
            self._first.setdefault(name, inputs[0])  # held, so its id stays unique
            room = self.limit - self._count.get(name, 0)
            if room <= 0:
                return
            x = inputs[0].detach()
            kept = x.reshape(-1, x.shape[-1])[:room].float().cpu()
            self._rows.setdefault(name, []).append(kept)
            self._count[name] = self._count.get(name, 0) + int(kept.shape[0])
        return record

    def capture(self, model: nn.Module, names: Sequence[str], feed: _CalibrationFeed,
                device: torch.device) -> None:
        handles = [model.get_submodule(n).register_forward_pre_hook(self._pre_hook(n))
                   for n in names]
        try:
            feed.replay(model, device)
        finally:
            for h in handles:
                h.remove()

    def rows_for(self, names: Sequence[str]) -> np.ndarray | None:
        """The recorded rows of `names` (in that order) as one float32 matrix."""
        parts = [t for n in names for t in self._rows.get(n, ())]
        if not parts:
            return None
        return np.ascontiguousarray(torch.cat(parts, 0).numpy(), dtype=np.float32)

    def release(self, names: Sequence[str]) -> None:
        for n in names:
            self._rows.pop(n, None)

    def siblings(self, names: Sequence[str]) -> list[list[str]]:
        """Groups (2..8 names, in `names` order) whose first call received the very
        same input tensor object."""
        by_input: dict[int, list[str]] = {}
        for n in names:
            x = self._first.get(n)
            if x is not None:
                by_input.setdefault(id(x), []).append(n)
        self._first.clear()
        return [g for g in by_input.values() if 2 <= len(g) <= 8]


@dataclass
class _LinearGroup:
    """All Linear modules that share one weight tensor (compressed once)."""
    names: list[str]
    output_head: bool  # the preserved semantic output head: kept FP16, listed as skipped
    tied: bool         # weight shared with an embedding: kept FP16 silently


def _linear_groups(model: nn.Module, preserve_head: bool) -> list[_LinearGroup]:
    embedding = {id(m.weight) for m in model.modules() if isinstance(m, nn.Embedding)}
    heads = _semanticOutputWeightIds(model) if preserve_head else set()
    groups: dict[int, _LinearGroup] = {}
    for name, module in model.named_modules():
        if isinstance(module, nn.Linear):
            key = id(module.weight)
            if key not in groups:
                groups[key] = _LinearGroup([], key in heads, key in embedding)
            groups[key].names.append(name)
    return list(groups.values())


def _compress_linear(module: nn.Linear, rows: np.ndarray, threshold: float, policy: str,
                     device: torch.device) -> tuple[RuntimeMatrix, int, float]:
    """Width selection on the module's FP16 weight, then the matrix on its GPU."""
    bits, err, codes, scales = _selectBitsTorch(module.weight, rows, threshold)
    with torch.cuda.device(device):
        if bits <= 15:
            matrix = RuntimeMatrix._compressSelectedCodes(codes, scales, bits, threshold, err,
                                                          decodePolicy=policy)
        else:  # 16: the FP16 weight itself
            matrix = RuntimeMatrix._compressSelected(module.weight.detach().float(), bits,
                                                     threshold, err, decodePolicy=policy)
    return matrix, bits, err


def _progress_enabled() -> bool:
    flag = os.environ.get("MLBRICKS_ELASTICBIT_PROGRESS", "")
    return flag.strip().lower() in {"1", "true", "yes", "on"}


def _write_artifact(model: nn.Module, ctl: "_ModelElasticBit", dest: Path) -> None:
    """The `.elasticbit` zip: manifest.json (the reference writer's keys and order),
    one MLB4 file per distinct matrix under matrices/, and state.pt (the model's
    state_dict).  Matrices are staged through a temporary file (the runtime writes
    MLB4 to a path); the manifest and state go straight into the archive."""
    layers: list[dict[str, Any]] = []
    members: dict[int, str] = {}
    with tempfile.TemporaryDirectory(prefix="elasticbit-save-") as tmp, \
            zipfile.ZipFile(dest, "w", compression=zipfile.ZIP_DEFLATED) as zf:
        for name in ctl.compressedNames:
            try:
                layer = model.get_submodule(name)
            except AttributeError:
                layer = None
            if not isinstance(layer, _ElasticLinear):
                raise RuntimeError(f"ElasticBit layer disappeared before save: {name}")
            member = members.get(id(layer.matrix))
            if member is None:
                member = f"matrix_{len(members):05d}.mlb"
                members[id(layer.matrix)] = member
                staged = Path(tmp) / member
                layer.matrix.save(staged)
                zf.write(staged, f"matrices/{member}")
            layers.append({"name": name, "matrix": member, "inFeatures": layer.inFeatures,
                           "outFeatures": layer.outFeatures, "hasBias": layer.bias is not None})
        manifest = {
            "format": _ARTIFACT_FORMAT,
            "version": _ARTIFACT_VERSION,
            "threshold": ctl.threshold,
            "decodePolicy": ctl.decodePolicy,
            "compressedNames": list(ctl.compressedNames),
            "skippedNames": list(ctl.skippedNames),
            "optimizationProfiles": ctl.optimizationProfiles,
            "layers": layers,
        }
        zf.writestr("manifest.json", json.dumps(manifest, indent=2))
        state = io.BytesIO()
        torch.save(model.state_dict(), state)
        zf.writestr("state.pt", state.getvalue())


def _read_artifact(model: nn.Module, src: Path, policy: str, route: str) -> nn.Module:
    """Rebuild a `.elasticbit` artifact's compressed layers inside `model` (the
    architecture), then load its state_dict; each MLB4 member is loaded once and
    shared by every layer entry naming it."""
    with zipfile.ZipFile(src, "r") as zf:
        manifest = json.loads(zf.read("manifest.json").decode("utf-8"))
        if (manifest.get("format") != _ARTIFACT_FORMAT
                or manifest.get("version") != _ARTIFACT_VERSION):
            raise ValueError("Unsupported ElasticBit model artifact")
        matrices: dict[str, RuntimeMatrix] = {}
        names: list[str] = []
        with tempfile.TemporaryDirectory(prefix="elasticbit-load-") as tmp:
            for entry in manifest["layers"]:
                name = str(entry["name"])
                try:
                    target = model.get_submodule(name)
                except AttributeError:
                    target = None
                if not isinstance(target, nn.Linear):
                    raise ValueError(
                        f"Model architecture does not contain expected Linear layer: {name}")
                device = target.weight.device
                if device.type != "cuda":
                    raise RuntimeError("ElasticBit.load() requires the target model on CUDA")
                member = str(entry["matrix"])
                if member not in matrices:
                    staged = Path(tmp) / Path(member).name
                    staged.write_bytes(zf.read(f"matrices/{member}"))
                    with torch.cuda.device(device):
                        matrices[member] = RuntimeMatrix.load(staged, decodePolicy=policy)
                bias = target.bias if bool(entry["hasBias"]) else None
                layer = _ElasticLinear(matrices[member], int(entry["inFeatures"]),
                                       int(entry["outFeatures"]), bias, backend=route)
                _swap_module(model, name, layer.to(device=device))
                names.append(name)
        state = torch.load(io.BytesIO(zf.read("state.pt")), map_location=_moduleDevice(model),
                           weights_only=True)
    model.load_state_dict(state, strict=True)
    model.elasticbit = _ModelElasticBit(
        model, threshold=float(manifest["threshold"]), decodePolicy=policy,
        compressedNames=names, skippedNames=tuple(manifest.get("skippedNames", ())),
        optimizationProfiles=manifest.get("optimizationProfiles", {}))
    return model


class ElasticBit:
    """ElasticBit public namespace."""

    RuntimeMatrix = RuntimeMatrix

    @staticmethod
    def analyze(weights: Any, calibrationData: Any, threshold: float) -> BitAnalysis:
        native = _requireNative()
        raw = native.analyze(_as_f32_matrix(weights, "weights"),
                             _as_f32_matrix(calibrationData, "calibrationData"),
                             float(threshold))
        cands = tuple(BitCandidate(
            bits=int(c["bits"]), hardwareNativeError=float(c["hardwareNativeError"]),
            fullPrecisionError=float(c["fullPrecisionError"]), error=float(c["error"]),
            storageBytes=int(c["storageBytes"]), memoryReduction=float(c["memoryReduction"]),
            passes=bool(c["passes"])) for c in raw["candidates"])
        return BitAnalysis(threshold=float(raw["threshold"]),
                           selectedBits=int(raw["selectedBits"]),
                           selectedError=float(raw["selectedError"]), candidates=cands)

    @staticmethod
    def compressMatrix(weights: Any, calibrationData: Any, threshold: float,
                       decodePolicy: str = "hardwareNative") -> RuntimeMatrix:
        return RuntimeMatrix.compress(weights, calibrationData, threshold,
                                      decodePolicy=decodePolicy)

    @staticmethod
    def loadMatrix(path: str | Path, decodePolicy: str = "hardwareNative") -> RuntimeMatrix:
        return RuntimeMatrix.load(path, decodePolicy=decodePolicy)

    @staticmethod
    def backend() -> BackendInfo:
        if not _nativeAvailable():
            err = _nativeImportError()
            return BackendInfo(available=False, device=None, deviceIndex=None, architecture=None,
                               weightWidths=(), activateDType=None, prefill=None,
                               decodePlanner=None, decodeEngine=None, decodeStatus=None,
                               decodeValidation=None, validated=False,
                               error=None if err is None else str(err))
        raw = _requireNative().backendInfo()
        return BackendInfo(
            available=True, device=str(raw["device"]), deviceIndex=int(raw["deviceIndex"]),
            architecture=str(raw["architecture"]),
            weightWidths=tuple(int(v) for v in raw["weightWidths"]),
            activateDType=str(raw["activateDType"]), prefill=str(raw["prefill"]),
            decodePlanner=str(raw["decodePlanner"]), decodeEngine=str(raw["decodeEngine"]),
            decodeStatus=str(raw["decodeStatus"]), decodeValidation=str(raw["decodeValidation"]),
            validated=bool(raw["validated"]))

    @staticmethod
    def optimize(model: nn.Module, force: bool = False) -> nn.Module:
        """Hardware profile hook (reference: Stage-2F, a T4/Granite-8B notebook port).

        The Stage-2F profile is specific to Tesla T4 and Granite shapes
        (stage2f.py); the B200 runtime already executes every compressed
        matrix through its native kernels, so no profile applies.  The model is
        validated and returned unchanged, with the decision recorded on
        ``model.elasticbit.activeOptimization``.
        """
        if not isinstance(model, nn.Module):
            raise TypeError("ElasticBit.optimize() expects a torch.nn.Module")
        controller = getattr(model, "elasticbit", None)
        if not isinstance(controller, _ModelElasticBit):
            raise ValueError("ElasticBit.optimize() expects a model produced by "
                             "ElasticBit.compress() or ElasticBit.load()")
        controller.activeOptimization = {
            "planner": "none",
            "reason": "Stage-2F profiles are Tesla-T4/Granite specific; B200 uses libebx kernels",
            "force": bool(force),
        }
        return model

    @staticmethod
    def reduce(model: nn.Module, sample: Any = None) -> nn.Module:
        """Stage-2G FX affine-chain reducer: outside the compressed-linear path."""
        raise NotImplementedError(
            "ElasticBit.reduce (Stage-2G graph reducer) is not part of the B200 runtime")

    @staticmethod
    def compress(model: nn.Module, calibrationData: Any, threshold: float,
                 decodePolicy: str = "hardwareNative", preserveOutputHead: bool = True,
                 backend: str = "auto") -> nn.Module:
        """Replace every compressible nn.Linear of a CUDA FP16 model by an ElasticBit
        layer whose storage width the calibration pass selects (reference:
        core.py:695-898; `backend` is an additive keyword choosing the route)."""
        if not isinstance(model, nn.Module):
            raise TypeError("ElasticBit.compress() expects a torch.nn.Module")
        _requireNative()
        policy = _checkPolicy(decodePolicy)
        route = normalize_backend(backend)
        feed = _CalibrationFeed(calibrationData)
        device = _moduleDevice(model)
        if device.type != "cuda":
            raise RuntimeError("ElasticBit model compression currently requires a CUDA model")
        if any(isinstance(m, nn.Linear) and m.weight.dtype != torch.float16
               for m in model.modules()):
            raise RuntimeError(
                "ElasticBit.compress() currently requires FP16 Linear weights. "
                "Convert the model to float16 before compression.")

        groups = _linear_groups(model, bool(preserveOutputHead))
        work = [g for g in groups if not (g.output_head or g.tied)]
        recorder = _RowRecorder(_CALIBRATION_ROWS)
        model.eval()
        recorder.capture(model, [n for g in work for n in g.names], feed, device)

        skipped = [n for g in groups if g.output_head for n in g.names]
        compressed: list[str] = []
        verbose = _progress_enabled()
        thr = float(threshold)
        for index, group in enumerate(work, start=1):
            rows = recorder.rows_for(group.names)
            if rows is None:  # never reached by the calibration inputs
                skipped.extend(group.names)
                continue
            module = model.get_submodule(group.names[0])
            if not isinstance(module, nn.Linear):
                raise RuntimeError(f"ElasticBit expected Linear module at {group.names[0]}")
            if verbose:
                print(f"[ElasticBit] {index}/{len(work)} analyzing {group.names[0]} "
                      f"shape={tuple(module.weight.shape)} rows={rows.shape[0]}", flush=True)
            matrix, bits, err = _compress_linear(module, rows, thr, policy, device)
            if verbose:
                print(f"[ElasticBit] {index}/{len(work)} selected {bits}-bit error={err:.6g}",
                      flush=True)
            for name in group.names:
                current = model.get_submodule(name)
                if not isinstance(current, nn.Linear):
                    raise RuntimeError(f"ElasticBit expected Linear module at {name}")
                layer = _ElasticLinear(matrix, current.in_features, current.out_features,
                                       current.bias, backend=route)
                _swap_module(model, name, layer.to(device=device))
                compressed.append(name)
            recorder.release(group.names)
            del module, matrix, rows
            gc.collect()
            torch.cuda.empty_cache()

        # siblings that read one input share a fused decode launch
        done = set(compressed)
        for names in recorder.siblings([n for g in work for n in g.names]):
            if all(n in done for n in names):
                layers = [model.get_submodule(n) for n in names]
                group = _FusedGroup(layers)
                for layer in layers:
                    layer._fused = group

        model.elasticbit = _ModelElasticBit(model, threshold=thr, decodePolicy=policy,
                                            compressedNames=compressed, skippedNames=skipped)
        return model

    @staticmethod
    def save(model: nn.Module, path: str | Path) -> Path:
        """Write the compressed model as a `.elasticbit` artifact (reference:
        core.py:900-953; same members, manifest keys and MLB4 files)."""
        ctl = getattr(model, "elasticbit", None)
        if not isinstance(ctl, _ModelElasticBit):
            raise ValueError("ElasticBit.save() expects a model produced by ElasticBit.compress()")
        dest = Path(path)
        dest.parent.mkdir(parents=True, exist_ok=True)
        _write_artifact(model, ctl, dest)
        return dest

    @staticmethod
    def load(model: nn.Module, path: str | Path, decodePolicy: str = "hardwareNative",
             backend: str = "auto") -> nn.Module:
        """Restore a `.elasticbit` artifact into `model`, the uncompressed architecture
        (reference: core.py:955-1017)."""
        if not isinstance(model, nn.Module):
            raise TypeError("ElasticBit.load() requires the model architecture as its first argument")
        _requireNative()
        src = Path(path)
        if not src.exists():
            raise FileNotFoundError(src)
        route = normalize_backend(backend)
        policy = _checkPolicy(decodePolicy)
        return _read_artifact(model, src, policy, route)
