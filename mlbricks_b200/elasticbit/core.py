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
    value = str(value)
    if value not in _POLICIES:
        raise ValueError("decodePolicy must be 'hardwareNative' or 'fullPrecision'")
    return value


def _toNumpy2D(value: Any, *, name: str) -> np.ndarray:
    if torch.is_tensor(value):
        value = value.detach().float().cpu().numpy()
    arr = np.asarray(value, dtype=np.float32)
    if arr.ndim != 2:
        raise ValueError(f"{name} must be a 2D matrix")
    return np.ascontiguousarray(arr, dtype=np.float32)


def _toCalibrationBatches(calibrationData: Any) -> list[Any]:
    if torch.is_tensor(calibrationData) or isinstance(calibrationData, Mapping):
        return [calibrationData]
    if isinstance(calibrationData, (str, bytes)):
        raise TypeError("calibrationData must contain model inputs, not text")
    try:
        batches = list(calibrationData)
    except TypeError as exc:
        raise TypeError(
            "calibrationData must be a model input or an iterable of model inputs") from exc
    if not batches:
        raise ValueError("calibrationData cannot be empty")
    return batches


def _callModel(model: nn.Module, batch: Any) -> Any:
    if isinstance(batch, Mapping):
        return model(**batch)
    if isinstance(batch, tuple):
        return model(*batch)
    return model(batch)


def _moveBatch(batch: Any, device: torch.device) -> Any:
    if torch.is_tensor(batch):
        return batch.to(device)
    if isinstance(batch, Mapping):
        return {k: _moveBatch(v, device) for k, v in batch.items()}
    if isinstance(batch, (tuple, list)):
        moved = [_moveBatch(v, device) for v in batch]
        return tuple(moved) if isinstance(batch, tuple) else moved
    return batch


def _relativeL2Torch(reference: torch.Tensor, candidate: torch.Tensor) -> float:
    ref = reference.float()
    cand = candidate.float()
    den = torch.linalg.vector_norm(ref).clamp_min(1.0e-30)
    return float((torch.linalg.vector_norm(cand - ref) / den).item())


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
    for p in module.parameters():
        return p.device
    for b in module.buffers():
        return b.device
    return torch.device("cpu")


def _replaceNamedModule(root: nn.Module, name: str, replacement: nn.Module) -> None:
    if not name:
        raise ValueError("ElasticBit cannot replace the root module")
    *parents, leaf = name.split(".")
    owner = root
    for part in parents:
        owner = owner._modules[part]
    owner._modules[leaf] = replacement


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
        w = _toNumpy2D(weights, name="weights")
        c = _toNumpy2D(calibrationData, name="calibrationData")
        return cls(native.RuntimeMatrix.compress(w, c, float(threshold), policy))

    @classmethod
    def _compressSelected(cls, weights: Any, selectedBits: int, threshold: float,
                          selectedError: float,
                          decodePolicy: str = "hardwareNative") -> "RuntimeMatrix":
        native = _requireNative()
        policy = _checkPolicy(decodePolicy)
        w = _toNumpy2D(weights, name="weights")
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

    def _layers(self) -> list[tuple[str, _ElasticLinear]]:
        modules = dict(self._model.named_modules())
        return [(n, modules[n]) for n in self.compressedNames
                if isinstance(modules.get(n), _ElasticLinear)]

    def setDecodePolicy(self, decodePolicy: str) -> "_ModelElasticBit":
        policy = _checkPolicy(decodePolicy)
        done: set[int] = set()
        for _, layer in self._layers():
            if id(layer.matrix) not in done:
                layer.matrix.setDecodePolicy(policy)
                done.add(id(layer.matrix))
        self.decodePolicy = policy
        return self

    def setBackend(self, backend: str) -> "_ModelElasticBit":
        for _, layer in self._layers():
            layer.set_backend(backend)
        return self

    def summary(self) -> str:
        be = ElasticBit.backend()
        lines = [
            "ElasticBit Summary",
            "-" * 60,
            f"Threshold       : {self.threshold}",
            f"Decode Policy   : {self.decodePolicy}",
            f"Backend         : {be.architecture or 'unavailable'}",
            f"Prefill         : {be.prefill or 'unknown'}",
            f"Decode Engine   : {be.decodeEngine or 'unknown'}",
            f"Decode Status   : {be.decodeStatus or 'unknown'}",
            f"Decode Planner  : {be.decodePlanner or 'unknown'}",
            f"Decode Validate : {be.decodeValidation or 'unknown'}",
            f"Activate DType  : {be.activateDType or 'unknown'}",
            f"Optimize Cache  : {len(self.optimizationProfiles)} profile(s)",
            "Optimize Active : " + ("none" if self.activeOptimization is None
                                    else str(self.activeOptimization.get("planner", "unknown"))),
            "",
            f"{'Layer':36s} {'Stored':>8s} {'Execute':>10s} {'Planner':>14s} {'Error':>10s}",
        ]
        for name, layer in self._layers():
            m = layer.matrix
            lines.append(f"{name[:36]:36s} {str(m.storageBits) + '-bit':>8s} "
                         f"{'W' + str(m.executionWidth) + 'A16':>10s} "
                         f"{m.executionPlanner:>14s} {m.error:10.6f}")
        if self.skippedNames:
            lines += ["", "Uncompressed (no safe calibration path):"]
            lines += [f"  {n}" for n in self.skippedNames]
        text = "\n".join(lines)
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


class ElasticBit:
    """ElasticBit public namespace."""

    RuntimeMatrix = RuntimeMatrix

    @staticmethod
    def analyze(weights: Any, calibrationData: Any, threshold: float) -> BitAnalysis:
        native = _requireNative()
        raw = native.analyze(_toNumpy2D(weights, name="weights"),
                             _toNumpy2D(calibrationData, name="calibrationData"),
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
        if not isinstance(model, nn.Module):
            raise TypeError("ElasticBit.compress() expects a torch.nn.Module")
        _requireNative()
        policy = _checkPolicy(decodePolicy)
        route = normalize_backend(backend)
        batches = _toCalibrationBatches(calibrationData)
        device = _moduleDevice(model)
        if device.type != "cuda":
            raise RuntimeError("ElasticBit model compression currently requires a CUDA model")
        for module in model.modules():
            if isinstance(module, nn.Linear) and module.weight.dtype != torch.float16:
                raise RuntimeError(
                    "ElasticBit.compress() currently requires FP16 Linear weights. "
                    "Convert the model to float16 before compression.")

        embedding_ids = {id(m.weight) for m in model.modules() if isinstance(m, nn.Embedding)}
        head_ids = _semanticOutputWeightIds(model) if bool(preserveOutputHead) else set()
        protected = embedding_ids | head_ids

        # Calibration capture: the first 32 input rows each Linear sees.
        captured: dict[str, list[np.ndarray]] = {}

        def make_hook(name: str):
            def hook(_mod: nn.Module, inputs: tuple[Any, ...]) -> None:
                if not inputs or not torch.is_tensor(inputs[0]):
                    return
                t = inputs[0]
                have = sum(a.shape[0] for a in captured.get(name, []))
                room = _CALIBRATION_ROWS - have
                if room <= 0:
                    return
                rows = t.detach().float().reshape(-1, t.shape[-1])[:room]
                captured.setdefault(name, []).append(rows.cpu().numpy().astype(np.float32))
            return hook

        names_by_weight: dict[int, list[str]] = {}
        hooks = []
        for name, module in model.named_modules():
            if isinstance(module, nn.Linear):
                names_by_weight.setdefault(id(module.weight), []).append(name)
                if id(module.weight) not in protected:
                    hooks.append(module.register_forward_pre_hook(make_hook(name)))
        model.eval()
        try:
            with torch.inference_mode():
                for batch in batches:
                    _callModel(model, _moveBatch(batch, device))
        finally:
            for h in hooks:
                h.remove()

        skipped = [n for wid, names in names_by_weight.items() if wid in head_ids for n in names]
        compressed: list[str] = []
        todo = [(wid, names) for wid, names in names_by_weight.items() if wid not in protected]
        progress = os.environ.get("MLBRICKS_ELASTICBIT_PROGRESS", "").strip().lower() in {
            "1", "true", "yes", "on"}

        for index, (_, names) in enumerate(todo, start=1):
            module = model.get_submodule(names[0])
            if not isinstance(module, nn.Linear):
                raise RuntimeError(f"ElasticBit expected Linear module at {names[0]}")
            parts = [a for n in names for a in captured.get(n, [])]
            if not parts:
                skipped.extend(names)
                continue
            calib = np.ascontiguousarray(np.concatenate(parts, axis=0), dtype=np.float32)
            if progress:
                print(f"[ElasticBit] {index}/{len(todo)} analyzing {names[0]} "
                      f"shape={tuple(module.weight.shape)} rows={calib.shape[0]}", flush=True)
            bits, err, codes, scales = _selectBitsTorch(module.weight, calib, float(threshold))
            with torch.cuda.device(device):
                if bits <= 15:
                    matrix = RuntimeMatrix._compressSelectedCodes(
                        codes, scales, bits, float(threshold), err, decodePolicy=policy)
                else:
                    matrix = RuntimeMatrix._compressSelected(
                        module.weight.detach().float(), bits, float(threshold), err,
                        decodePolicy=policy)
            if progress:
                print(f"[ElasticBit] {index}/{len(todo)} selected {bits}-bit error={err:.6g}",
                      flush=True)
            for name in names:
                current = model.get_submodule(name)
                if not isinstance(current, nn.Linear):
                    raise RuntimeError(f"ElasticBit expected Linear module at {name}")
                repl = _ElasticLinear(matrix, current.in_features, current.out_features,
                                      current.bias, backend=route).to(device=device)
                _replaceNamedModule(model, name, repl)
                compressed.append(name)
                captured.pop(name, None)
            del module, codes, scales, calib, parts, matrix
            gc.collect()
            torch.cuda.empty_cache()

        model.elasticbit = _ModelElasticBit(model, threshold=float(threshold), decodePolicy=policy,
                                            compressedNames=compressed, skippedNames=skipped)
        return model

    @staticmethod
    def save(model: nn.Module, path: str | Path) -> Path:
        ctl = getattr(model, "elasticbit", None)
        if not isinstance(ctl, _ModelElasticBit):
            raise ValueError("ElasticBit.save() expects a model produced by ElasticBit.compress()")
        dest = Path(path)
        dest.parent.mkdir(parents=True, exist_ok=True)
        modules = dict(model.named_modules())
        with tempfile.TemporaryDirectory(prefix="elasticbit-save-") as tmp:
            root = Path(tmp)
            (root / "matrices").mkdir()
            files: dict[int, str] = {}
            layers = []
            for name in ctl.compressedNames:
                layer = modules.get(name)
                if not isinstance(layer, _ElasticLinear):
                    raise RuntimeError(f"ElasticBit layer disappeared before save: {name}")
                fname = files.get(id(layer.matrix))
                if fname is None:
                    fname = f"matrix_{len(files):05d}.mlb"
                    layer.matrix.save(root / "matrices" / fname)
                    files[id(layer.matrix)] = fname
                layers.append({"name": name, "matrix": fname, "inFeatures": layer.inFeatures,
                               "outFeatures": layer.outFeatures,
                               "hasBias": layer.bias is not None})
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
            (root / "manifest.json").write_text(json.dumps(manifest, indent=2), encoding="utf-8")
            torch.save(model.state_dict(), root / "state.pt")
            with zipfile.ZipFile(dest, "w", compression=zipfile.ZIP_DEFLATED) as zf:
                for f in sorted(root.rglob("*")):
                    if f.is_file():
                        zf.write(f, f.relative_to(root).as_posix())
        return dest

    @staticmethod
    def load(model: nn.Module, path: str | Path, decodePolicy: str = "hardwareNative",
             backend: str = "auto") -> nn.Module:
        if not isinstance(model, nn.Module):
            raise TypeError("ElasticBit.load() requires the model architecture as its first argument")
        _requireNative()
        src = Path(path)
        if not src.exists():
            raise FileNotFoundError(src)
        route = normalize_backend(backend)
        with tempfile.TemporaryDirectory(prefix="elasticbit-load-") as tmp:
            root = Path(tmp)
            with zipfile.ZipFile(src, "r") as zf:
                zf.extractall(root)
            manifest = json.loads((root / "manifest.json").read_text(encoding="utf-8"))
            if (manifest.get("format") != _ARTIFACT_FORMAT
                    or manifest.get("version") != _ARTIFACT_VERSION):
                raise ValueError("Unsupported ElasticBit model artifact")
            policy = _checkPolicy(decodePolicy)
            modules = dict(model.named_modules())
            cache: dict[str, RuntimeMatrix] = {}
            names: list[str] = []
            for entry in manifest["layers"]:
                name = str(entry["name"])
                target = modules.get(name)
                if not isinstance(target, nn.Linear):
                    raise ValueError(
                        f"Model architecture does not contain expected Linear layer: {name}")
                device = target.weight.device
                if device.type != "cuda":
                    raise RuntimeError("ElasticBit.load() requires the target model on CUDA")
                fname = str(entry["matrix"])
                matrix = cache.get(fname)
                if matrix is None:
                    with torch.cuda.device(device):
                        matrix = RuntimeMatrix.load(root / "matrices" / fname, decodePolicy=policy)
                    cache[fname] = matrix
                repl = _ElasticLinear(matrix, int(entry["inFeatures"]), int(entry["outFeatures"]),
                                      target.bias if bool(entry["hasBias"]) else None,
                                      backend=route).to(device=device)
                _replaceNamedModule(model, name, repl)
                names.append(name)
                modules[name] = repl
            state = torch.load(root / "state.pt", map_location=_moduleDevice(model),
                               weights_only=True)
            model.load_state_dict(state, strict=True)
            model.elasticbit = _ModelElasticBit(
                model, threshold=float(manifest["threshold"]), decodePolicy=policy,
                compressedNames=names, skippedNames=tuple(manifest.get("skippedNames", ())),
                optimizationProfiles=manifest.get("optimizationProfiles", {}))
            return model


__all__ = ["ElasticBit", "RuntimeMatrix", "BitAnalysis", "BitCandidate", "BackendInfo"]
