"""Operator route planner for ``backend='auto'`` (reference: mlbricks/planner.py).

Only the operator-routing half of the reference planner is on the
compressed-linear path: ``qualify_operator_once`` (planner.py:570-776),
``select_operator`` (:778-835), the parity comparison (:453-568) and the
operator defaults (:34-54, ``elastic_linear -> pytorch``).  Semantics kept:

* explicit ``native`` / ``pytorch`` requests are never overridden; ``native``
  raises when the native route is unavailable;
* ``auto`` runs the PyTorch candidate once as the reference, requires the
  native output to be allclose (fp16/bf16: rtol = atol = 2e-2) before native
  may compete, then times each candidate (median of `trials` CUDA-event
  samples) and keeps the default unless the other is >= `switch_margin`
  faster; the decision is frozen per owner object;
* a native exception or parity failure freezes ``pytorch`` for that owner.
"""
from __future__ import annotations

import time
from typing import Callable, Final, Mapping

import torch

from .runtime import normalize_backend

AUTO_OPERATOR_DEFAULTS: Final[dict[str, str]] = {"elastic_linear": "pytorch"}


class MLBricksExecutionPlanner:
    def __init__(self) -> None:
        self.operator_cache: dict[tuple[object, ...], str] = {}
        self.operator_benchmarks: dict[tuple[object, ...], dict[str, float]] = {}
        self.operator_reasons: dict[tuple[object, ...], str] = {}
        self._operator_revision = 0

    # -- keys ----------------------------------------------------------------
    @staticmethod
    def operator_key(op: str, tensor: torch.Tensor, *, training: bool,
                     extra: tuple[object, ...] = ()) -> tuple[object, ...]:
        dev = tensor.device
        cap = torch.cuda.get_device_capability(dev) if dev.type == "cuda" else (0, 0)
        return (str(op), dev.type, dev.index, tuple(cap), str(tensor.dtype),
                tuple(tensor.shape[-1:]), bool(training), tuple(extra))

    def _auto_default(self, op: str, fallback: str | None = None) -> str:
        v = str(fallback or AUTO_OPERATOR_DEFAULTS.get(str(op), "pytorch")).lower()
        return v if v in {"native", "pytorch"} else "pytorch"

    @staticmethod
    def _parity_tolerances(tensor: torch.Tensor, *, rtol: float | None,
                           atol: float | None) -> tuple[float, float]:
        low = tensor.dtype in {torch.float16, torch.bfloat16}
        rtol = (2.0e-2 if low else 1.0e-4) if rtol is None else float(rtol)
        atol = (2.0e-2 if low else 1.0e-5) if atol is None else float(atol)
        return max(0.0, rtol), max(0.0, atol)

    @staticmethod
    def _compare_candidate_outputs(reference: object, candidate: object, *, rtol: float,
                                   atol: float, path: str = "output") -> tuple[bool, dict]:
        stats: dict[str, object] = {"checked": True, "allclose": True, "rtol": rtol, "atol": atol,
                                    "tensor_leaves": 0, "max_abs": 0.0, "max_relative_l2": 0.0,
                                    "mismatch": None}

        def fail(where: str, why: str) -> bool:
            stats["allclose"] = False
            if stats["mismatch"] is None:
                stats["mismatch"] = f"{where}: {why}"
            return False

        def visit(ref: object, cand: object, where: str) -> bool:
            if torch.is_tensor(ref) or torch.is_tensor(cand):
                if not (torch.is_tensor(ref) and torch.is_tensor(cand)):
                    return fail(where, "tensor/non-tensor type mismatch")
                if tuple(ref.shape) != tuple(cand.shape):
                    return fail(where, f"shape {tuple(ref.shape)} != {tuple(cand.shape)}")
                r = ref.detach()
                c = cand.detach().to(r.device)
                if r.is_floating_point():
                    rf, cf = r.float(), c.float()
                    diff = (cf - rf).abs()
                    if diff.numel():
                        stats["max_abs"] = max(float(stats["max_abs"]), float(diff.max()))
                        rel = float(torch.linalg.vector_norm(cf - rf) /
                                    (torch.linalg.vector_norm(rf) + 1.0e-12))
                        stats["max_relative_l2"] = max(float(stats["max_relative_l2"]), rel)
                    ok = bool(torch.allclose(cf, rf, rtol=rtol, atol=atol))
                else:
                    ok = bool(torch.equal(c, r))
                stats["tensor_leaves"] = int(stats["tensor_leaves"]) + 1
                return True if ok else fail(where, "tensor values differ from PyTorch reference")
            if isinstance(ref, Mapping) or isinstance(cand, Mapping):
                if not (isinstance(ref, Mapping) and isinstance(cand, Mapping)):
                    return fail(where, "mapping/non-mapping type mismatch")
                if set(ref) != set(cand):
                    return fail(where, "mapping keys differ")
                return all([visit(ref[k], cand[k], f"{where}[{k!r}]") for k in sorted(ref, key=repr)])
            if isinstance(ref, (tuple, list)) or isinstance(cand, (tuple, list)):
                if type(ref) is not type(cand) or len(ref) != len(cand):
                    return fail(where, "sequence type or length differs")
                return all([visit(a, b, f"{where}[{i}]") for i, (a, b) in enumerate(zip(ref, cand))])
            if ref is None or cand is None:
                return True if ref is cand else fail(where, "None/non-None mismatch")
            return True if ref == cand else fail(where, f"value mismatch: {ref!r} != {cand!r}")

        ok = visit(reference, candidate, path)
        stats["allclose"] = bool(ok and stats["allclose"])
        return bool(stats["allclose"]), stats

    # -- selection -----------------------------------------------------------
    def select_operator(self, op: str, tensor: torch.Tensor, *, requested_backend: str = "auto",
                        native_available: bool, native_supports_training: bool = False,
                        training: bool | None = None, extra: tuple[object, ...] = (),
                        default_auto: str | None = None) -> str:
        policy = normalize_backend(requested_backend, warn_legacy=True)
        is_training = bool(torch.is_grad_enabled()) if training is None else bool(training)
        if policy == "pytorch":
            return "pytorch"
        if policy == "native":
            if not native_available:
                raise RuntimeError(
                    f"backend='native' requested but native route for {op!r} is unavailable")
            if is_training and not native_supports_training:
                raise RuntimeError(f"backend='native' requested for {op!r}, but its native route "
                                   "is inference-only for this call")
            return "native"
        key = self.operator_key(op, tensor, training=is_training, extra=extra)
        if is_training and not native_supports_training:
            self.operator_cache[key], self.operator_reasons[key] = "pytorch", "training-safe:pytorch"
            return "pytorch"
        if not native_available:
            self.operator_cache[key] = "pytorch"
            self.operator_reasons[key] = "native-unavailable:pytorch"
            return "pytorch"
        cached = self.operator_cache.get(key)
        if cached in {"native", "pytorch"}:
            return cached
        route = self._auto_default(op, default_auto)
        self.operator_cache[key], self.operator_reasons[key] = route, f"heuristic:{route}"
        return route

    def select_operator_once(self, owner: object, op: str, tensor: torch.Tensor, **kw) -> str:
        cache = getattr(owner, "_mlbricks_frozen_auto_routes", None)
        training = kw.get("training")
        key = (str(op), bool(torch.is_grad_enabled() if training is None else training))
        if isinstance(cache, dict) and cache.get(key) in {"native", "pytorch"}:
            return cache[key]
        route = self.select_operator(op, tensor, **kw)
        try:
            if not isinstance(cache, dict):
                cache = {}
                setattr(owner, "_mlbricks_frozen_auto_routes", cache)
            cache[key] = route
        except Exception:
            pass
        return route

    def qualify_operator_once(self, owner: object, op: str, tensor: torch.Tensor,
                              candidates: Mapping[str, Callable[[], object]], *,
                              requested_backend: str = "auto", native_available: bool,
                              native_supports_training: bool = False, training: bool | None = None,
                              extra: tuple[object, ...] = (), default_auto: str | None = None,
                              warmup: int = 2, trials: int = 5, switch_margin: float = 0.05,
                              verify_parity: bool = True, parity_rtol: float | None = None,
                              parity_atol: float | None = None,
                              freeze_on: tuple[object, ...] = ()) -> str:
        """One parity-checked timing race per (op, training, *freeze_on), then frozen.

        ``freeze_on`` names the regime a decision holds for (for example the
        row-count regime of a linear): each distinct value races and freezes on
        its own, so a decision taken on one regime never routes another.
        """
        policy = normalize_backend(requested_backend, warn_legacy=True)
        is_training = bool(torch.is_grad_enabled()) if training is None else bool(training)
        common = dict(native_available=native_available,
                      native_supports_training=native_supports_training, training=is_training,
                      extra=extra, default_auto=default_auto)
        if policy != "auto":
            return self.select_operator(op, tensor, requested_backend=policy, **common)
        if is_training and not native_supports_training:
            return "pytorch"
        if not native_available:
            return self.select_operator_once(owner, op, tensor, requested_backend="auto", **common)
        cache = getattr(owner, "_mlbricks_frozen_auto_routes", None)
        if not isinstance(cache, dict):
            cache = {}
            try:
                setattr(owner, "_mlbricks_frozen_auto_routes", cache)
            except Exception:
                pass
        fkey = (str(op), bool(is_training), *freeze_on)
        if cache.get(fkey) in {"native", "pytorch"}:
            return cache[fkey]
        usable = {n: f for n, f in candidates.items() if n in {"native", "pytorch"} and callable(f)}
        if not usable:
            return self.select_operator_once(owner, op, tensor, requested_backend="auto", **common)

        key = self.operator_key(op, tensor, training=is_training, extra=extra)
        timings: dict[str, float] = {}
        errors: dict[str, str] = {}
        parity: dict[str, object] = {"checked": False, "allclose": None}

        def freeze(route: str, reason: str) -> str:
            self.operator_benchmarks[key] = dict(timings)
            if self.operator_cache.get(key) != route:
                self._operator_revision += 1
            self.operator_cache[key] = route
            self.operator_reasons[key] = reason
            cache[fkey] = route
            try:
                details = getattr(owner, "_mlbricks_frozen_auto_details", None)
                if not isinstance(details, dict):
                    details = {}
                    setattr(owner, "_mlbricks_frozen_auto_details", details)
                details[fkey] = {"route": route, "timings_ms": dict(timings),
                                 "errors": dict(errors), "parity": dict(parity), "reason": reason}
            except Exception:
                pass
            return route

        def sync() -> None:
            if tensor.is_cuda:
                torch.cuda.synchronize(tensor.device)

        if verify_parity and "pytorch" in usable and "native" in usable:
            rtol, atol = self._parity_tolerances(tensor, rtol=parity_rtol, atol=parity_atol)
            try:
                ref_out = usable["pytorch"]()
                sync()
            except Exception as exc:
                errors["pytorch_reference"] = f"{type(exc).__name__}: {exc}"
                parity.update({"checked": False, "rtol": rtol, "atol": atol,
                               "reference_error": errors["pytorch_reference"]})
                return freeze("pytorch", "correctness-gate:reference-error;pytorch")
            try:
                nat_out = usable["native"]()
                sync()
            except Exception as exc:
                errors["native_validation"] = f"{type(exc).__name__}: {exc}"
                parity.update({"checked": True, "allclose": False, "rtol": rtol, "atol": atol,
                               "mismatch": "native candidate raised during correctness validation"})
                return freeze("pytorch", "correctness-gate:native-error;pytorch")
            ok, details = self._compare_candidate_outputs(ref_out, nat_out, rtol=rtol, atol=atol)
            parity.clear()
            parity.update(details)
            if not ok:
                return freeze("pytorch", "correctness-gate:parity-failed;pytorch")

        for name, fn in usable.items():
            try:
                for _ in range(max(0, int(warmup))):
                    fn()
                sync()
                samples = []
                for _ in range(max(1, int(trials))):
                    if tensor.is_cuda:
                        a = torch.cuda.Event(enable_timing=True)
                        b = torch.cuda.Event(enable_timing=True)
                        a.record()
                        fn()
                        b.record()
                        b.synchronize()
                        samples.append(float(a.elapsed_time(b)))
                    else:
                        t0 = time.perf_counter()
                        fn()
                        samples.append((time.perf_counter() - t0) * 1e3)
                samples.sort()
                timings[name] = samples[len(samples) // 2]
            except Exception as exc:
                errors[name] = f"{type(exc).__name__}: {exc}"
        if not timings:
            return self.select_operator_once(owner, op, tensor, requested_backend="auto", **common)
        fastest = min(timings, key=timings.get)
        default = self._auto_default(op, default_auto)
        route = fastest
        if default in timings and fastest != default:
            gain = (timings[default] - timings[fastest]) / max(timings[default], 1.0e-12)
            if gain < max(0.0, float(switch_margin)):
                route = default
        reason = ("correctness-pass;benchmark-once:" if parity.get("checked") else
                  "benchmark-once:") + ",".join(f"{n}={ms:.6f}ms" for n, ms in sorted(timings.items()))
        if errors:
            reason += ";errors=" + ",".join(f"{k}:{v}" for k, v in sorted(errors.items()))
        return freeze(route, reason)

    def set_operator_route(self, op: str, tensor: torch.Tensor, route: str, *,
                           training: bool = False, extra: tuple[object, ...] = ()) -> None:
        route = normalize_backend(route)
        if route not in {"native", "pytorch"}:
            raise ValueError("route must be 'native' or 'pytorch'")
        key = self.operator_key(op, tensor, training=training, extra=extra)
        self.operator_cache[key] = route
        self.operator_reasons[key] = f"manual:{route}"
        self._operator_revision += 1


EXECUTION_PLANNER = MLBricksExecutionPlanner()

__all__ = ["AUTO_OPERATOR_DEFAULTS", "MLBricksExecutionPlanner", "EXECUTION_PLANNER"]
