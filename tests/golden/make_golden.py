"""Generate golden vectors from the reference's own compiled ElasticBit runtime.

Run in a container that has the MLBricks reference tree:

    python oracle/build.py --reference      # builds oracle/_ref/_C.so from the reference source
    python tests/golden/make_golden.py      # writes tests/golden/analyze_golden.json

The reference extension's host analyzer ``_C.analyze`` (elasticbit_runtime.cu:
438-483) runs without a GPU.  For each case below the inputs are regenerated
from their numpy seed (their SHA-256 is stored so a changed RNG stream is
detected) and the analyzer's full output is recorded with repr()-exact floats.
tests/test_oracle.py pins the C oracle to these values; the GPU analyzer test
pins libebx's device analyzer to them.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "analyze_golden.json"


def _baseline_weights(rows: int, cols: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    sigma = np.exp(rng.uniform(np.log(0.005), np.log(0.05), size=(rows, 1)))
    w = rng.standard_normal((rows, cols), dtype=np.float32) * sigma.astype(np.float32)
    w[rng.random((rows, cols)) < 1.0e-3] *= 10.0
    return w.astype(np.float32)


def _normal(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).normal(0.0, scale, size=shape)).astype(np.float32)


def case_inputs(name: str):
    """(weights, calibration, threshold) for a named case; shared with the tests."""
    if name == "smoke_seed7":  # mlbricks/elasticbit/smoke.py:12-15
        rng = np.random.default_rng(7)
        w = rng.normal(0, 0.05, size=(64, 128)).astype(np.float32)
        c = rng.normal(0, 1, size=(8, 128)).astype(np.float32)
        return w, c, 0.02
    if name == "threshold_contract":  # tests/test_elasticbit_native.py:23-26
        rng = np.random.default_rng(20260918)
        w = rng.normal(0, 0.04, size=(96, 128)).astype(np.float32)
        c = rng.normal(0, 1, size=(12, 128)).astype(np.float32)
        return w, c, 0.02
    if name == "hardware_validation":  # examples/elasticbit_hardware_validation.py:26-29
        rng = np.random.default_rng(20260918)
        w = rng.normal(0.0, 0.04, size=(512, 512)).astype(np.float32)
        c = rng.normal(0.0, 1.0, size=(16, 512)).astype(np.float32)
        return w, c, 0.01
    if name.startswith("config1_"):  # 1536x384, 32 calibration rows
        thr = float(name.split("_")[1])
        w = _baseline_weights(1536, 384, seed=0)
        c = _normal((64, 128, 384), seed=1)[0, :32]
        return w, c, thr
    if name == "ragged_zero_row":  # odd shape, one all-zero row, outliers
        w = _baseline_weights(40, 72, seed=11)
        w[5] = 0.0
        c = _normal((9, 72), seed=12)
        return w, c, 0.03
    if name == "fp16_fallback":  # no width passes a zero threshold
        w = _normal((24, 40), seed=21, scale=0.03)
        c = _normal((5, 40), seed=22)
        return w, c, 0.0
    raise KeyError(name)


CASES = ["smoke_seed7", "threshold_contract", "hardware_validation", "config1_0.005",
         "config1_0.01", "config1_0.02", "ragged_zero_row", "fp16_fallback"]


def sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_reference():
    import torch  # noqa: F401  (loads libc10/libtorch that the extension links)
    so = ROOT / "oracle" / "_ref" / "_C.so"
    if not so.exists():
        sys.path.insert(0, str(ROOT))
        from oracle import build
        so = build.build_reference()
    spec = importlib.util.spec_from_file_location("_C", so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ref = load_reference()
    out = {"generator": "reference _C.analyze (mlbricks/elasticbit/csrc/elasticbit_runtime.cu)",
           "cases": {}}
    for name in CASES:
        w, c, thr = case_inputs(name)
        res = ref.analyze(w, c, thr)
        out["cases"][name] = {
            "shape": list(w.shape), "samples": int(c.shape[0]), "threshold": thr,
            "inputs_sha256": sha(w, c),
            "selectedBits": int(res["selectedBits"]),
            "selectedError": repr(float(res["selectedError"])),
            "candidates": [{k: (repr(float(v)) if isinstance(v, float) else v)
                            for k, v in cand.items()} for cand in res["candidates"]],
        }
        print(name, res["selectedBits"], res["selectedError"])
    OUT.write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", OUT)


if __name__ == "__main__":
    main()
