"""Golden vectors from the reference's own RuntimeMatrix, run on a GPU.

The reference's packing, MLB4 writer, dequantisation and FastWarp forward only
run with a CUDA device (every RuntimeMatrix constructor calls cudaGetDevice,
elasticbit_runtime.cu:1102,1129,1155).  This script loads the reference
extension built out of tree by ``oracle/build.py`` (``oracle/_ref/_C.so``) on
a GPU machine and records, for seeded small cases:

* the exact MLB4 file bytes written by ``RuntimeMatrix.save`` (base64);
* the dequantised weights of ``RuntimeMatrix.dequantize`` (SHA-256 of float32);
* the FP16 output of ``forwardTorch`` (FastWarp, M = 1) under
  ``fullPrecision`` (base64 of the fp16 bytes);
* for ``RuntimeMatrix.compress`` (matrix path): the selected width and error.

Usage (GPU machine, repo root; OUT is any writable path):
    python tests/golden/make_golden_ref_gpu.py OUT.json
then copy the JSON to tests/golden/ref_gpu_golden.json.
"""
from __future__ import annotations

import base64
import hashlib
import importlib.util
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def load_reference():
    import torch  # noqa: F401  (libc10/libtorch for the extension)

    so = ROOT / "oracle" / "_ref" / "_C.so"
    spec = importlib.util.spec_from_file_location("_C", so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def code_cases():
    """(name, rows, cols, bits, seed): random valid codes, scales U(0.002, 0.05)."""
    out = []
    for bits in (3, 4, 5, 7, 8, 9, 10, 11, 12, 15):
        out.append((f"codes_b{bits}_64x128", 64, 128, bits, 100 + bits))
    out += [("codes_b9_7x13", 7, 13, 9, 7), ("codes_b10_33x65", 33, 65, 10, 33),
            ("codes_b11_17x32", 17, 32, 11, 17)]
    return out


def case_codes(rows, cols, bits, seed):
    qm = (1 << (bits - 1)) - 1
    rng = np.random.default_rng(seed)
    q = rng.integers(-qm, qm + 1, size=(rows, cols), dtype=np.int16)
    s = rng.uniform(0.002, 0.05, size=rows).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32).astype(np.float16)
    return q, s, x


def matrix_cases():
    """(name, weights, calibration, threshold) for RuntimeMatrix.compress."""
    from oracle import oracle as O

    return [
        ("compress_baseline_256x384", O.baseline_weights(256, 384, seed=3),
         O.normal((32, 384), seed=4), 0.01),
        ("compress_normal_96x128", O.normal((96, 128), seed=5, scale=0.04),
         O.normal((12, 128), seed=6), 0.02),
    ]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(out_path: str) -> None:
    import torch

    ref = load_reference()
    res = {"generator": "reference RuntimeMatrix (mlbricks/elasticbit/csrc/elasticbit_runtime.cu)"
                        " built by oracle/build.py, run on " + torch.cuda.get_device_name(0),
           "codes": {}, "compress": {}}
    with tempfile.TemporaryDirectory() as tmp:
        for name, rows, cols, bits, seed in code_cases():
            q, s, x = case_codes(rows, cols, bits, seed)
            m = ref.RuntimeMatrix._compressSelectedCodes(q, s, bits, 0.01, 0.0, "fullPrecision")
            path = Path(tmp) / f"{name}.mlb"
            m.save(str(path))
            deq = np.asarray(m.dequantize(), dtype=np.float32)
            y = m.forwardTorch(torch.from_numpy(x).cuda()).cpu().numpy().astype(np.float16)
            res["codes"][name] = {
                "rows": rows, "cols": cols, "bits": bits, "seed": seed,
                "inputs_sha256": sha(q) + sha(s) + sha(x),
                "mlb4_b64": base64.b64encode(path.read_bytes()).decode(),
                "dequant_sha256": sha(deq),
                "forward_fp16_b64": base64.b64encode(y.tobytes()).decode(),
                "executionWidth": int(m.executionWidth),
            }
        for name, w, c, thr in matrix_cases():
            m = ref.RuntimeMatrix.compress(w, c, thr, "fullPrecision")
            res["compress"][name] = {"inputs_sha256": sha(w) + sha(c), "threshold": thr,
                                     "storageBits": int(m.storageBits),
                                     "error": repr(float(m.error)),
                                     "dequant_sha256": sha(np.asarray(m.dequantize(),
                                                                      dtype=np.float32))}
    Path(out_path).parent.mkdir(parents=True, exist_ok=True)
    Path(out_path).write_text(json.dumps(res, indent=1) + "\n")
    print("wrote", out_path, len(res["codes"]), "code cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_ref_gpu.py OUT.json")
    main(sys.argv[1])
