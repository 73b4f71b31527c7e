"""Parity against outputs of the reference's own RuntimeMatrix, run on a B200
(tests/golden/ref_gpu_golden.json, made by tests/golden/make_golden_ref_gpu.py):
MLB4 file bytes, dequantised weights, the FastWarp fp16 forward (M = 1,
fullPrecision) and the matrix-path compress result; and a `.elasticbit` model
artifact holding a reference-written MLB4 file, read by ElasticBit.load."""
from __future__ import annotations

import base64
import hashlib
import io
import json
import zipfile
from pathlib import Path

import numpy as np
import pytest

import make_golden_ref_gpu as G
from oracle import oracle as O

GOLD = json.loads((Path(__file__).parent / "golden" / "ref_gpu_golden.json").read_text())
CODE_CASES = {name: (rows, cols, bits, seed) for name, rows, cols, bits, seed in G.code_cases()}


def _sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _inputs(name):
    rows, cols, bits, seed = CODE_CASES[name]
    q, s, x = G.case_codes(rows, cols, bits, seed)
    assert _sha(q) + _sha(s) + _sha(x) == GOLD["codes"][name]["inputs_sha256"]
    return rows, cols, bits, q, s, x


def _fp16_close(y, ref16):
    """|y - ref| <= max(2e-3, one fp16 ulp of the reference value)."""
    r = ref16.astype(np.float32)
    ulp = np.spacing(np.abs(ref16)).astype(np.float32)
    return np.all(np.abs(y.astype(np.float32) - r) <= np.maximum(2e-3, ulp))


@pytest.mark.parametrize("name", list(GOLD["codes"]))
def test_oracle_writes_reference_mlb4_bytes(name):
    rows, cols, bits, q, s, x = _inputs(name)
    ref = base64.b64decode(GOLD["codes"][name]["mlb4_b64"])
    mine = O.mlb4_bytes(rows, cols, bits, s, O.pack_codes(q, bits), 0.01, 0.0)
    assert mine == ref
    parsed = O.mlb4_parse(ref)
    assert np.array_equal(O.unpack_codes(parsed["payload"], rows, cols, bits), q)


@pytest.mark.parametrize("name", list(GOLD["codes"]))
def test_oracle_dequant_and_forward_match_reference(name):
    rows, cols, bits, q, s, x = _inputs(name)
    w16 = O.dequantize_codes(q, s).astype(np.float32)
    assert _sha(w16) == GOLD["codes"][name]["dequant_sha256"]
    ref_y = np.frombuffer(base64.b64decode(GOLD["codes"][name]["forward_fp16_b64"]), np.float16)
    oracle_y = O.linear_full(x[None, :], w16)[0]
    assert _fp16_close(oracle_y, ref_y)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(GOLD["codes"]))
def test_libebx_matches_reference_runtime_matrix(cuda_ok, name, tmp_path):
    import torch

    from mlbricks_b200 import RuntimeMatrix

    rows, cols, bits, q, s, x = _inputs(name)
    m = RuntimeMatrix._compressSelectedCodes(q, s, bits, 0.01, 0.0, decodePolicy="fullPrecision")
    path = tmp_path / "m.mlb"
    m.save(path)
    assert path.read_bytes() == base64.b64decode(GOLD["codes"][name]["mlb4_b64"])
    assert _sha(m.dequantize()) == GOLD["codes"][name]["dequant_sha256"]
    y = m.forward(torch.from_numpy(x).cuda()).cpu().numpy()
    ref_y = np.frombuffer(base64.b64decode(GOLD["codes"][name]["forward_fp16_b64"]), np.float16)
    assert _fp16_close(y, ref_y)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(GOLD["compress"]))
def test_libebx_compress_matches_reference(cuda_ok, name):
    from mlbricks_b200 import RuntimeMatrix

    cases = {n: (w, c, t) for n, w, c, t in G.matrix_cases()}
    w, c, thr = cases[name]
    gold = GOLD["compress"][name]
    assert _sha(w) + _sha(c) == gold["inputs_sha256"]
    m = RuntimeMatrix.compress(w, c, thr, decodePolicy="fullPrecision")
    assert m.storageBits == gold["storageBits"]
    assert abs(m.error - float(gold["error"])) <= 1e-12 * float(gold["error"])
    assert _sha(m.dequantize()) == gold["dequant_sha256"]


def _reference_artifact(path, mlb4, rows, cols, policy):
    """A model artifact laid out as the reference's ElasticBit.save writes it
    (mlbricks/elasticbit/core.py:900-953): manifest.json with the reference's keys
    in its order, state.pt (the compressed model's state_dict: empty for a Linear
    without bias) and matrices/matrix_00000.mlb (here the reference's own bytes)."""
    import torch

    manifest = {
        "format": "ElasticBitModel", "version": 1, "threshold": 0.01, "decodePolicy": policy,
        "compressedNames": ["0"], "skippedNames": [], "optimizationProfiles": {},
        "layers": [{"name": "0", "matrix": "matrix_00000.mlb", "inFeatures": cols,
                    "outFeatures": rows, "hasBias": False}],
    }
    state = io.BytesIO()
    torch.save({}, state)
    with zipfile.ZipFile(path, "w", compression=zipfile.ZIP_DEFLATED) as zf:
        zf.writestr("manifest.json", json.dumps(manifest, indent=2))
        zf.writestr("matrices/matrix_00000.mlb", base64.b64decode(GOLD["codes"][mlb4]["mlb4_b64"]))
        zf.writestr("state.pt", state.getvalue())
    return path


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["codes_b10_33x65", "codes_b4_64x128", "codes_b9_7x13"])
def test_load_model_artifact_with_reference_matrix(cuda_ok, name, tmp_path):
    import torch

    from mlbricks_b200 import ElasticBit

    rows, cols, bits, q, s, x = _inputs(name)
    path = _reference_artifact(tmp_path / "ref.elasticbit", name, rows, cols, "fullPrecision")
    shell = torch.nn.Sequential(torch.nn.Linear(cols, rows, bias=False)).cuda().half().eval()
    ElasticBit.load(shell, path, decodePolicy="fullPrecision", backend="native")
    m = shell[0].matrix
    assert m.storageBits == bits and m.shape == (rows, cols)
    assert _sha(m.dequantize()) == GOLD["codes"][name]["dequant_sha256"]
    y = shell(torch.from_numpy(x).cuda()[None]).detach().cpu().numpy()[0]
    ref_y = np.frombuffer(base64.b64decode(GOLD["codes"][name]["forward_fp16_b64"]), np.float16)
    assert _fp16_close(y, ref_y)
    # saving the loaded model writes the reference's matrix bytes back unchanged
    out = ElasticBit.save(shell, tmp_path / "again.elasticbit")
    with zipfile.ZipFile(out) as zf:
        assert zf.read("matrices/matrix_00000.mlb") == base64.b64decode(GOLD["codes"][name]["mlb4_b64"])
