"""Public API on the GPU: the reference's native-test contracts
(tests/test_elasticbit_native.py in MLBricks) plus route parity."""
from __future__ import annotations

import io
import json
import zipfile

import numpy as np
import pytest
import torch

from mlbricks_b200 import ElasticBit, RuntimeMatrix
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rel(actual, reference):
    a = np.asarray(actual, dtype=np.float32)
    r = np.asarray(reference, dtype=np.float32)
    return float(np.linalg.norm(a - r) / max(np.linalg.norm(r), 1e-12))


def test_backend_reports_available(cuda_ok):
    info = ElasticBit.backend()
    assert info.available and info.architecture.startswith("sm")
    assert info.prefill == "native" and info.decodePlanner == "cudaAutoTune"


def test_threshold_contract_and_policy_switch(cuda_ok, tmp_path):
    rng = np.random.default_rng(20260918)
    weights = rng.normal(0, 0.04, size=(96, 128)).astype(np.float32)
    calib = rng.normal(0, 1, size=(12, 128)).astype(np.float32)
    threshold = 0.02
    analysis = ElasticBit.analyze(weights, calib, threshold)
    assert 3 <= analysis.selectedBits <= 16
    assert analysis.selectedError <= threshold + 1e-12
    assert analysis == ElasticBit.analyze(weights, calib, threshold)  # deterministic

    matrix = ElasticBit.compressMatrix(weights, calib, threshold)
    assert matrix.storageBits == analysis.selectedBits
    assert matrix.activateDType == "float16"
    assert matrix.executionPlanner == "cudaAutoTune"
    b = matrix.storageBits
    legal = {4, 8, 16} if b <= 4 else {8, 16} if b <= 8 else {12, 16} if b <= 12 else {16}
    assert matrix.executionWidth in legal

    x = calib[0]
    hardware = np.asarray(matrix.forward(x))
    matrix.setDecodePolicy("fullPrecision")
    assert matrix.executionWidth == 16 and matrix.executionPlanner == "fullPrecision"
    full = np.asarray(matrix.forward(x))
    assert _rel(hardware, full) <= 2.0 * threshold + 1e-3

    # bit-exact storage: codes and dequantised weights equal the oracle's
    s = O.row_scales(weights, matrix.storageBits)
    q = O.quantize(weights, s, matrix.storageBits)
    assert np.array_equal(matrix.dequantize(), O.dequantize_codes(q, s).astype(np.float32))

    path = tmp_path / "matrix.mlb"
    matrix.setDecodePolicy("hardwareNative")
    matrix.save(path)
    blob = path.read_bytes()
    parsed = O.mlb4_parse(blob)  # the oracle reader accepts our file
    assert np.array_equal(O.unpack_codes(parsed["payload"], 96, 128, matrix.storageBits), q)
    assert blob == O.mlb4_bytes(96, 128, matrix.storageBits, s, O.pack_codes(q, matrix.storageBits),
                                threshold, matrix.error)
    loaded = ElasticBit.loadMatrix(path, decodePolicy="hardwareNative")
    assert loaded.storageBits == matrix.storageBits
    loaded_out = np.asarray(loaded.forward(x))
    if loaded.executionWidth == matrix.executionWidth:
        np.testing.assert_array_equal(loaded_out, hardware)
    assert _rel(loaded_out, hardware) <= 2.0 * threshold + 1e-3


def test_model_compress_switch_and_artifact(cuda_ok, tmp_path):
    torch.manual_seed(20260918)

    def make():
        return torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.GELU(),
                                   torch.nn.Linear(96, 32)).cuda().half().eval()

    model = make()
    calib = [torch.randn(4, 64, device="cuda", dtype=torch.float16) for _ in range(2)]
    ElasticBit.compress(model, calib, 0.03)
    prefill = model(torch.randn(4, 64, device="cuda", dtype=torch.float16))
    assert prefill.shape == (4, 32) and torch.isfinite(prefill).all()

    x = torch.randn(1, 64, device="cuda", dtype=torch.float16)
    model.elasticbit.setDecodePolicy("hardwareNative")
    hardware = model(x).detach()
    model.elasticbit.setDecodePolicy("fullPrecision")
    full = model(x).detach()
    assert torch.nn.functional.cosine_similarity(hardware.float(), full.float(), dim=-1).item() > 0.999

    artifact = tmp_path / "model.elasticbit"
    ElasticBit.save(model, artifact)
    shell = make()
    ElasticBit.load(shell, artifact, decodePolicy="fullPrecision")
    restored = shell(x).detach()
    torch.testing.assert_close(restored, full, atol=0, rtol=0)


# the reference writer's manifest and layer-entry keys, in its order
# (mlbricks/elasticbit/core.py:928-947)
REF_MANIFEST_KEYS = ["format", "version", "threshold", "decodePolicy", "compressedNames",
                     "skippedNames", "optimizationProfiles", "layers"]
REF_LAYER_KEYS = ["name", "matrix", "inFeatures", "outFeatures", "hasBias"]


def test_model_artifact_layout_follows_reference_writer(cuda_ok, tmp_path):
    torch.manual_seed(11)
    model = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.GELU(),
                                torch.nn.Linear(96, 40, bias=False)).cuda().half().eval()
    ElasticBit.compress(model, [torch.randn(4, 64, device="cuda", dtype=torch.float16)], 0.03)
    path = ElasticBit.save(model, tmp_path / "m.elasticbit")
    with zipfile.ZipFile(path) as zf:
        names = sorted(zf.namelist())
        assert names == ["manifest.json", "matrices/matrix_00000.mlb", "matrices/matrix_00001.mlb",
                         "state.pt"]
        manifest = json.loads(zf.read("manifest.json"))
        blobs = {n: zf.read(n) for n in names if n.endswith(".mlb")}
        state = torch.load(io.BytesIO(zf.read("state.pt")), weights_only=True)
    assert list(manifest) == REF_MANIFEST_KEYS
    assert (manifest["format"], manifest["version"]) == ("ElasticBitModel", 1)
    assert manifest["threshold"] == 0.03 and manifest["decodePolicy"] == "hardwareNative"
    assert manifest["compressedNames"] == ["0", "2"] and manifest["skippedNames"] == []
    for i, entry in enumerate(manifest["layers"]):
        assert list(entry) == REF_LAYER_KEYS
        layer = model[int(entry["name"])]
        m = layer.matrix
        assert entry["matrix"] == f"matrix_{i:05d}.mlb"
        assert (entry["inFeatures"], entry["outFeatures"], entry["hasBias"]) == \
            (layer.inFeatures, layer.outFeatures, layer.bias is not None)
        parsed = O.mlb4_parse(blobs["matrices/" + entry["matrix"]])
        assert (parsed["rows"], parsed["cols"], parsed["bits"]) == (m.rows, m.cols, m.storageBits)
        assert parsed["threshold"] == 0.03 and parsed["selectedError"] == m.error
        if m.storageBits == 16:
            w = parsed["payload"].view(np.float16).reshape(m.rows, m.cols).astype(np.float32)
        else:
            codes = O.unpack_codes(parsed["payload"], m.rows, m.cols, m.storageBits)
            w = O.dequantize_codes(codes, parsed["scales"]).astype(np.float32)
        assert np.array_equal(w, m.dequantize())
    assert set(state) == set(model.state_dict()) == {"0.bias"}
    torch.testing.assert_close(state["0.bias"], model[0].bias, atol=0, rtol=0)


def test_model_analyzer_result_reuse_and_policy(cuda_ok, tmp_path):
    torch.manual_seed(20260918)
    model = torch.nn.Sequential(torch.nn.Linear(128, 128, bias=False)).cuda().half().eval()
    ElasticBit.compress(model, [torch.randn(8, 128, device="cuda", dtype=torch.float16)],
                        threshold=0.03)
    matrix = model[0].matrix
    assert matrix.activateDType == "float16" and 3 <= matrix.storageBits <= 16
    x = torch.randn(1, 128, device="cuda", dtype=torch.float16)
    model.elasticbit.setDecodePolicy("fullPrecision")
    a = model(x).detach()
    model.elasticbit.setDecodePolicy("hardwareNative")
    b = model(x).detach()
    assert torch.nn.functional.cosine_similarity(a.float(), b.float(), dim=-1).item() > 0.999
    ElasticBit.save(model, tmp_path / "fastwarp.elasticbit")
    assert (tmp_path / "fastwarp.elasticbit").exists()


@pytest.mark.parametrize("storage_bits", [3, 4, 5, 7, 8, 9, 15])
@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 13), (8, 31), (17, 32), (33, 65)])
def test_model_agnostic_shape_contract(cuda_ok, storage_bits, rows, cols):
    qm = (1 << (storage_bits - 1)) - 1
    rng = np.random.default_rng(rows * 1000 + cols * 10 + storage_bits)
    codes = rng.integers(-max(qm, 1), max(qm, 1) + 1, size=(rows, cols), dtype=np.int16)
    scales = rng.uniform(0.002, 0.05, size=(rows,)).astype(np.float32)
    matrix = RuntimeMatrix._compressSelectedCodes(codes, scales, storage_bits, threshold=0.01,
                                                  selectedError=0.0, decodePolicy="hardwareNative")
    x = torch.randn(1, cols, device="cuda", dtype=torch.float16)
    y = matrix.forward(x)
    weight = matrix._materializeTorch()
    assert torch.equal(weight.cpu(), torch.from_numpy(O.dequantize_codes(codes, scales)))
    reference = torch.nn.functional.linear(x, weight)
    assert y.shape == (1, rows) and torch.isfinite(y).all()
    assert torch.nn.functional.cosine_similarity(y.float(), reference.float(), dim=-1).item() > 0.999


def test_select_bits_matches_oracle_restatement(cuda_ok):
    from mlbricks_b200.elasticbit.core import _selectBitsTorch

    w = torch.from_numpy(O.baseline_weights(384, 256, seed=4)).half().cuda()
    c = O.normal((32, 256), seed=5)
    for thr in (0.005, 0.01, 0.02):
        bits, err, codes, scales = _selectBitsTorch(w, c, thr)
        obits, oerr, ocodes, oscales = O.select_bits_torch(w, c, thr)
        assert bits == obits and err == oerr
        assert np.array_equal(codes.cpu().numpy(), ocodes)
        assert np.array_equal(scales.cpu().numpy(), oscales)


def test_config1_backends_agree(cuda_ok):
    """Linear 384->1536, zero bias, calibration (64,128,384),
    threshold 0.01, x (2,128,384); backend='pytorch' vs 'native'."""
    torch.manual_seed(0)
    w = torch.from_numpy(O.baseline_weights(1536, 384, seed=0))

    def make():
        lin = torch.nn.Linear(384, 1536)
        with torch.no_grad():
            lin.weight.copy_(w)
            lin.bias.zero_()
        # compress replaces child modules, never the root (core.py:206-213)
        return torch.nn.Sequential(lin).cuda().half().eval()

    calib = torch.from_numpy(O.normal((64, 128, 384), seed=1)).cuda().half()
    x = torch.from_numpy(O.normal((2, 128, 384), seed=2)).cuda().half()
    # the model path's selection restated by the oracle, on the FP16 weight and the first
    # 32 calibration rows compress captures (core.py:734)
    obits, _, oq, os_ = O.select_bits_torch(make()[0].weight.detach(),
                                            calib[0, :32].float().cpu().numpy(), 0.01)
    ref_model = ElasticBit.compress(make(), calib, 0.01, backend="pytorch")
    nat_model = ElasticBit.compress(make(), calib, 0.01, backend="native")
    assert ref_model[0].matrix.storageBits == nat_model[0].matrix.storageBits == obits
    assert np.array_equal(nat_model[0].matrix.dequantize(),
                          O.dequantize_codes(oq, os_).astype(np.float32))
    y_ref = ref_model(x).float().cpu().numpy()
    y_nat = nat_model(x).float().cpu().numpy()
    # north_star bar: relative L2 <= 1e-3, max-abs <= 2e-3 (or one fp16 ulp of
    # the value where that is larger: both routes round an fp32 sum to fp16)
    rel = np.linalg.norm(y_nat - y_ref) / np.linalg.norm(y_ref)
    assert rel <= 1e-3
    ulp = np.spacing(np.abs(y_ref.astype(np.float16))).astype(np.float32)
    assert np.all(np.abs(y_nat - y_ref) <= np.maximum(2e-3, ulp))


def test_auto_route_decides_per_row_regime(cuda_ok):
    """`auto` races once per row regime: a prefill-sized call whose native
    candidate is made slow freezes `pytorch` for prefill only, and the first
    decode call still races and goes native (the per-call materialise of the
    pytorch route is far slower for one token)."""
    import time

    from mlbricks_b200.elasticbit.core import _ElasticLinear

    rows, cols = 1024, 2048
    w = O.baseline_weights(rows, cols, seed=41)
    model = torch.nn.Sequential(torch.nn.Linear(cols, rows, bias=False)).cuda().half().eval()
    with torch.no_grad():
        model[0].weight.copy_(torch.from_numpy(w))
    calib = torch.from_numpy(O.normal((32, cols), seed=42)).cuda().half()
    ElasticBit.compress(model, calib, 0.01, backend="auto")
    layer = model[0]
    assert isinstance(layer, _ElasticLinear)
    native = layer._forward_native

    def slow_for_prefill(x):
        if x.numel() // cols > 256:
            torch.cuda.synchronize()
            time.sleep(0.05)
        return native(x)

    layer._forward_native = slow_for_prefill
    with torch.no_grad():
        model(torch.from_numpy(O.normal((1024, cols), seed=43)).cuda().half())
        model(torch.from_numpy(O.normal((1, cols), seed=44)).cuda().half())
    routes = layer._mlbricks_frozen_auto_routes
    assert routes[("elastic_linear", False, "prefill")] == "pytorch"
    assert routes[("elastic_linear", False, "decode")] == "native"
