"""Public API contract, mirroring the reference's tests/test_elasticbit.py
(CPU-safe: no kernels run)."""
from __future__ import annotations

import inspect

import pytest
import torch.nn as nn

import mlbricks_b200 as mlb
from mlbricks_b200 import BackendInfo, ElasticBit, RuntimeMatrix
from mlbricks_b200.elasticbit.core import _semanticOutputWeightIds
from mlbricks_b200.runtime import normalize_backend


def test_clean_public_surface_has_no_fixed_bit_api():
    for name in ("bits", "quantize", "dequantize", "quantize_module", "apply"):
        assert not hasattr(ElasticBit, name)
    assert not hasattr(RuntimeMatrix, "from_auto")
    assert set(mlb.__all__) == {"ElasticBit", "RuntimeMatrix", "BitAnalysis", "BitCandidate",
                                "BackendInfo"}


def test_public_api_uses_camel_case_names():
    sig = inspect.signature(ElasticBit.compressMatrix)
    assert "calibrationData" in sig.parameters and "decodePolicy" in sig.parameters
    assert sig.parameters["decodePolicy"].default == "hardwareNative"
    assert inspect.signature(ElasticBit.loadMatrix).parameters["decodePolicy"].default == "hardwareNative"
    assert inspect.signature(RuntimeMatrix.compress).parameters["decodePolicy"].default == "hardwareNative"
    assert inspect.signature(RuntimeMatrix.load).parameters["decodePolicy"].default == "hardwareNative"
    assert "calibration_data" not in sig.parameters and "decode_policy" not in sig.parameters
    comp = inspect.signature(ElasticBit.compress).parameters
    assert list(comp)[:5] == ["model", "calibrationData", "threshold", "decodePolicy",
                              "preserveOutputHead"]
    assert comp["preserveOutputHead"].default is True
    assert comp["backend"].default == "auto"  # additive keyword
    assert hasattr(RuntimeMatrix, "setDecodePolicy")


def test_backend_api_is_safe_without_native_extension():
    info = ElasticBit.backend()
    assert isinstance(info, BackendInfo)
    assert isinstance(info.available, bool) and isinstance(info.validated, bool)
    if info.available:
        assert info.prefill == "native"
        assert info.decodePlanner in {"t4Validated", "cudaAutoTune"}
        assert info.decodeEngine == "FastWarp"
        assert info.decodeStatus == "experimental"
        assert info.decodeValidation == "unvalidated"
    else:
        assert "unavailable" in str(info)


def test_native_only_calls_fail_cleanly_when_extension_missing():
    if ElasticBit.backend().available:
        pytest.skip("native ElasticBit runtime is available here")
    with pytest.raises(RuntimeError, match="CUDA runtime"):
        ElasticBit.analyze([[1.0, 2.0]], [[1.0, 1.0]], 0.01)
    with pytest.raises(RuntimeError, match="CUDA runtime"):
        ElasticBit.compress(nn.Linear(2, 2), [[1.0, 1.0]], 0.01)


def test_runtime_matrix_has_only_threshold_driven_factories():
    assert callable(RuntimeMatrix.compress) and callable(RuntimeMatrix.load)
    assert not hasattr(RuntimeMatrix, "auto")


def test_semantic_output_head_detection_is_model_agnostic():
    class ToyDecoder(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed = nn.Embedding(31, 8)
            self.block = nn.Linear(8, 8, bias=False)
            self.vocab_projection = nn.Linear(8, 31, bias=False)

        def get_output_embeddings(self):
            return self.vocab_projection

    model = ToyDecoder()
    protected = _semanticOutputWeightIds(model)
    assert protected == {id(model.vocab_projection.weight)}
    assert id(model.block.weight) not in protected


def test_semantic_output_head_detection_never_depends_on_module_name():
    class OddNames(nn.Module):
        def __init__(self):
            super().__init__()
            self.not_a_head = nn.Linear(4, 7, bias=False)

        def get_output_embeddings(self):
            return self.not_a_head

    model = OddNames()
    assert _semanticOutputWeightIds(model) == {id(model.not_a_head.weight)}


def test_backend_names_and_legacy_aliases():
    assert normalize_backend(None) == "auto"
    assert normalize_backend("Native") == "native"
    assert normalize_backend("cuda") == "native"
    assert normalize_backend("torch") == "pytorch"
    with pytest.raises(ValueError):
        normalize_backend("triton")


def test_decode_policy_validation_is_host_side():
    from mlbricks_b200.elasticbit.core import _checkPolicy

    assert _checkPolicy("fullPrecision") == "fullPrecision"
    with pytest.raises(ValueError, match="decodePolicy"):
        _checkPolicy("int4")
