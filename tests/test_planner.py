"""The `auto` route planner: parity gate, timing race, freezing (CPU tensors)."""
from __future__ import annotations

import pytest
import torch

from mlbricks_b200.planner import AUTO_OPERATOR_DEFAULTS, MLBricksExecutionPlanner


class Owner:
    pass


def test_elastic_linear_default_is_pytorch():
    assert AUTO_OPERATOR_DEFAULTS["elastic_linear"] == "pytorch"


def test_explicit_routes_are_strict():
    p = MLBricksExecutionPlanner()
    x = torch.zeros(2, 4)
    assert p.select_operator("elastic_linear", x, requested_backend="pytorch",
                             native_available=False) == "pytorch"
    with pytest.raises(RuntimeError, match="unavailable"):
        p.select_operator("elastic_linear", x, requested_backend="native", native_available=False)


def test_parity_failure_freezes_pytorch():
    p = MLBricksExecutionPlanner()
    x = torch.ones(2, 4, dtype=torch.float16)
    owner = Owner()
    route = p.qualify_operator_once(owner, "elastic_linear", x,
                                    {"native": lambda: x * 2, "pytorch": lambda: x},
                                    native_available=True, training=False)
    assert route == "pytorch"
    details = owner._mlbricks_frozen_auto_details[("elastic_linear", False)]
    assert details["reason"].startswith("correctness-gate:parity-failed")


def test_native_error_freezes_pytorch():
    p = MLBricksExecutionPlanner()
    x = torch.ones(2, 4)

    def boom():
        raise RuntimeError("kernel failed")

    owner = Owner()
    assert p.qualify_operator_once(owner, "elastic_linear", x, {"native": boom, "pytorch": lambda: x},
                                   native_available=True, training=False) == "pytorch"
    # frozen: later calls do not re-run candidates
    assert p.qualify_operator_once(owner, "elastic_linear", x, {}, native_available=True,
                                   training=False) == "pytorch"


def test_faster_native_wins_only_past_margin():
    import time

    p = MLBricksExecutionPlanner()
    x = torch.ones(4, 4)

    def slow():
        time.sleep(0.004)
        return x

    def fast():
        return x.clone()

    owner = Owner()
    assert p.qualify_operator_once(owner, "elastic_linear", x, {"native": fast, "pytorch": slow},
                                   native_available=True, training=False) == "native"
    owner2 = Owner()
    assert p.qualify_operator_once(owner2, "elastic_linear", x, {"native": slow, "pytorch": slow},
                                   native_available=True, training=False, switch_margin=10.0) == "pytorch"


def test_training_never_selects_inference_only_native():
    p = MLBricksExecutionPlanner()
    x = torch.ones(2)
    assert p.qualify_operator_once(Owner(), "elastic_linear", x, {"native": lambda: x},
                                   native_available=True, training=True) == "pytorch"
