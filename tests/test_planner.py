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


def test_auto_freeze_is_per_row_regime():
    """A race lost by native on a prefill-sized call does not route decode calls."""
    import time

    from mlbricks_b200.elasticbit.core import _row_regime

    assert [_row_regime(m) for m in (1, 16, 17, 256, 257, 4096)] == [
        "decode", "decode", "small-batch", "small-batch", "prefill", "prefill"]
    p = MLBricksExecutionPlanner()
    owner = Owner()

    def slow_native():
        time.sleep(0.004)
        return x_big.clone()

    x_big = torch.ones(4096, 8)
    x_one = torch.ones(1, 8)
    calls = {"native": 0}

    def fast_native():
        calls["native"] += 1
        return x_one.clone()

    def slow_pytorch():
        time.sleep(0.004)
        return x_one

    r_prefill = p.qualify_operator_once(owner, "elastic_linear", x_big,
                                        {"native": slow_native, "pytorch": lambda: x_big},
                                        native_available=True, training=False,
                                        freeze_on=(_row_regime(4096),))
    assert r_prefill == "pytorch"
    r_decode = p.qualify_operator_once(owner, "elastic_linear", x_one,
                                       {"native": fast_native, "pytorch": slow_pytorch},
                                       native_available=True, training=False,
                                       freeze_on=(_row_regime(1),))
    assert r_decode == "native" and calls["native"] > 0
    routes = owner._mlbricks_frozen_auto_routes
    assert routes[("elastic_linear", False, "prefill")] == "pytorch"
    assert routes[("elastic_linear", False, "decode")] == "native"
    # both frozen: later calls of each regime keep their own route without racing
    assert p.qualify_operator_once(owner, "elastic_linear", x_big, {}, native_available=True,
                                   training=False, freeze_on=("prefill",)) == "pytorch"
    assert p.qualify_operator_once(owner, "elastic_linear", x_one, {}, native_available=True,
                                   training=False, freeze_on=("decode",)) == "native"
