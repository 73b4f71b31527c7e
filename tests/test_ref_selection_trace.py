"""Model-path width selection pinned to the reference's own computation.

tests/golden/selection_trace_*.json hold the ATen operation sequence of the
reference's ``_selectBitsTorch`` (mlbricks/elasticbit/core.py:112-195),
recorded from the reference source by tests/golden/make_selection_trace.py.
Here that sequence is replayed on the GPU -- the reference's arithmetic, op for
op, on the same device as ours -- and the widths, errors, codes and scales it
selects are compared bit for bit with ``mlbricks_b200``'s ``_selectBitsTorch``
and with the matrices ``ElasticBit.compress`` builds, for BASELINE config 1
(nn.Linear 384 -> 1536, calibration (64, 128, 384) of which the first 32 rows
reach the analyzer) and a config-2 4096 x 4096 matrix, at thresholds 0.005,
0.01 and 0.02.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
THRESHOLDS = (0.005, 0.01, 0.02)


def _trace(rows: int, cols: int, samples: int) -> dict:
    return json.loads((GOLDEN / f"selection_trace_{rows}x{cols}_s{samples}.json").read_text())


def replay(trace: dict, weight: torch.Tensor, calibration: np.ndarray):
    """Run the recorded operations on the GPU.  Returns (errors per width 3..15 as
    (hardware, full) pairs, scales per width, codes per width)."""
    device = weight.device
    host_calib = torch.from_numpy(np.ascontiguousarray(calibration, dtype=np.float32))
    env = {trace["weight_tid"]: weight}

    def dec(a):
        if "t" in a:
            return env[a["t"]]
        if "in" in a:
            assert a["in"] == "calibration"
            return host_calib
        if "scalar_tensor" in a:
            return torch.tensor(float(a["scalar_tensor"]), dtype=getattr(torch, a["dtype"]))
        if "dtype" in a:
            return getattr(torch, a["dtype"])
        if "device" in a:
            return device if a["device"] == "cuda" else torch.device(a["device"])
        if "enum" in a:
            return getattr(torch, a["enum"])
        if "seq" in a:
            return [dec(x) for x in a["seq"]]
        if "f" in a:
            return float(a["f"])
        return a["v"]

    reads, scales, codes = [], [], []
    with torch.inference_mode():
        for op in trace["ops"]:
            _, name, overload = op["op"].split(".")
            fn = getattr(getattr(torch.ops.aten, name), overload)
            out = fn(*[dec(a) for a in op["args"]], **{k: dec(v) for k, v in op["kwargs"].items()})
            if op.get("scalar"):
                reads.append(float(out))
                continue
            outs = out if isinstance(out, (list, tuple)) else [out]
            for tid, o in zip(op["out"], outs):
                env[tid] = o
            if name == "where":
                scales.append(out)
            elif name == "clamp":
                codes.append(out)
    assert len(scales) == len(codes) == 13 and len(reads) == 6 * 2 + 7
    errors, i = [], 0
    for bits in range(3, 16):
        full = reads[i]
        i += 1
        hw = full
        if bits <= 8:
            hw = reads[i]
            i += 1
        errors.append((hw, full))
    return errors, scales, codes


def reference_selection(trace, weight, calibration, threshold):
    errors, scales, codes = replay(trace, weight, calibration)
    for bits, (hw, full) in zip(range(3, 16), errors):
        err = max(hw, full)
        if err <= threshold:
            return bits, err, codes[bits - 3].to(torch.int16), scales[bits - 3].float()
    return 16, 0.0, None, None


CASES = {
    "config1_1536x384": (1536, 384, lambda: O.baseline_weights(1536, 384, seed=0),
                         lambda: O.normal((64, 128, 384), seed=1).reshape(-1, 384)[:32]),
    "config2_4096x4096": (4096, 4096, lambda: O.baseline_weights(4096, 4096, seed=2),
                          lambda: O.normal((32, 4096), seed=3)),
}


@pytest.mark.parametrize("case", list(CASES))
def test_selection_matches_reference_trace(cuda_ok, case):
    from mlbricks_b200.elasticbit.core import _selectBitsTorch

    rows, cols, wfn, cfn = CASES[case]
    trace = _trace(rows, cols, 32)
    weight = torch.from_numpy(wfn()).cuda().half()
    calib = np.ascontiguousarray(cfn(), dtype=np.float32)
    picked = []
    for thr in THRESHOLDS:
        rb, rerr, rq, rs = reference_selection(trace, weight, calib, thr)
        ob, oerr, oq, os_ = _selectBitsTorch(weight, calib, thr)
        assert (ob, oerr) == (rb, rerr), (case, thr)
        if rb <= 15:
            assert torch.equal(oq, rq) and torch.equal(os_, rs), (case, thr)
        picked.append(rb)
    assert picked == sorted(picked, reverse=True)  # looser threshold, no wider codes


def test_compress_matches_reference_trace_config1(cuda_ok):
    """ElasticBit.compress on BASELINE config 1: the stored width and the exactly
    dequantised weight equal those of the reference's replayed selection."""
    from mlbricks_b200 import ElasticBit

    rows, cols, wfn, cfn = CASES["config1_1536x384"]
    w = wfn()
    calib_full = O.normal((64, 128, 384), seed=1)
    model = torch.nn.Sequential(torch.nn.Linear(cols, rows)).cuda().half().eval()
    with torch.no_grad():
        model[0].weight.copy_(torch.from_numpy(w))
        model[0].bias.zero_()
    weight16 = model[0].weight.detach().clone()
    rb, _, rq, rs = reference_selection(_trace(rows, cols, 32), weight16,
                                        calib_full.reshape(-1, cols)[:32], 0.01)
    ElasticBit.compress(model, torch.from_numpy(calib_full).cuda().half(), 0.01,
                        backend="native")
    m = model[0].matrix
    assert m.storageBits == rb
    expect = (rq.float() * rs[:, None]).half().float().cpu().numpy()
    assert np.array_equal(m.dequantize(), expect)
