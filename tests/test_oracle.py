"""CPU oracle pinned to the reference's own outputs (tests/golden) and to
the reference's storage rules (elasticbit_runtime.cu:64-238, 682-871)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
import make_golden as G

GOLDEN = json.loads((Path(__file__).parent / "golden" / "analyze_golden.json").read_text())


@pytest.mark.parametrize("name", G.CASES)
def test_oracle_analyzer_matches_reference_golden(name):
    case = GOLDEN["cases"][name]
    w, c, thr = G.case_inputs(name)
    assert G.sha(w, c) == case["inputs_sha256"], "numpy RNG stream changed; regenerate goldens"
    res = O.analyze(w, c, thr)
    assert res["selectedBits"] == case["selectedBits"]
    assert res["selectedError"] == float(case["selectedError"])
    for mine, ref in zip(res["candidates"], case["candidates"]):
        assert mine["bits"] == ref["bits"]
        # Same float order + long double norms: bit-identical to the reference.
        for key in ("hardwareNativeError", "fullPrecisionError", "error", "memoryReduction"):
            assert mine[key] == float(ref[key]), (key, mine["bits"])
        assert mine["storageBytes"] == ref["storageBytes"]
        assert mine["passes"] == ref["passes"]


def test_baseline_config1_widths_follow_threshold():
    bits = [GOLDEN["cases"][f"config1_{t}"]["selectedBits"] for t in ("0.005", "0.01", "0.02")]
    assert bits == [10, 9, 8]


@pytest.mark.parametrize("bits", list(range(3, 16)))
@pytest.mark.parametrize("shape", [(1, 1), (7, 13), (8, 31), (17, 32), (33, 65)])
def test_pack_unpack_roundtrip_and_dequant(bits, shape):
    rows, cols = shape
    qm = O.qmax(bits)
    rng = np.random.default_rng(rows * 1000 + cols * 10 + bits)
    q = rng.integers(-qm, qm + 1, size=shape, dtype=np.int16)
    s = rng.uniform(0.002, 0.05, size=rows).astype(np.float32)
    payload = O.pack_codes(q, bits)
    assert payload.size == (rows * cols * bits + 7) // 8
    assert np.array_equal(O.unpack_codes(payload, rows, cols, bits), q)
    # codes are stored biased by qmax (cu:171)
    assert O.lib().ebo_extract_code(payload.ctypes.data, payload.size, 0, bits) == q.flat[0] + qm
    deq = O.dequantize_fp16(payload, s, rows, cols, bits)
    assert np.array_equal(deq.view(np.uint16), O.dequantize_codes(q, s).view(np.uint16))


def test_pack_rejects_out_of_range_codes():
    q = np.array([[0, 4]], dtype=np.int16)
    with pytest.raises(ValueError, match="exceeds selected bit range"):
        O.pack_codes(q, 3)  # qmax(3) = 3


def test_quantize_matches_reference_rules():
    w = np.array([[0.0, 0.0, 0.0, 0.0], [1.0, -0.5, 0.3, 0.1], [2.5, 1.5, -2.5, 7.0]],
                 dtype=np.float32)
    s = O.row_scales(w, 4)
    assert s[0] == 1.0  # all-zero row -> scale 1 (cu:98)
    assert s[1] == np.float32(1.0) / np.float32(7.0)
    assert s[2] == 1.0
    q = O.quantize(w, s, 4)
    assert q[2].tolist() == [2, 2, -2, 7]  # exact ties round half to even (nearbyint)
    for r in range(3):
        for c in range(4):
            assert q[r, c] == O.lib().ebo_quantize_scalar(float(w[r, c]), float(s[r]), 4)


def test_fp16_fallback_packs_raw_halves():
    w = O.normal((3, 5), seed=3, scale=0.1)
    payload = O.pack_weights(w, 16)
    assert np.array_equal(payload.view(np.float16).reshape(3, 5), w.astype(np.float16))
    assert np.array_equal(O.dequantize(payload, None, 3, 5, 16), w.astype(np.float16).astype(np.float32))


def test_mlb4_roundtrip_and_corruption():
    w = O.baseline_weights(16, 24, seed=5)
    s = O.row_scales(w, 9)
    q = O.quantize(w, s, 9)
    blob = O.mlb4_bytes(16, 24, 9, s, O.pack_codes(q, 9), 0.01, 0.004)
    assert len(blob) == 80 + 16 * 4 + (16 * 24 * 9 + 7) // 8
    m = O.mlb4_parse(blob)
    assert m["bits"] == 9 and np.array_equal(m["scales"], s)
    assert np.array_equal(O.unpack_codes(m["payload"], 16, 24, 9), q)
    bad = bytearray(blob)
    bad[-1] ^= 0x40
    with pytest.raises(ValueError, match="checksum"):
        O.mlb4_parse(bytes(bad))
    with pytest.raises(ValueError, match="metadata"):
        O.mlb4_parse(blob[:-1])
    with pytest.raises(ValueError, match="invalid ElasticBit MLB4 file"):
        O.mlb4_parse(b"MLB3" + blob[4:])


def test_fnv1a64_matches_reference_variant():
    # The reference's MLB4 checksum (cu:682-690) starts from 1469598103934665603,
    # i.e. the published FNV-1a 64 offset basis 14695981039346656037 with its
    # last digit dropped.  Byte-compatible files need that exact variant.
    def fnv(data: bytes) -> int:
        h = 1469598103934665603
        for b in data:
            h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        return h

    assert O.fnv1a64(b"") == 1469598103934665603
    for data in (b"a", b"foobar", bytes(range(256)) * 3):
        assert O.fnv1a64(data) == fnv(data)


def test_linear_semantics_full_vs_hw():
    w = O.baseline_weights(32, 64, seed=9)
    s = O.row_scales(w, 8)
    q = O.quantize(w, s, 8)
    x = O.normal((3, 64), seed=10).astype(np.float16)
    full = O.linear_full(x, O.dequantize_codes(q, s).astype(np.float32))
    hw = O.linear_hw(x, q, s)
    rel = np.linalg.norm(full - hw) / np.linalg.norm(full)
    assert 0 < rel < 2e-3  # per-weight fp16 rounding is the only difference


def test_select_bits_torch_restatement_runs_on_cpu():
    import torch

    w = torch.from_numpy(O.baseline_weights(64, 128, seed=2)).half()
    c = O.normal((32, 128), seed=3)
    bits, err, codes, scales = O.select_bits_torch(w, c, 0.01)
    assert 3 <= bits <= 16 and err <= 0.01
    if bits <= 15:
        assert np.abs(codes).max() <= O.qmax(bits)


def test_reference_selection_trace_replays_on_host():
    """The recorded reference selection (tests/golden/selection_trace_*.json) replays
    on the host and agrees with the oracle's restatement run there: BASELINE
    config 1 selects 10 / 9 / 8 bits at thresholds 0.005 / 0.01 / 0.02."""
    import torch

    from tests.test_ref_selection_trace import CASES, THRESHOLDS, _trace, reference_selection

    rows, cols, wfn, cfn = CASES["config1_1536x384"]
    trace = _trace(rows, cols, 32)
    w = torch.from_numpy(wfn()).half()
    calib = cfn()
    picked = []
    for thr in THRESHOLDS:
        rb, rerr, rq, rs = reference_selection(trace, w, calib, thr)
        ob, oerr, oq, os_ = O.select_bits_torch(w, calib, thr)
        assert (rb, rerr) == (ob, oerr)
        assert np.array_equal(rq.numpy(), oq) and np.array_equal(rs.numpy(), os_)
        picked.append(rb)
    assert picked == [10, 9, 8]
