"""libebx kernels vs the CPU oracle, called through the C ABI (include/ebx.h).

Bars: codes, packed payloads, scales and dequantised fp16 weights bit-exact;
linear outputs within max-abs 2e-3 and relative-L2 1e-3 of the float64
oracle on the fp32 output (y32), and the fp16 output within one fp16 ulp of
the correctly rounded oracle value.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from mlbricks_b200 import _ebx
from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
REL_L2 = 1e-3
ODD_SHAPES = [(1, 1), (7, 13), (8, 31), (17, 32), (33, 65), (16, 64), (48, 200)]


@pytest.fixture(scope="module")
def lib(cuda_ok):
    return _ebx.load()


def dev():
    return torch.device("cuda", 0)


def stream():
    return _ebx.stream_ptr()


class Handle:
    def __init__(self, ptr: int):
        self.h = ctypes.c_void_p(ptr)

    def __del__(self):
        if self.h.value:
            _ebx.load().ebx_matrix_destroy(self.h)


def from_codes(lib, q: np.ndarray, s: np.ndarray, bits: int) -> Handle:
    qd = torch.from_numpy(np.ascontiguousarray(q, dtype=np.int16)).to(dev())
    sd = torch.from_numpy(np.ascontiguousarray(s, dtype=np.float32)).to(dev())
    h = ctypes.c_void_p()
    _ebx.check(lib.ebx_matrix_create_from_codes(qd.data_ptr(), sd.data_ptr(), q.shape[0],
                                                q.shape[1], bits, 0, stream(), ctypes.byref(h)))
    return Handle(h.value)


def random_codes(rows, cols, bits, seed):
    qm = O.qmax(bits)
    rng = np.random.default_rng(seed)
    q = rng.integers(-qm, qm + 1, size=(rows, cols), dtype=np.int16)
    s = rng.uniform(0.002, 0.05, size=rows).astype(np.float32)
    return q, s


def export_payload(lib, h: Handle, nbytes: int) -> np.ndarray:
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev())
    _ebx.check(lib.ebx_matrix_export_payload(h.h, buf.data_ptr(), nbytes, stream()))
    return buf.cpu().numpy()


def materialize(lib, h: Handle, rows, cols) -> np.ndarray:
    out = torch.empty((rows, cols), dtype=torch.float16, device=dev())
    _ebx.check(lib.ebx_matrix_materialize(h.h, out.data_ptr(), stream()))
    return out.cpu().numpy()


def linear(lib, h: Handle, x: np.ndarray, rows: int, bias: np.ndarray | None = None):
    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float16)).to(dev())
    M = xd.shape[0]
    y = torch.empty((M, rows), dtype=torch.float16, device=dev())
    y32 = torch.empty((M, rows), dtype=torch.float32, device=dev())
    bd = None if bias is None else torch.from_numpy(bias.astype(np.float16)).to(dev())
    nws = int(lib.ebx_linear_workspace_bytes(h.h, M))
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=dev())
    _ebx.check(lib.ebx_linear(h.h, xd.data_ptr(), M, None if bd is None else bd.data_ptr(),
                              y.data_ptr(), y32.data_ptr(), ws.data_ptr(), nws, stream()))
    torch.cuda.synchronize()
    return y.cpu().numpy(), y32.cpu().numpy()


def assert_close_to_oracle(y16, y32, ref):
    err = np.abs(y32.astype(np.float64) - ref)
    assert err.max() <= MAX_ABS, err.max()
    rel = np.linalg.norm(y32 - ref) / max(np.linalg.norm(ref), 1e-30)
    assert rel <= REL_L2, rel
    # fp16 output is RN(y32); it can differ from RN(ref) only where y32 and
    # ref straddle a rounding boundary: by at most one fp16 ulp of the value.
    assert np.array_equal(y16, y32.astype(np.float16))
    r16 = ref.astype(np.float16)
    ulp = np.spacing(np.abs(r16)).astype(np.float64)  # gap away from zero
    gap = np.abs(y16.astype(np.float64) - r16.astype(np.float64))
    assert np.all(gap <= ulp + 2.0 * np.abs(y32.astype(np.float64) - ref))


@pytest.mark.parametrize("bits", list(range(3, 16)))
@pytest.mark.parametrize("shape", ODD_SHAPES)
def test_pack_export_and_dequant_bit_exact(lib, bits, shape):
    rows, cols = shape
    q, s = random_codes(rows, cols, bits, seed=rows * 1000 + cols * 10 + bits)
    h = from_codes(lib, q, s, bits)
    payload = export_payload(lib, h, O.packed_bytes(rows * cols, bits))
    assert np.array_equal(payload, O.pack_codes(q, bits))
    w16 = materialize(lib, h, rows, cols)
    assert np.array_equal(w16.view(np.uint16), O.dequantize_codes(q, s).view(np.uint16))


@pytest.mark.parametrize("bits", [3, 8, 9, 10, 11, 15, 16])
def test_payload_roundtrip(lib, bits):
    rows, cols = 40, 136
    if bits == 16:
        w = O.normal((rows, cols), seed=4, scale=0.05)
        payload = O.pack_weights(w, 16)
        scales = np.zeros(0, np.float32)
    else:
        q, scales = random_codes(rows, cols, bits, seed=bits)
        payload = O.pack_codes(q, bits)
    h = ctypes.c_void_p()
    _ebx.check(lib.ebx_matrix_create_from_payload(
        payload.ctypes.data, payload.size, scales.ctypes.data if scales.size else None, rows, cols,
        bits, 0, 0, stream(), ctypes.byref(h)))
    hh = Handle(h.value)
    assert np.array_equal(export_payload(lib, hh, payload.size), payload)
    ref = O.dequantize_fp16(payload, scales if bits != 16 else None, rows, cols, bits)
    assert np.array_equal(materialize(lib, hh, rows, cols).view(np.uint16), ref.view(np.uint16))


def test_out_of_range_codes_rejected(lib):
    q = np.zeros((4, 8), np.int16)
    q[2, 3] = 8  # qmax(4) = 7
    with pytest.raises(ValueError, match="exceeds selected bit range"):
        from_codes(lib, q, np.ones(4, np.float32), 4)


@pytest.mark.parametrize("bits", [3, 5, 8, 9, 10, 11, 12, 15, 16])
@pytest.mark.parametrize("M", [1, 2, 3, 8, 9, 16])
def test_decode_linear_full_semantics(lib, bits, M):
    rows, cols = 80, 384
    w = O.baseline_weights(rows, cols, seed=bits)
    if bits == 16:
        w16 = w.astype(np.float16)
        wd = torch.from_numpy(w16).to(dev())
        h = ctypes.c_void_p()
        _ebx.check(lib.ebx_matrix_create_from_fp16(wd.data_ptr(), rows, cols, 0, stream(),
                                                   ctypes.byref(h)))
        hh = Handle(h.value)
    else:
        s = O.row_scales(w, bits)
        q = O.quantize(w, s, bits)
        w16 = O.dequantize_codes(q, s)
        hh = from_codes(lib, q, s, bits)
    x = O.normal((M, cols), seed=100 + M).astype(np.float16)
    bias = O.normal((rows,), seed=7, scale=0.1).astype(np.float16)
    y16, y32 = linear(lib, hh, x, rows, bias)
    ref = O.linear_full(x, w16.astype(np.float32), bias.astype(np.float32))
    assert_close_to_oracle(y16, y32, ref)


@pytest.mark.parametrize("bits", [3, 4, 6, 8])
@pytest.mark.parametrize("M", [1, 5, 16])
def test_decode_linear_integer_semantics(lib, bits, M):
    rows, cols = 64, 256
    w = O.baseline_weights(rows, cols, seed=30 + bits)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    h = from_codes(lib, q, s, bits)
    _ebx.check(lib.ebx_matrix_set_execution_width(h.h, 8))
    x = O.normal((M, cols), seed=M).astype(np.float16)
    y16, y32 = linear(lib, h, x, rows)
    ref = O.linear_hw(x, q, s)
    assert_close_to_oracle(y16, y32, ref)
    with pytest.raises(ValueError):
        _ebx.check(lib.ebx_matrix_set_execution_width(h.h, 4 if bits > 4 else 3))


@pytest.mark.parametrize("shape", ODD_SHAPES)
@pytest.mark.parametrize("bits", [3, 7, 9, 15])
def test_decode_odd_shapes(lib, shape, bits):
    rows, cols = shape
    q, s = random_codes(rows, cols, bits, seed=rows + cols + bits)
    h = from_codes(lib, q, s, bits)
    x = O.normal((3, cols), seed=5).astype(np.float16)
    y16, y32 = linear(lib, h, x, rows)
    ref = O.linear_full(x, O.dequantize_codes(q, s).astype(np.float32))
    assert_close_to_oracle(y16, y32, ref)


@pytest.mark.parametrize("M", [17, 40, 256])
def test_multi_row_linear(lib, M):
    rows, cols, bits = 96, 512, 10
    w = O.baseline_weights(rows, cols, seed=M)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    h = from_codes(lib, q, s, bits)
    x = O.normal((M, cols), seed=M + 1).astype(np.float16)
    y16, y32 = linear(lib, h, x, rows)
    ref = O.linear_full(x, O.dequantize_codes(q, s).astype(np.float32))
    assert_close_to_oracle(y16, y32, ref)


def test_linear_is_deterministic(lib):
    rows, cols, bits = 512, 1024, 10
    q, s = random_codes(rows, cols, bits, seed=3)
    h = from_codes(lib, q, s, bits)
    x = O.normal((5, cols), seed=9).astype(np.float16)
    a = linear(lib, h, x, rows)[1]
    b = linear(lib, h, x, rows)[1]
    assert np.array_equal(a, b)


def test_empty_input_is_a_no_op(lib):
    q, s = random_codes(16, 64, 9, seed=1)
    h = from_codes(lib, q, s, 9)
    assert lib.ebx_linear(h.h, None, 0, None, None, None, None, 0, stream()) == 0


GOLDEN = json.loads((Path(__file__).parent / "golden" / "analyze_golden.json").read_text())


@pytest.mark.parametrize("name", list(GOLDEN["cases"]))
def test_device_analyzer_matches_reference_golden(lib, name):
    import make_golden as G

    case = GOLDEN["cases"][name]
    w, c, thr = G.case_inputs(name)
    assert G.sha(w, c) == case["inputs_sha256"]
    rows, cols = w.shape
    wd = torch.from_numpy(w).to(dev())
    cd = torch.from_numpy(c).to(dev())
    nws = int(lib.ebx_analyze_workspace_bytes(rows, c.shape[0]))
    ws = torch.empty(nws, dtype=torch.uint8, device=dev())
    hw = torch.empty(14, dtype=torch.float64, device=dev())
    full = torch.empty(14, dtype=torch.float64, device=dev())
    _ebx.check(lib.ebx_analyze(wd.data_ptr(), rows, cols, cd.data_ptr(), c.shape[0],
                               hw.data_ptr(), full.data_ptr(), ws.data_ptr(), nws, stream()))
    hw, full = hw.cpu().numpy(), full.cpu().numpy()
    for i, cand in enumerate(case["candidates"]):
        for mine, key in ((hw[i], "hardwareNativeError"), (full[i], "fullPrecisionError")):
            ref = float(cand[key])
            assert abs(mine - ref) <= 1e-12 * max(ref, 1e-300) + 1e-300, (key, cand["bits"])
    err = np.maximum(hw, full)
    sel = next((b for b in range(3, 16) if err[b - 3] <= thr), 16)
    assert sel == case["selectedBits"]


@pytest.mark.parametrize("bits", [3, 6, 9, 12, 15])
def test_device_quantizer_bit_exact(lib, bits):
    w = O.baseline_weights(70, 150, seed=bits)
    w[3] = 0.0
    wd = torch.from_numpy(w).to(dev())
    codes = torch.empty((70, 150), dtype=torch.int16, device=dev())
    scales = torch.empty(70, dtype=torch.float32, device=dev())
    _ebx.check(lib.ebx_quantize(wd.data_ptr(), 70, 150, bits, codes.data_ptr(), scales.data_ptr(),
                                stream()))
    s_ref = O.row_scales(w, bits)
    assert np.array_equal(scales.cpu().numpy(), s_ref)
    assert np.array_equal(codes.cpu().numpy(), O.quantize(w, s_ref, bits))


@pytest.mark.parametrize("bits", [2, 3, 5, 8])
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,group", [(3, 50), (70, 30)])
def test_elastic_linear_packed_op(lib, bits, xdt, rows, group):
    """Rows beyond one 8-row chunk and one 64-row block, and scale groups that straddle
    output features (group 30 over 100 inputs), against the oracle's scalar loop."""
    import mlbricks_b200.native as native

    inf, outf = 100, 24
    rng = np.random.default_rng(bits)
    uq = rng.integers(0, 1 << bits, size=outf * inf)
    packed = np.zeros((outf * inf * bits + 7) // 8 + 1, np.uint8)
    for i, u in enumerate(uq):  # LSB-first bitstream
        for b in range(bits):
            if (int(u) >> b) & 1:
                packed[(i * bits + b) // 8] |= 1 << ((i * bits + b) % 8)
    scales = rng.uniform(0.01, 0.1, size=(outf * inf) // group).astype(np.float32)
    x = O.normal((rows, inf), seed=1)
    bias = O.normal((outf,), seed=2)
    xt = torch.from_numpy(x).to(dev(), xdt)
    out = native.elastic_linear_packed(xt, torch.from_numpy(packed).to(dev()),
                                       torch.from_numpy(scales).to(dev()),
                                       torch.from_numpy(bias).to(dev(), xdt), bits, group, outf, inf)
    ref = O.elastic_linear_packed(xt.float().cpu().numpy(), packed, scales,
                                  torch.from_numpy(bias).to(xdt).float().numpy(), bits, group,
                                  outf, inf)
    tol = 1e-4 if xdt == torch.float32 else 3e-2
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=tol, atol=tol)


@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 14336), (14336, 4096)])
def test_baseline_decode_shapes(lib, K, N):
    bits = 10
    w = O.baseline_weights(N, K, seed=K + N)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    h = from_codes(lib, q, s, bits)
    payload = export_payload(lib, h, O.packed_bytes(N * K, bits))
    # checksum of the MLB4 payload instead of a byte compare of ~70 MB
    assert O.fnv1a64(payload) == O.fnv1a64(O.pack_codes(q, bits))
    x = O.normal((16, K), seed=3).astype(np.float16)
    y16, y32 = linear(lib, h, x, N)
    ref = O.linear_full(x, O.dequantize_codes(q, s).astype(np.float32))
    assert_close_to_oracle(y16, y32, ref)
    # linearity in x (a size-independent property): f(2x) == 2 f(x) exactly in fp32
    y16b, y32b = linear(lib, h, (x.astype(np.float32) * 2).astype(np.float16), N)
    assert np.array_equal(y32b, 2 * y32)


def test_device_status_healthy_after_all_kernels(lib):
    st = ctypes.c_int32(-1)
    _ebx.check(lib.ebx_device_status(0, ctypes.byref(st), 0))
    assert st.value == 0


# ragged token counts and rows (last tiles partly past M and N), K not a multiple of 64
@pytest.mark.parametrize("M,rows,cols", [(65, 96, 512), (128, 256, 64), (300, 1000, 520),
                                         (256, 1536, 384), (512, 4096, 4096), (200, 4096, 14336),
                                         (1024, 4096, 512), (2048, 4096, 256), (2100, 2600, 200)])
def test_prefill_gemm(lib, M, rows, cols):
    """Larger M with the workspace ebx_linear_workspace_bytes offers: materialise +
    tcgen05 GEMM; 16 < M <= 256: the decode-GEMM with the weights as the MMA's
    128-row side."""
    bits = 10
    w = O.baseline_weights(rows, cols, seed=M + rows)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    h = from_codes(lib, q, s, bits)
    if M > 256:  # optional workspace: the exact fp16 weight (materialise + GEMM route)
        assert lib.ebx_linear_workspace_bytes(h.h, M) >= rows * cols * 2
    x = O.normal((M, cols), seed=M).astype(np.float16)
    bias = O.normal((rows,), seed=5, scale=0.1).astype(np.float16)
    y16, y32 = linear(lib, h, x, rows, bias)
    w16 = O.dequantize_codes(q, s).astype(np.float64)
    ref = x.astype(np.float64) @ w16.T + bias.astype(np.float64)
    assert_close_to_oracle(y16, y32, ref)
    y16b, y32b = linear(lib, h, x, rows, bias)
    assert np.array_equal(y32b, y32)  # deterministic


@pytest.mark.parametrize("M,rows,cols,bits", [(300, 1000, 520, 10), (1024, 4096, 512, 9),
                                              (2100, 2600, 200, 12), (512, 4096, 4096, 11)])
def test_prefill_without_workspace(lib, M, rows, cols, bits):
    """Larger M and no workspace: the prefill decode-GEMM decodes the codes into the
    tensor-core B tile per k-block (no memory beyond inputs and outputs)."""
    w = O.baseline_weights(rows, cols, seed=M + bits)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    h = from_codes(lib, q, s, bits)
    x = torch.from_numpy(O.normal((M, cols), seed=M).astype(np.float16)).to(dev())
    bias = torch.from_numpy(O.normal((rows,), seed=5, scale=0.1).astype(np.float16)).to(dev())
    xb = x.cpu().numpy().astype(np.float64)
    bb = bias.cpu().numpy().astype(np.float64)
    w16 = O.dequantize_codes(q, s).astype(np.float64)
    refs = {16: xb @ w16.T + bb,  # fullPrecision: fp16(q * s) operands
            12: (xb @ q.astype(np.float64).T) * s.astype(np.float64) + bb}  # integer codes
    for width in (16, 12):
        _ebx.check(lib.ebx_matrix_set_execution_width(h.h, width))
        y = torch.empty((M, rows), dtype=torch.float16, device=dev())
        y32 = torch.empty((M, rows), dtype=torch.float32, device=dev())
        _ebx.check(lib.ebx_linear(h.h, x.data_ptr(), M, bias.data_ptr(), y.data_ptr(),
                                  y32.data_ptr(), None, 0, stream()))
        torch.cuda.synchronize()
        assert_close_to_oracle(y.cpu().numpy(), y32.cpu().numpy(), refs[width])


def test_split_k_without_workspace_is_refused(lib):
    # decode-GEMM with K split over CTAs: the fp32 partials need the caller's workspace
    q, s = random_codes(512, 4096, 9, seed=3)
    h = from_codes(lib, q, s, 9)
    assert lib.ebx_linear_workspace_bytes(h.h, 100) > 0
    x = torch.zeros((100, 4096), dtype=torch.float16, device=dev())
    y = torch.empty((100, 512), dtype=torch.float16, device=dev())
    st = lib.ebx_linear(h.h, x.data_ptr(), 100, None, y.data_ptr(), None, None, 0, stream())
    assert st == _ebx.EBX_ERR_WORKSPACE
