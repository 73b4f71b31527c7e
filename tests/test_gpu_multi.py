"""One decode launch over several matrices that read the same activations
(ebx_linear_multi; reference: fused multi-matrix execution, stage2f.py:382-420),
through the C ABI and from ElasticBit.compress-produced models (Q/K/V siblings).

Bars as for the single-matrix decode: y32 within max-abs 2e-3 and relative L2
1e-3 of the float64 product with the exactly dequantised weight (fullPrecision)
or of s * (x @ q) (integer-code semantics), y = RN_fp16(y32).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from mlbricks_b200 import _ebx
from oracle import oracle as O

pytestmark = pytest.mark.gpu

MATS = [(4096, 4096, 9), (512, 4096, 10), (1000, 4096, 12)]  # rows, cols, bits (ragged rows)


@pytest.fixture(scope="module")
def lib(cuda_ok):
    return _ebx.load()


def _make(lib, rows, cols, bits, seed, width):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qm = O.qmax(bits)
    q = torch.randint(-qm, qm + 1, (rows, cols), device="cuda", generator=g).to(torch.int16)
    s = torch.rand(rows, device="cuda", generator=g) * 2e-4 + 1e-5
    h = ctypes.c_void_p()
    _ebx.check(lib.ebx_matrix_create_from_codes(q.data_ptr(), s.data_ptr(), rows, cols, bits, 0,
                                                _ebx.stream_ptr(), ctypes.byref(h)))
    _ebx.check(lib.ebx_matrix_set_execution_width(h, width))
    return h, q, s


def _check(y, y32, ref):
    err = (y32.double() - ref).abs().max().item()
    rel = ((y32.double() - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert err <= 2e-3 and rel <= 1e-3, (err, rel)
    assert torch.equal(y, y32.half())


@pytest.mark.parametrize("integer", [True, False])
@pytest.mark.parametrize("M", [1, 5, 8, 16])
def test_linear_multi_matches_each_matrix(lib, integer, M):
    made = [_make(lib, r, c, b, 7 * i + M, 12 if integer else 16) for i, (r, c, b) in enumerate(MATS)]
    x = torch.randn((M, 4096), device="cuda", dtype=torch.float16)
    biases = [None, (0.1 * torch.randn(512, device="cuda")).half(), None]
    ys = [torch.empty((M, r), device="cuda", dtype=torch.float16) for r, _, _ in MATS]
    y32s = [torch.empty((M, r), device="cuda", dtype=torch.float32) for r, _, _ in MATS]
    n = len(MATS)
    hs = (ctypes.c_void_p * n)(*[h.value for h, _, _ in made])
    bp = (ctypes.c_void_p * n)(*[None if b is None else b.data_ptr() for b in biases])
    yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
    y32p = (ctypes.c_void_p * n)(*[y.data_ptr() for y in y32s])
    _ebx.check(lib.ebx_linear_multi(hs, n, x.data_ptr(), M, bp, yp, y32p, _ebx.stream_ptr()))
    torch.cuda.synchronize()
    for (h, q, s), b, y, y32 in zip(made, biases, ys, y32s):
        if integer:
            ref = (x.double() @ q.double().t()) * s.double()
        else:
            w16 = (q.float() * s[:, None]).half()
            ref = x.double() @ w16.double().t()
        if b is not None:
            ref = ref + b.double()
        _check(y, y32, ref)
    for h, _, _ in made:
        lib.ebx_matrix_destroy(h)
    st = ctypes.c_int32(-1)
    _ebx.check(lib.ebx_device_status(0, ctypes.byref(st), 0))
    assert st.value == 0


def test_linear_multi_refuses_what_one_launch_cannot_run(lib):
    h13, _, _ = _make(lib, 64, 256, 13, 1, 16)
    h10, _, _ = _make(lib, 64, 256, 10, 2, 12)
    x = torch.randn((2, 256), device="cuda", dtype=torch.float16)
    ys = [torch.empty((2, 64), device="cuda", dtype=torch.float16) for _ in range(2)]
    hs = (ctypes.c_void_p * 2)(h13.value, h10.value)
    yp = (ctypes.c_void_p * 2)(*[y.data_ptr() for y in ys])
    assert lib.ebx_linear_multi(hs, 2, x.data_ptr(), 2, None, yp, None,
                                _ebx.stream_ptr()) == _ebx.EBX_ERR_UNSUPPORTED
    assert lib.ebx_linear_multi(hs, 2, x.data_ptr(), 17, None, yp, None,
                                _ebx.stream_ptr()) == _ebx.EBX_ERR_INVALID
    lib.ebx_matrix_destroy(h13)
    lib.ebx_matrix_destroy(h10)


class _Attn(torch.nn.Module):
    def __init__(self, d=512, kv=64):
        super().__init__()
        self.q = torch.nn.Linear(d, d, bias=False)
        self.k = torch.nn.Linear(d, kv, bias=True)
        self.v = torch.nn.Linear(d, kv, bias=False)
        self.o = torch.nn.Linear(d + 2 * kv, d, bias=False)

    def forward(self, x):
        return self.o(torch.cat([self.q(x), self.k(x), self.v(x)], dim=-1))


def test_compress_fuses_siblings_into_one_launch(cuda_ok, monkeypatch):
    from mlbricks_b200 import ElasticBit
    from mlbricks_b200.elasticbit import _native

    torch.manual_seed(5)
    model = _Attn().cuda().half().eval()
    with torch.no_grad():  # different scales -> different selected widths
        model.q.weight.copy_(torch.from_numpy(O.baseline_weights(512, 512, seed=1)))
        model.k.weight.mul_(0.3)
        model.v.weight.copy_(torch.from_numpy(O.baseline_weights(64, 512, seed=2)) * 4)
    calib = torch.randn(4, 16, 512, device="cuda", dtype=torch.float16)
    ElasticBit.compress(model, calib, 0.01, backend="native")
    group = model.q._fused
    assert group is not None and model.k._fused is group and model.v._fused is group
    assert model.o._fused is None
    calls = {"multi": 0}
    real = _native.RuntimeMatrix.linear_multi

    def counting(mats, x, biases=None):
        calls["multi"] += 1
        return real(mats, x, biases)

    monkeypatch.setattr(_native.RuntimeMatrix, "linear_multi", staticmethod(counting))
    for M in (1, 8, 16):
        x = torch.randn(M, 512, device="cuda", dtype=torch.float16)
        before = calls["multi"]
        fused = model(x)
        assert calls["multi"] == before + 1  # q, k and v in one launch
        for layer in (model.q, model.k, model.v):
            layer._fused = None
        alone = model(x)
        for layer in (model.q, model.k, model.v):
            layer._fused = group
        torch.testing.assert_close(fused, alone, atol=2e-3, rtol=2e-3)
    big = torch.randn(64, 512, device="cuda", dtype=torch.float16)
    before = calls["multi"]
    model(big)  # prefill sizes run each member on its own
    assert calls["multi"] == before
