"""Decode (M <= 16 per launch) and the decode-GEMM (16 < M <= 256) at BASELINE sizes and
ragged shapes, through the C ABI.

Covers the 4096x4096, 14336x4096 and 4096x14336 decode shapes and ragged ones
(N not a multiple of 16, one or two k-tiles per row) at every bit-width class
of the decode kernel (b = 9..12 are stored in the plane layout and decoded
with byte permutes, b = 8 takes the paired f32x2 dequantisation under the full
semantics, b = 13 the per-code one), the full and the integer (scale after
accumulation; execution width 12 for b = 9..12) semantics, back-to-back launches of one matrix, first launches of matrices
created on recycled device memory, CUDA-graph replays of launches that may
overlap through programmatic dependent launch, and bit-identical repeats.

Bars: y32 within max-abs 2e-3 and relative L2 1e-3 of the float64 product of
the activations with the exactly dequantised weight (itself pinned bit-exact
to the oracle by test_gpu_kernels), and y = RN_fp16(y32).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from mlbricks_b200 import _ebx
from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
REL_L2 = 1e-3


@pytest.fixture(scope="module")
def lib(cuda_ok):
    return _ebx.load()


def dev():
    return torch.device("cuda", 0)


class Handle:
    def __init__(self, ptr: int):
        self.h = ctypes.c_void_p(ptr)

    def __del__(self):
        if self.h.value:
            _ebx.load().ebx_matrix_destroy(self.h)


def make(lib, rows, cols, bits, seed):
    """Seeded BASELINE-style weights quantised on the host (oracle), packed on the device."""
    g = torch.Generator(device=dev())
    g.manual_seed(seed)
    sig = torch.empty((rows, 1), device=dev()).uniform_(np.log(0.005), np.log(0.05), generator=g)
    w = (torch.randn((rows, cols), device=dev(), generator=g) * torch.exp(sig)).half().float()
    qm = O.qmax(bits)
    amax = w.abs().amax(dim=1)
    s = torch.where(amax > 0, amax / qm, torch.ones_like(amax)).float()
    q = torch.round(w / s[:, None]).clamp(-qm, qm).to(torch.int16).contiguous()
    h = ctypes.c_void_p()
    _ebx.check(lib.ebx_matrix_create_from_codes(q.data_ptr(), s.data_ptr(), rows, cols, bits, 0,
                                                _ebx.stream_ptr(), ctypes.byref(h)))
    return Handle(h.value), q, s


def materialize(lib, h, rows, cols):
    out = torch.empty((rows, cols), dtype=torch.float16, device=dev())
    _ebx.check(lib.ebx_matrix_materialize(h.h, out.data_ptr(), _ebx.stream_ptr()))
    return out


def run(lib, h, x, rows, bias=None, y=None, y32=None):
    M = x.shape[0]
    y = torch.empty((M, rows), dtype=torch.float16, device=dev()) if y is None else y
    y32 = torch.empty((M, rows), dtype=torch.float32, device=dev()) if y32 is None else y32
    _ebx.check(lib.ebx_linear(h.h, x.data_ptr(), M, None if bias is None else bias.data_ptr(),
                              y.data_ptr(), y32.data_ptr(), None, 0, _ebx.stream_ptr()))
    return y, y32


def check(y, y32, ref):
    err = (y32.double() - ref).abs().max().item()
    rel = ((y32.double() - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert err <= MAX_ABS, err
    assert rel <= REL_L2, rel
    assert torch.equal(y, y32.half())


SHAPES = [
    (4096, 4096, 10),   # config 2, 4096x4096
    (14336, 4096, 9),   # N = 14336, K = 4096 (a grid of about two waves)
    (4096, 14336, 11),  # N = 4096, K = 14336
    (4096, 4096, 12),   # 12-bit codes: in-place offsets 0, 4, 8
    (512, 1024, 8),     # 8-bit codes, full semantics
    (1000, 576, 9),     # N not a multiple of 16, 9 k-tiles per row
    (4097, 128, 12),    # two k-tiles per row, a last group of one row
    (30, 64, 13),       # one k-tile per row, fewer tiles than one round; per-code decode
]


@pytest.mark.parametrize("rows,cols,bits", SHAPES)
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
def test_decode_full_semantics(lib, rows, cols, bits, M):
    h, q, s = make(lib, rows, cols, bits, seed=rows + cols + bits)
    w16 = materialize(lib, h, rows, cols)
    x = torch.randn((M, cols), device=dev()).half()
    bias = (0.1 * torch.randn(rows, device=dev())).half()
    y, y32 = run(lib, h, x, rows, bias)
    torch.cuda.synchronize()
    ref = x.double() @ w16.double().t() + bias.double()
    check(y, y32, ref)


@pytest.mark.parametrize("bits", [4, 8, 9, 10, 11, 12])
@pytest.mark.parametrize("M", [1, 6, 16])
def test_decode_integer_semantics(lib, bits, M):
    rows, cols = 3000, 1024
    h, q, s = make(lib, rows, cols, bits, seed=bits + M)
    _ebx.check(lib.ebx_matrix_set_execution_width(h.h, 8 if bits <= 8 else 12))
    x = torch.randn((M, cols), device=dev()).half()
    y, y32 = run(lib, h, x, rows)
    torch.cuda.synchronize()
    ref = (x.double() @ q.double().t()) * s.double()
    check(y, y32, ref)


@pytest.mark.parametrize("rows,cols,bits", [sh for sh in SHAPES if 8 <= sh[2] <= 12])
@pytest.mark.parametrize("M", [1, 2, 8, 16])
def test_decode_integer_semantics_shapes(lib, rows, cols, bits, M):
    """Execution width 12 (8 for b = 8) at the BASELINE and ragged shapes:
    y = fp16(s * sum_k x_k q_k + bias), the reference's W8A16 arithmetic."""
    h, q, s = make(lib, rows, cols, bits, seed=3 * rows + cols + bits)
    _ebx.check(lib.ebx_matrix_set_execution_width(h.h, 8 if bits <= 8 else 12))
    x = torch.randn((M, cols), device=dev()).half()
    bias = (0.1 * torch.randn(rows, device=dev())).half()
    y, y32 = run(lib, h, x, rows, bias)
    torch.cuda.synchronize()
    ref = (x.double() @ q.double().t()) * s.double() + bias.double()
    check(y, y32, ref)


def test_decode_repeats_are_bit_identical(lib):
    rows, cols, bits = 14336, 4096, 10
    h, q, s = make(lib, rows, cols, bits, seed=5)
    w16 = materialize(lib, h, rows, cols).double()
    outs = []
    for M in (1, 16, 5, 16, 1):  # back-to-back launches of one matrix, different M
        x = torch.randn((M, cols), device=dev(), generator=torch.Generator(device=dev()).manual_seed(M)).half()
        outs.append((M, x, run(lib, h, x, rows)))
    torch.cuda.synchronize()
    for M, x, (y, y32) in outs:
        check(y, y32, x.double() @ w16.t())
    assert torch.equal(outs[0][2][1], outs[4][2][1])
    assert torch.equal(outs[1][2][1], outs[3][2][1])


def test_decode_fresh_matrices_on_recycled_memory(lib):
    """Matrices created after others were destroyed (their device memory is
    recycled) give correct results on their first launches."""
    rows, cols, bits = 4096, 4096, 11
    for seed in range(4):
        h, q, s = make(lib, rows, cols, bits, seed=100 + seed)
        w16 = materialize(lib, h, rows, cols).double()
        x = torch.randn((5, cols), device=dev()).half()
        y, y32 = run(lib, h, x, rows)
        torch.cuda.synchronize()
        check(y, y32, x.double() @ w16.t())
        del h
        torch.cuda.synchronize()


def test_decode_graph_replay_matches_eager(lib):
    """Several launches of one matrix captured in a CUDA graph (consecutive kernels
    may overlap through programmatic dependent launch) give the eager results."""
    rows, cols, bits = 4096, 4096, 10
    h, q, s = make(lib, rows, cols, bits, seed=9)
    xs = [torch.randn((M, cols), device=dev()).half() for M in (1, 4, 16, 4)]
    ys = [torch.empty((x.shape[0], rows), dtype=torch.float16, device=dev()) for x in xs]
    y32s = [torch.empty((x.shape[0], rows), dtype=torch.float32, device=dev()) for x in xs]
    eager = [run(lib, h, x, rows)[1].clone() for x in xs]
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(dev())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for x, y, y32 in zip(xs, ys, y32s):
            _ebx.check(lib.ebx_linear(h.h, x.data_ptr(), x.shape[0], None, y.data_ptr(),
                                      y32.data_ptr(), None, 0, _ebx.stream_ptr()))
    for _ in range(3):
        for y32 in y32s:
            y32.zero_()
        g.replay()
        torch.cuda.synchronize()
        for a, b in zip(eager, y32s):
            assert torch.equal(a, b)
    st = ctypes.c_int32(-1)
    _ebx.check(lib.ebx_device_status(0, ctypes.byref(st), 0))
    assert st.value == 0


# ---------------------------------------------------------------------------
# 16 < M <= 256: the decode-GEMM (codes decoded straight into tensor-core tiles)
# ---------------------------------------------------------------------------
def run_ws(lib, h, x, rows, bias=None):
    """ebx_linear with the workspace ebx_linear_workspace_bytes asks for."""
    M = x.shape[0]
    y = torch.empty((M, rows), dtype=torch.float16, device=dev())
    y32 = torch.empty((M, rows), dtype=torch.float32, device=dev())
    nws = int(lib.ebx_linear_workspace_bytes(h.h, M))
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=dev())
    _ebx.check(lib.ebx_linear(h.h, x.data_ptr(), M, None if bias is None else bias.data_ptr(),
                              y.data_ptr(), y32.data_ptr(), ws.data_ptr(), nws, _ebx.stream_ptr()))
    return y, y32


DG_SHAPES = [
    (4096, 4096, 10),   # K split over CTAs (32 weight-row blocks)
    (14336, 4096, 9),   # 112 row blocks
    (4096, 14336, 11),  # K = 14336
    (1000, 576, 12),    # ragged rows, 9 k-tiles
    (200, 72, 13),      # K not a multiple of 64 (activations past K read as zeros)
]


@pytest.mark.parametrize("rows,cols,bits", DG_SHAPES)
@pytest.mark.parametrize("M", [17, 33, 64, 100, 256])
def test_decode_gemm_full_semantics(lib, rows, cols, bits, M):
    h, q, s = make(lib, rows, cols, bits, seed=rows + cols + bits + M)
    w16 = materialize(lib, h, rows, cols)
    x = torch.randn((M, cols), device=dev()).half()
    bias = (0.1 * torch.randn(rows, device=dev())).half()
    y, y32 = run_ws(lib, h, x, rows, bias)
    torch.cuda.synchronize()
    check(y, y32, x.double() @ w16.double().t() + bias.double())
    st = ctypes.c_int32(-1)
    _ebx.check(lib.ebx_device_status(0, ctypes.byref(st), 0))
    assert st.value == 0


@pytest.mark.parametrize("bits", [4, 8, 9, 10, 11, 12])
@pytest.mark.parametrize("M", [24, 128, 300, 1024])
def test_decode_gemm_integer_semantics(lib, bits, M):
    rows, cols = 3000, 1024
    h, q, s = make(lib, rows, cols, bits, seed=bits + M)
    _ebx.check(lib.ebx_matrix_set_execution_width(h.h, 8 if bits <= 8 else 12))
    x = torch.randn((M, cols), device=dev()).half()
    if M > 256:
        # prefill sizes honour integer semantics on the workspace-free decode-GEMM route (the
        # optional fp16 workspace route computes the reference's fp16(q * s) prefill)
        y, y32 = run(lib, h, x, rows)
    else:
        y, y32 = run_ws(lib, h, x, rows)
    torch.cuda.synchronize()
    check(y, y32, (x.double() @ q.double().t()) * s.double())


def test_decode_gemm_fp16_storage(lib):
    rows, cols, M = 640, 512, 48
    w = (0.02 * torch.randn((rows, cols), device=dev())).half().contiguous()
    hp = ctypes.c_void_p()
    _ebx.check(lib.ebx_matrix_create_from_fp16(w.data_ptr(), rows, cols, 0, _ebx.stream_ptr(),
                                               ctypes.byref(hp)))
    h = Handle(hp.value)
    x = torch.randn((M, cols), device=dev()).half()
    y, y32 = run_ws(lib, h, x, rows)
    torch.cuda.synchronize()
    check(y, y32, x.double() @ w.double().t())


def test_decode_gemm_graph_replay_and_repeats(lib):
    rows, cols, bits = 4096, 4096, 10
    h, q, s = make(lib, rows, cols, bits, seed=77)
    outs = []
    for M in (64, 200, 64):
        x = torch.randn((M, cols), device=dev(), generator=torch.Generator(device=dev()).manual_seed(M)).half()
        outs.append(run_ws(lib, h, x, rows)[1].clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[2])
    M = 96
    x = torch.randn((M, cols), device=dev()).half()
    eager = run_ws(lib, h, x, rows)[1].clone()
    nws = int(lib.ebx_linear_workspace_bytes(h.h, M))
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=dev())
    y = torch.empty((M, rows), dtype=torch.float16, device=dev())
    y32 = torch.empty((M, rows), dtype=torch.float32, device=dev())
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(dev())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        _ebx.check(lib.ebx_linear(h.h, x.data_ptr(), M, None, y.data_ptr(), y32.data_ptr(),
                                  ws.data_ptr(), nws, _ebx.stream_ptr()))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(eager, y32)
