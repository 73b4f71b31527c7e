"""libebx tensor-parallel exchange on one GPU (world = 1): the row-parallel
decode kernel's exchange epilogue (p_0 + bias, rounded once) must agree with
ebx_linear to within one fp16 ulp (the plain route runs the stream-K kernel,
whose fp32 summation order differs), and repeat bit for bit over successive
calls (epochs alternate the two slots) and inside a replayed CUDA graph.  The
multi-GPU form is covered in test_gpu_tp.py."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from mlbricks_b200 import RuntimeMatrix
from mlbricks_b200.elasticbit.tensor_parallel import Exchange
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _close(y, y32, ref, ref32):
    """fp32 sums agree to summation-order rounding; fp16 outputs to one ulp."""
    r32 = ref32.double()
    assert torch.all((y32.double() - r32).abs() <= 1e-5 * r32.abs().clamp_min(1.0))
    r16 = ref.float()
    ulp = torch.from_numpy(np.spacing(np.abs(ref.cpu().numpy())).astype(np.float32)).to(ref.device)
    assert torch.all((y.float() - r16).abs() <= torch.maximum(ulp, torch.full_like(ulp, 2e-3)))


def _single_rank_exchange(max_m=16, max_n=4096):
    return Exchange(max_m, max_n, 1, 0, torch.cuda.current_device(), lambda b: [b])


def _matrix(N, K, bits, seed):
    w = O.baseline_weights(N, K, seed=seed)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    return RuntimeMatrix._compressSelectedCodes(q, s, bits, 0.0, 0.0, decodePolicy="fullPrecision")


@pytest.mark.parametrize("N,K,bits", [(512, 1024, 10), (300, 520, 11), (98, 192, 5), (4096, 512, 12)])
@pytest.mark.parametrize("protocol", ["auto", "broadcast", "two_phase"])
def test_exchange_world1_matches_linear(cuda_ok, N, K, bits, protocol):
    """Both exchange protocols (with one rank, the two-phase owner is this rank for
    every output: it sums its own words and has nobody to store the sum to)."""
    m = _matrix(N, K, bits, seed=N + K)
    ex = _single_rank_exchange()
    ex.set_protocol(protocol)
    bias = torch.from_numpy(O.normal((N,), seed=3, scale=0.1).astype(np.float16)).cuda()
    try:
        for M in (1, 5, 16):
            x = torch.from_numpy(O.normal((M, K), seed=M).astype(np.float16)).cuda()
            for b in (None, bias):
                ref, ref32 = m._native.linear(x, b, out32=True)
                first = None
                for _ in range(3):  # successive epochs use both slots
                    y, y32 = m._native.linear_allreduce(x, ex, bias=b, out32=True)
                    _close(y, y32, ref, ref32)
                    if first is None:
                        first = (y.clone(), y32.clone())
                    assert torch.equal(y, first[0]) and torch.equal(y32, first[1])
    finally:
        torch.cuda.synchronize()
        ex.close()


def test_exchange_world1_in_cuda_graph(cuda_ok):
    N, K = 1024, 2048
    m = _matrix(N, K, 10, seed=5)
    ex = _single_rank_exchange()
    try:
        x = torch.from_numpy(O.normal((4, K), seed=9).astype(np.float16)).cuda()
        ref = m._native.linear_allreduce(x, ex)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            m._native.linear_allreduce(x, ex)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            y = m._native.linear_allreduce(x, ex)
        for i in range(4):
            y.zero_()
            with torch.cuda.stream(s):
                g.replay()
            s.synchronize()
            assert torch.equal(y, ref), i
        del g
    finally:
        torch.cuda.synchronize()
        ex.close()


def test_exchange_limits_and_same_gpu_refusal(cuda_ok):
    m = _matrix(64, 128, 9, seed=1)
    ex = _single_rank_exchange(max_m=4, max_n=64)
    try:
        x = torch.zeros((5, 128), dtype=torch.float16, device="cuda")
        with pytest.raises(ValueError, match="max_m"):
            m._native.linear_allreduce(x, ex)
        big = _matrix(80, 128, 9, seed=2)
        with pytest.raises(ValueError, match="max_n"):
            big._native.linear_allreduce(x[:1], ex)
    finally:
        ex.close()
    # two "ranks" on one GPU: connect must refuse (kernels that wait on each other
    # must never share a GPU), before anything is launched
    import ctypes

    from mlbricks_b200 import _ebx
    lib = _ebx.load()
    hs, raw = [], []
    for r in range(2):
        blob = (ctypes.c_uint8 * _ebx.EXCHANGE_HANDLE_BYTES)()
        h = ctypes.c_void_p()
        _ebx.check(lib.ebx_exchange_create(2, r, torch.cuda.current_device(), 1, 64, blob,
                                           ctypes.byref(h)))
        hs.append(h)
        raw.append(bytes(blob))
    try:
        st = lib.ebx_exchange_connect(hs[0], raw[0] + raw[1])
        assert st == _ebx.EBX_ERR_UNSUPPORTED and "share one GPU" in _ebx.last_error()
    finally:
        for h in hs:
            lib.ebx_exchange_destroy(h)
