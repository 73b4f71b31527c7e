"""ebx_linear_swiglu (decode batches): silu(g) * u straight from the fp32 sums of a
gate/up matrix interleaved in blocks of 8, against the same sums taken from
ebx_linear's fp32 output of that matrix with the activation done in torch fp32."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from mlbricks_b200 import RuntimeMatrix
from mlbricks_b200.elasticbit.tensor_parallel import SwiGLULinear, interleave_by8
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _pair(I, K, bits, seed):
    out = []
    for j in range(2):
        w = O.baseline_weights(I, K, seed=seed + j)
        s = O.row_scales(w, bits)
        out.append((O.quantize(w, s, bits), s))
    return out


# K = 4096 / 520: pipelined and generic decode kernels; M up to 16; 8192 x 4096 interleaved
# rows (a grid of several waves)
@pytest.mark.parametrize("I,K,bits", [(512, 4096, 10), (136, 520, 11), (1792, 1024, 9),
                                        (4096, 4096, 10)])
@pytest.mark.parametrize("M", [1, 5, 16])
@pytest.mark.parametrize("with_bias", [False, True])
def test_swiglu_matches_linear_then_activation(cuda_ok, I, K, bits, M, with_bias):
    (gq, gs), (uq, us) = _pair(I, K, bits, seed=I + K)
    q = interleave_by8(gq, uq)
    s = interleave_by8(gs, us)
    m = RuntimeMatrix._compressSelectedCodes(q, s, bits, 0.0, 0.0, decodePolicy="fullPrecision")
    x = torch.from_numpy(O.normal((M, K), seed=M).astype(np.float16)).cuda()
    bias = (torch.from_numpy(O.normal((2 * I,), seed=7, scale=0.1).astype(np.float16)).cuda()
            if with_bias else None)
    y, y32 = m._native.linear_swiglu(x, bias, out32=True)
    _, full32 = m._native.linear(x, bias, out32=True)
    f = full32.view(M, I // 8, 2, 8)
    g, u = f[:, :, 0, :].reshape(M, I), f[:, :, 1, :].reshape(M, I)
    ref32 = g / (1.0 + torch.exp(-g)) * u
    assert torch.allclose(y32, ref32, rtol=2e-6, atol=1e-6)
    ref16 = ref32.half().cpu().numpy()                        # float16
    ulp = np.spacing(np.abs(ref16)).astype(np.float32)         # one fp16 ulp
    assert np.all(np.abs(y.float().cpu().numpy() - ref16.astype(np.float32)) <= ulp)
    # the module takes the fused launch for decode batches, the composed path above 16 rows
    mod = SwiGLULinear(m, I, K)
    assert torch.equal(mod(x), m._native.linear_swiglu(x))
    x_big = torch.from_numpy(O.normal((40, K), seed=3).astype(np.float16)).cuda()
    big = mod(x_big)
    fb = m._native.linear(x_big, None, out32=True)[1].view(40, I // 8, 2, 8)
    expect = (torch.nn.functional.silu(fb[:, :, 0, :]) * fb[:, :, 1, :]).reshape(40, I).half()
    assert torch.equal(big, expect)  # fp32 sums, fp32 activation, one rounding


def test_swiglu_argument_checks(cuda_ok):
    (gq, gs), (uq, us) = _pair(16, 64, 9, seed=1)
    m = RuntimeMatrix._compressSelectedCodes(interleave_by8(gq, uq), interleave_by8(gs, us), 9,
                                             0.0, 0.0, decodePolicy="fullPrecision")
    with pytest.raises(ValueError, match="M <= 16"):
        m._native.linear_swiglu(torch.zeros((17, 64), dtype=torch.float16, device="cuda"))
    odd = RuntimeMatrix._compressSelectedCodes(gq[:8], gs[:8], 9, 0.0, 0.0,
                                               decodePolicy="fullPrecision")
    with pytest.raises(ValueError, match="multiple of 16"):
        odd._native.linear_swiglu(torch.zeros((1, 64), dtype=torch.float16, device="cuda"))
