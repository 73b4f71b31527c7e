"""torch.library registrations of the native compressed-linear operators.

Counterpart of the reference's ``mlbricks/custom_ops.py`` (FakeTensor kernel
for ``mlbricks_native::elastic_linear_packed`` at custom_ops.py:226-236, 346)
plus the C++ schema the reference declares in ops.cpp:1132.  Here both the
schema and the CUDA implementation are registered from Python over libebx:

* ``mlbricks_native::elastic_linear_packed(Tensor x, Tensor packed,
  Tensor scales, Tensor bias, int bits, int group_size, int out_features,
  int in_features) -> Tensor`` -- same schema and checks as the reference op
  (ops.cpp:1012-1043); an empty ``bias`` means no bias;
* ``mlbricks_native::elastic_linear(Tensor x, int matrix, int out_features,
  Tensor? bias) -> Tensor`` -- the RuntimeMatrix route (``matrix`` is the libebx
  handle of a live RuntimeMatrix), so torch.compile / FakeTensor tracing see a
  stable dispatcher op instead of a ctypes call.

Both have fake (meta) kernels and no autograd (inference-only, as in the
reference).
"""
from __future__ import annotations

import torch

from . import _ebx

_NAMESPACE = "mlbricks_native"
_REGISTERED = False
_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _elastic_linear_packed_impl(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                                bias: torch.Tensor, bits: int, group_size: int,
                                out_features: int, in_features: int) -> torch.Tensor:
    _check(x.is_cuda, "elastic_linear_packed is CUDA-only")
    _check(x.is_contiguous() and packed.is_contiguous() and scales.is_contiguous(),
           "x/packed/scales must be contiguous")
    _check(x.is_floating_point() and scales.is_floating_point(), "x/scales must be floating point")
    _check(packed.dtype == torch.uint8, "packed weight must be uint8")
    _check(x.shape[-1] == in_features, "input feature mismatch")
    _check(2 <= bits <= 8, "bits must be in [2,8]")
    _check(group_size > 0 and out_features > 0 and in_features > 0,
           "invalid ElasticBit dimensions")
    _check(packed.device == x.device and scales.device == x.device,
           "ElasticBit buffers must be on the same CUDA device as x")
    _check(bias.numel() == 0 or (bias.device == x.device and bias.dtype == x.dtype
                                 and bias.numel() == out_features),
           "bias must be empty or match output features/device/dtype")
    _check(x.dtype in _DTYPE_CODE and scales.dtype in _DTYPE_CODE, "unsupported dtype")
    rows = x.numel() // in_features
    out = torch.empty((*x.shape[:-1], out_features), dtype=x.dtype, device=x.device)
    lib = _ebx.load()
    with torch.cuda.device(x.device):
        _ebx.check(lib.ebx_elastic_linear_packed(
            x.data_ptr(), _DTYPE_CODE[x.dtype], rows, packed.data_ptr(), scales.data_ptr(),
            _DTYPE_CODE[scales.dtype], bias.data_ptr() if bias.numel() else None, int(bits),
            int(group_size), int(out_features), int(in_features), out.data_ptr(),
            _ebx.stream_ptr()))
    return out


def _elastic_linear_impl(x: torch.Tensor, matrix: int, out_features: int,
                         bias: torch.Tensor | None) -> torch.Tensor:
    _check(x.is_cuda and x.dtype == torch.float16, "elastic_linear requires FP16 CUDA input")
    xc = x.contiguous()
    rows = xc.numel() // xc.shape[-1]
    out = torch.empty((*x.shape[:-1], out_features), dtype=torch.float16, device=x.device)
    lib = _ebx.load()
    b = None if bias is None else bias.to(device=x.device, dtype=torch.float16).contiguous()
    ws_bytes = int(lib.ebx_linear_workspace_bytes(matrix, rows))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
    with torch.cuda.device(x.device):
        _ebx.check(lib.ebx_linear(matrix, xc.data_ptr(), rows, None if b is None else b.data_ptr(),
                                  out.data_ptr(), None, None if ws is None else ws.data_ptr(),
                                  ws_bytes, _ebx.stream_ptr()))
    return out


def register_native_custom_ops() -> bool:
    """Define the two ops (idempotent).  Returns True once registered."""
    global _REGISTERED
    if _REGISTERED:
        return True
    try:
        getattr(torch.ops, _NAMESPACE).elastic_linear_packed
        _REGISTERED = True  # already defined in this process
        return True
    except (AttributeError, RuntimeError):
        pass

    op_packed = torch.library.custom_op(
        f"{_NAMESPACE}::elastic_linear_packed", mutates_args=(), device_types="cuda")(
            _elastic_linear_packed_impl)

    @op_packed.register_fake
    def _fake_packed(x, packed, scales, bias, bits, group_size, out_features, in_features):
        return x.new_empty((*x.shape[:-1], out_features))

    op_linear = torch.library.custom_op(
        f"{_NAMESPACE}::elastic_linear", mutates_args=(), device_types="cuda")(
            _elastic_linear_impl)

    @op_linear.register_fake
    def _fake_linear(x, matrix, out_features, bias):
        return x.new_empty((*x.shape[:-1], out_features))

    _REGISTERED = True
    return True


__all__ = ["register_native_custom_ops"]
