"""Megatron-style tensor parallelism for compressed ElasticBit linears.

The reference has no distributed code; this module adds the multi-GPU form of
the same forward.  A matrix is compressed once, globally (bits, codes and row
scales are exactly the single-GPU ones), then sliced:

* ``column`` parallel (QKV, gate/up, lm_head): rank r keeps output rows
  [r*N/W, (r+1)*N/W) and their scales; no collective -- the output stays
  sharded along features (``gather=True`` all-gathers it);
* ``row`` parallel (O, down): rank r keeps input columns [r*K/W, (r+1)*K/W)
  and all row scales; each rank produces the fp32 partial sum over its K slice
  (libebx ``y32``), one all-reduce (sum, fp32) combines them, and the bias is
  added before the single fp16 rounding -- the same arithmetic as the unsharded
  kernel up to fp32 summation order.

Everything here is host orchestration; the per-rank compute is libebx
(``RuntimeMatrix.linear``).  The collective is pluggable (``allreduce`` /
``allgather`` callables) so the orchestration can be exercised with gloo ranks on
CPU and a stand-in compute function.

For decode-sized inputs (M <= 16) a row-parallel layer can skip the collective
altogether: with an :class:`Exchange` attached, one libebx call
(``ebx_linear_allreduce``) runs the shard's decode kernel, which stores its fp32
partials straight into every rank's exchange region over NVLink and sums all ranks'
partials in rank order.  Up to the exchange's ``max_m`` rows the shard's fp32 output
is summed the same way by ``ebx_exchange_allreduce`` instead of an NCCL all-reduce.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch

MODES = ("column", "row")


def shard_bounds(total: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """[lo, hi) of rank's slice; every interior boundary is a multiple of `align`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    units = -(-total // align)
    lo = (units * rank) // world * align
    hi = (units * (rank + 1)) // world * align
    return min(lo, total), min(hi, total)


def shard_codes(codes, scales, mode: str, world: int, rank: int):
    """Slice globally selected int16 codes [N, K] and fp32 scales [N] for one rank.

    Column shards are aligned to 16 rows (one row group), row shards to 64
    columns (one k-tile) so every shard keeps the device tile layout dense.
    Works on numpy arrays or torch tensors.
    """
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}")
    N, K = int(codes.shape[0]), int(codes.shape[1])
    if mode == "column":
        lo, hi = shard_bounds(N, world, rank, align=16)
        return codes[lo:hi], scales[lo:hi], (lo, hi)
    lo, hi = shard_bounds(K, world, rank, align=64)
    return codes[:, lo:hi], scales, (lo, hi)


@dataclass
class Collectives:
    """The two collectives a sharded linear needs (defaults: torch.distributed)."""
    allreduce: Callable[[torch.Tensor], None]
    allgather: Callable[[torch.Tensor], torch.Tensor]

    @staticmethod
    def from_group(group=None) -> "Collectives":
        import torch.distributed as dist

        def allreduce(t: torch.Tensor) -> None:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)

        def allgather(t: torch.Tensor) -> torch.Tensor:
            world = dist.get_world_size(group)
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t.contiguous(), group=group)
            return torch.cat(parts, dim=-1)

        return Collectives(allreduce, allgather)


class Exchange:
    """This rank's libebx tensor-parallel exchange (``ebx_exchange_*``).

    ``allgather_bytes(blob) -> [blob of rank 0, ..., blob of rank world-1]`` is the
    host transport for the opaque handles (``from_group`` uses torch.distributed).
    Close it only after every rank has finished its last exchange (a barrier):
    peers write into this rank's region until then.
    """

    def __init__(self, max_m: int, max_n: int, world: int, rank: int, device: int,
                 allgather_bytes: Callable[[bytes], list]) -> None:
        import ctypes

        from .. import _ebx

        self._lib = _ebx.load()
        self.max_m, self.max_n, self.world, self.rank = int(max_m), int(max_n), int(world), int(rank)
        blob = (ctypes.c_uint8 * _ebx.EXCHANGE_HANDLE_BYTES)()
        h = ctypes.c_void_p()
        _ebx.check(self._lib.ebx_exchange_create(world, rank, device, max_m, max_n, blob,
                                                 ctypes.byref(h)))
        self.handle = h
        blobs = allgather_bytes(bytes(blob))
        if len(blobs) != world or any(len(b) != _ebx.EXCHANGE_HANDLE_BYTES for b in blobs):
            self.close()
            raise RuntimeError("exchange handle all-gather returned malformed blobs")
        try:
            _ebx.check(self._lib.ebx_exchange_connect(h, b"".join(blobs)))
        except Exception:
            self.close()
            raise

    @staticmethod
    def from_group(max_m: int, max_n: int, group=None) -> "Exchange":
        import torch.distributed as dist

        world = dist.get_world_size(group)

        def allgather_bytes(b: bytes) -> list:
            out = [None] * world
            dist.all_gather_object(out, b, group=group)
            return out

        ex = Exchange(max_m, max_n, world, dist.get_rank(group), torch.cuda.current_device(),
                      allgather_bytes)
        dist.barrier(group)  # every rank has mapped every region before the first use
        return ex

    PROTOCOLS = {"auto": 0, "broadcast": 1, "two_phase": 2}

    def set_protocol(self, protocol: str) -> None:
        """Exchange protocol of this rank's later calls (``ebx_exchange_set_protocol``;
        every rank must choose the same): ``"auto"`` (two-phase once world x M >= 48),
        ``"broadcast"`` (every partial into every rank's region, one hop) or
        ``"two_phase"`` (each output's partials to one owner rank, which sums them and
        stores the sum into every other rank's region).  All give the same bits."""
        from .. import _ebx

        if protocol not in self.PROTOCOLS:
            raise ValueError(f"protocol must be one of {sorted(self.PROTOCOLS)}")
        _ebx.check(self._lib.ebx_exchange_set_protocol(self.handle, self.PROTOCOLS[protocol]))

    def allreduce(self, partial: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        """fp16(sum over ranks of `partial` + bias) for an fp32 [M, N] partial this rank
        holds (ebx_exchange_allreduce; M <= max_m, N <= max_n): one launch over NVLink
        peer memory instead of an NCCL all-reduce, summed in rank order on every rank."""
        from .. import _ebx

        part = partial.contiguous()
        M, N = (int(part.shape[0]), int(part.shape[1])) if part.dim() == 2 else (1, int(part.numel()))
        y = torch.empty(part.shape, dtype=torch.float16, device=part.device)
        b = None
        if bias is not None:
            b = bias.detach().to(device=part.device, dtype=torch.float16).contiguous()
        _ebx.check(self._lib.ebx_exchange_allreduce(self.handle, part.data_ptr(), M, N,
                                                    None if b is None else b.data_ptr(),
                                                    y.data_ptr(), None,
                                                    _ebx.stream_ptr(device=part.device.index)))
        return y

    def close(self) -> None:
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            self._lib.ebx_exchange_destroy(h)
            self.handle = None

    def __del__(self) -> None:  # pragma: no cover - interpreter teardown order
        try:
            self.close()
        except Exception:
            pass


class ShardedLinear(torch.nn.Module):
    """One rank's part of a tensor-parallel compressed linear.

    ``local`` computes y_local = x @ W_shard^T for the shard; by default it is
    the shard RuntimeMatrix's libebx call (fp32 partial for row mode).
    """

    def __init__(self, matrix, mode: str, out_features: int, in_features: int,
                 bounds: tuple[int, int], bias: torch.Tensor | None = None,
                 collectives: Collectives | None = None,
                 local: Callable[[torch.Tensor, bool], torch.Tensor] | None = None,
                 gather: bool = False, input_is_local: bool = False,
                 exchange: Exchange | None = None) -> None:
        super().__init__()
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        self.matrix = matrix
        self.mode = mode
        self.out_features = int(out_features)
        self.in_features = int(in_features)
        self.bounds = bounds
        self.gather = bool(gather)
        self.input_is_local = bool(input_is_local)  # row mode: x already holds this K slice
        self.collectives = collectives
        self.exchange = exchange  # row mode, M <= exchange.max_m: ebx_linear_allreduce
        self._local = local
        if bias is None:
            self.register_parameter("bias", None)
        else:
            b = bias.detach()
            if mode == "column":
                b = b[bounds[0]:bounds[1]]
            self.bias = torch.nn.Parameter(b.clone(), requires_grad=False)

    def _compute(self, x: torch.Tensor, fp32: bool, bias: torch.Tensor | None) -> torch.Tensor:
        if self._local is not None:
            y = self._local(x, fp32)
            if bias is not None:  # stand-in compute: bias before the single rounding
                y = (y.float() + bias.float()).to(y.dtype)
            return y
        native = getattr(self.matrix, "_native", self.matrix)
        if fp32:
            return native.linear(x, None, out32=True)[1]
        return native.linear(x, bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode == "column":
            if x.shape[-1] != self.in_features:
                raise ValueError(f"expected last dimension {self.in_features}")
            y = self._compute(x, False, self.bias)
            if self.gather:
                if self.collectives is None:
                    raise RuntimeError("column gather needs collectives")
                y = self.collectives.allgather(y)
            return y
        # row parallel: x is the full activation; use this rank's K slice
        lo, hi = self.bounds
        xs = x.contiguous() if self.input_is_local else x[..., lo:hi].contiguous()
        ex = self.exchange
        rows = xs.numel() // max(1, xs.shape[-1])
        if ex is not None and self._local is None and rows <= min(16, ex.max_m):
            native = getattr(self.matrix, "_native", self.matrix)
            return native.linear_allreduce(xs, ex, bias=self.bias)
        part = self._compute(xs, True, None)
        if ex is not None and self._local is None and rows <= ex.max_m and \
                self.out_features <= ex.max_n:
            y = ex.allreduce(part.reshape(rows, self.out_features), self.bias)
            return y.view(*part.shape)
        if self.collectives is not None:
            self.collectives.allreduce(part)
        if self.bias is not None:
            part = part + self.bias.float()
        return part.to(torch.float16)


def integer_width(bits: int) -> int:
    """Integer-code execution width for `bits`-bit codes (4, 8 or 12; 16 when the
    codes do not fit an exact fp16 operand)."""
    return 4 if bits <= 4 else 8 if bits <= 8 else 12 if bits <= 12 else 16


def _make_matrix(codes, scales, bits: int, threshold: float, error: float, decodePolicy: str,
                 integer: bool):
    """A shard's RuntimeMatrix.  integer=True pins the integer-code width (scale
    after accumulation) on every rank instead of letting each rank's own timing
    choose, so all ranks execute the same arithmetic."""
    from .core import RuntimeMatrix

    m = RuntimeMatrix._compressSelectedCodes(codes, scales, bits, threshold, error,
                                             decodePolicy="fullPrecision" if integer else decodePolicy)
    if integer:
        getattr(m, "_native", m)._pin_width(integer_width(bits), planner="tensorParallel")
    return m


def build_sharded(codes, scales, bits: int, mode: str, world: int, rank: int, *,
                  threshold: float = 0.0, error: float = 0.0, bias=None,
                  collectives: Collectives | None = None, gather: bool = False,
                  input_is_local: bool = False, exchange: Exchange | None = None,
                  decodePolicy: str = "fullPrecision", integer: bool = False) -> ShardedLinear:
    """Create this rank's shard (libebx matrix) from the global analyzer result."""
    N, K = int(codes.shape[0]), int(codes.shape[1])
    c, s, bounds = shard_codes(codes, scales, mode, world, rank)
    if torch.is_tensor(c):
        c = c.contiguous()
    else:
        c = np.ascontiguousarray(c)
    m = _make_matrix(c, s, bits, threshold, error, decodePolicy, integer)
    return ShardedLinear(m, mode, N, K, bounds, bias=bias, collectives=collectives, gather=gather,
                         input_is_local=input_is_local, exchange=exchange if mode == "row" else None)


def build_column_fused(parts, bits: int, world: int, rank: int, *, threshold: float = 0.0,
                       error: float = 0.0, decodePolicy: str = "fullPrecision",
                       integer: bool = False) -> ShardedLinear:
    """One column-parallel shard holding this rank's rows of several matrices that
    read the same input and share a storage width (gate and up; Q, K and V): the
    rank's slice of each part, concatenated along rows, so one decode launch serves
    them all.  The local output is [part 0 slice | part 1 slice | ...]."""
    cs, ss, widths = [], [], []
    K = int(parts[0][0].shape[1])
    for codes, scales in parts:
        if int(codes.shape[1]) != K:
            raise ValueError("fused column parts must share in_features")
        c, s, (lo, hi) = shard_codes(codes, scales, "column", world, rank)
        cs.append(c)
        ss.append(s)
        widths.append(hi - lo)
    if torch.is_tensor(cs[0]):
        c = torch.cat([t.contiguous() for t in cs], 0).contiguous()
        s = torch.cat([torch.as_tensor(t) for t in ss], 0).contiguous()
    else:
        c = np.ascontiguousarray(np.concatenate(cs, 0))
        s = np.ascontiguousarray(np.concatenate(ss, 0))
    m = _make_matrix(c, s, bits, threshold, error, decodePolicy, integer)
    lin = ShardedLinear(m, "column", int(c.shape[0]), K, (0, int(c.shape[0])))
    lin.part_widths = widths
    return lin


def interleave_by8(gate, up):
    """Rows of `gate` and `up` ([I, ...] each, I % 8 == 0) interleaved in blocks of 8:
    rows 16j..16j+7 = gate rows 8j..8j+7, rows 16j+8..16j+15 = up rows 8j..8j+7
    (the layout ebx_linear_swiglu reads).  numpy arrays or torch tensors."""
    n = int(gate.shape[0])
    if n % 8 or int(up.shape[0]) != n:
        raise ValueError("gate and up need the same row count, a multiple of 8")
    rest = tuple(gate.shape[1:])
    if torch.is_tensor(gate):
        return torch.stack([gate.reshape(n // 8, 8, *rest), up.reshape(n // 8, 8, *rest)], 1) \
            .reshape(2 * n, *rest).contiguous()
    g = np.asarray(gate).reshape(n // 8, 8, *rest)
    u = np.asarray(up).reshape(n // 8, 8, *rest)
    return np.ascontiguousarray(np.stack([g, u], 1).reshape(2 * n, *rest))


class SwiGLULinear(torch.nn.Module):
    """One rank's column-parallel gate/up pair with the SwiGLU activation fused:
    forward(x) = silu(x @ Wg_r^T) * (x @ Wu_r^T) over this rank's slice of the
    intermediate dimension.  Decode batches (<= 16 rows) run ebx_linear_swiglu (one
    launch, activation from the fp32 sums); larger batches run ebx_linear on the
    interleaved matrix (fp32 sums) and the activation in torch (fp32, one rounding)."""

    def __init__(self, matrix, width: int, in_features: int) -> None:
        super().__init__()
        self.matrix = matrix
        self.width = int(width)
        self.in_features = int(in_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        native = getattr(self.matrix, "_native", self.matrix)
        if x.numel() // x.shape[-1] <= 16:
            return native.linear_swiglu(x)
        # the fp32 sums, activation in fp32, one rounding (the fused kernel's arithmetic)
        y = native.linear(x, None, out32=True)[1].view(*x.shape[:-1], self.width // 8, 2, 8)
        return (torch.nn.functional.silu(y[..., 0, :]) * y[..., 1, :]).reshape(
            *x.shape[:-1], self.width).to(torch.float16)


def build_column_swiglu(gate, up, bits: int, world: int, rank: int, *, threshold: float = 0.0,
                        error: float = 0.0, decodePolicy: str = "fullPrecision",
                        integer: bool = False) -> SwiGLULinear:
    """This rank's column slice of a gate/up pair (global codes and scales each, same
    width) as one interleaved matrix with the SwiGLU activation fused."""
    (gc, gs), (uc, us) = gate, up
    K = int(gc.shape[1])
    cg, sg, (lo, hi) = shard_codes(gc, gs, "column", world, rank)
    cu, su, _ = shard_codes(uc, us, "column", world, rank)
    width = hi - lo
    c = interleave_by8(cg, cu)
    s = interleave_by8(sg if torch.is_tensor(sg) else np.asarray(sg),
                       su if torch.is_tensor(su) else np.asarray(su))
    m = _make_matrix(c, s, bits, threshold, error, decodePolicy, integer)
    return SwiGLULinear(m, width, K)


def greedy_argmax(local_logits: torch.Tensor, offset: int,
                  collectives: Collectives | None) -> torch.Tensor:
    """Greedy next-token ids from column-parallel logits: each rank reduces its
    vocabulary slice [offset, offset + width) to (max value, global index) per
    row, one all-gather exchanges those pairs, and every rank picks the largest
    value, the lowest index among equal values (torch.argmax's rule on the full
    logits; shards are in rank order, so the first maximum wins).  The indices
    travel as fp32, exact below 2^24 (the 128256-entry vocabulary fits)."""
    val, idx = local_logits.float().max(dim=-1)
    pair = torch.stack([val, (idx + int(offset)).float()], dim=-1)  # [M, 2]
    if collectives is None:
        return pair[..., 1].long()
    allp = collectives.allgather(pair)                                # [M, 2 * world]
    vals, ids = allp[..., 0::2], allp[..., 1::2]
    best = vals.argmax(dim=-1, keepdim=True)
    return ids.gather(-1, best).squeeze(-1).long()


__all__ = ["MODES", "shard_bounds", "shard_codes", "Collectives", "Exchange", "ShardedLinear",
           "build_sharded", "build_column_fused", "interleave_by8", "SwiGLULinear",
           "build_column_swiglu", "greedy_argmax", "integer_width"]
