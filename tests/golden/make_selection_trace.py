"""Record the reference's model-path width selection as an ATen op trace.

The reference selects storage widths on the model's GPU with
``mlbricks.elasticbit.core._selectBitsTorch`` (core.py:112-195): thirteen rounds
of quantise, dequantise, two GEMMs and norms in torch.  Its results depend on
the GPU's arithmetic (cuBLAS GEMMs, the GPU's scalar division), so a golden file
written on a CPU would pin nothing.  This script instead imports that function
from the reference tree and runs it once on the host under a dispatch mode
that presents its inputs as CUDA tensors, executes every ATen operation on the
CPU, and records the operation sequence: the op overload, its arguments
(tensor references, shapes, dtypes, scalars) and which tensors it produced.
The trace is the reference's own computation, with no restatement in between;
``tests/test_ref_selection_trace.py`` replays it on a B200 and compares the
widths, errors, codes and scales with ``mlbricks_b200``'s ``_selectBitsTorch``.

Threshold 0 makes every width fail (a relative error is never exactly 0 for
these inputs), so one trace covers all thirteen candidate widths; the
selection rule itself (smallest width whose max(hardware, full) error is within
the threshold) is applied to the replayed errors at any threshold.

Usage (build container, repo root):
    python tests/golden/make_selection_trace.py MLBRICKS_TREE
writes tests/golden/selection_trace_{N}x{K}_s{S}.json for the traced shapes.
"""
from __future__ import annotations

import importlib
import json
import sys
from pathlib import Path

import numpy as np
import torch
from torch.utils._python_dispatch import TorchDispatchMode

HERE = Path(__file__).resolve().parent

# (rows N, cols K, calibration rows S): BASELINE config 1 (nn.Linear 384 -> 1536, 32 of
# its calibration rows reach the analyzer) and one config-2 decode matrix (4096 x 4096)
SHAPES = [(1536, 384, 32), (4096, 4096, 32)]


class _Cuda(torch.Tensor):
    """A host tensor whose `device` reads cuda (the reference checks it); its
    real device stays the host's, so no device guard reaches for a GPU."""

    @staticmethod
    def __new__(cls, elem: torch.Tensor, tid: int):
        r = torch.Tensor._make_wrapper_subclass(cls, elem.shape, strides=elem.stride(),
                                                dtype=elem.dtype, device="cpu",
                                                requires_grad=False)
        r.elem = elem
        r.tid = tid
        return r

    @property
    def device(self) -> torch.device:  # what the traced Python code sees
        return torch.device("cuda")

    __torch_function__ = torch._C._disabled_torch_function_impl

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):  # pragma: no cover
        raise RuntimeError("tensors of the trace run only under the recorder")


class Recorder(TorchDispatchMode):
    def __init__(self) -> None:
        super().__init__()
        self.ops: list[dict] = []
        self.inputs: dict[int, str] = {}  # id(host tensor) -> input name
        self._keep: list[torch.Tensor] = []
        self._next = 0
        self.expect_calibration: tuple[int, int] | None = None

    def new_id(self) -> int:
        self._next += 1
        return self._next

    def wrap(self, t: torch.Tensor) -> _Cuda:
        return _Cuda(t, self.new_id())

    def input(self, t: torch.Tensor, name: str) -> None:
        self.inputs[id(t)] = name
        self._keep.append(t)

    def _enc(self, v):
        if isinstance(v, _Cuda):
            return {"t": v.tid}, v.elem
        if isinstance(v, torch.Tensor):
            if id(v) in self.inputs:
                return {"in": self.inputs[id(v)]}, v
            if v.dim() == 0:  # a Python number the dispatcher wrapped as a host scalar tensor
                return {"scalar_tensor": repr(v.item()), "dtype": str(v.dtype).replace("torch.", "")}, v
            if self.expect_calibration is not None and tuple(v.shape) == self.expect_calibration \
                    and v.dtype == torch.float32 and "calibration" not in self.inputs.values():
                # the host copy of the calibration matrix (torch.from_numpy in the reference)
                self.input(v, "calibration")
                return {"in": "calibration"}, v
            raise RuntimeError("untraced host tensor entered the computation")
        if isinstance(v, torch.dtype):
            return {"dtype": str(v).replace("torch.", "")}, v
        if isinstance(v, torch.device):
            return {"device": v.type}, torch.device("cpu")
        if isinstance(v, (torch.layout, torch.memory_format)):
            return {"enum": str(v).replace("torch.", "")}, v
        if isinstance(v, (list, tuple)):
            pairs = [self._enc(x) for x in v]
            return {"seq": [p[0] for p in pairs]}, type(v)(p[1] for p in pairs)
        if isinstance(v, float):
            return {"f": repr(v)}, v
        if isinstance(v, (bool, int, str)) or v is None:
            return {"v": v}, v
        raise TypeError(f"cannot record argument of type {type(v).__name__}")

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        enc_args, run_args = zip(*[self._enc(a) for a in args]) if args else ((), ())
        enc_kw, run_kw = {}, {}
        for k, v in kwargs.items():
            enc_kw[k], run_kw[k] = self._enc(v)
        out = func(*run_args, **run_kw)
        entry = {"op": str(func), "args": list(enc_args), "kwargs": enc_kw}
        if isinstance(out, torch.Tensor):
            w = self.wrap(out)
            entry["out"] = [w.tid]
            self.ops.append(entry)
            return w
        if isinstance(out, (list, tuple)) and all(isinstance(o, torch.Tensor) for o in out):
            ws = [self.wrap(o) for o in out]
            entry["out"] = [w.tid for w in ws]
            self.ops.append(entry)
            return type(out)(ws)
        entry["scalar"] = True  # aten._local_scalar_dense: a value read by the host
        self.ops.append(entry)
        return out


def trace(select_bits, rows: int, cols: int, samples: int) -> dict:
    rec = Recorder()
    # any non-degenerate values: the recorded operations do not depend on them
    # (threshold 0 keeps every width's branch the same)
    g = torch.Generator().manual_seed(0)
    calib = torch.randn((samples, cols), generator=g).numpy()
    with torch.inference_mode():  # the reference function runs in inference mode
        w = rec.wrap((0.02 * torch.randn((rows, cols), generator=g)).half())
    rec.expect_calibration = (samples, cols)
    # Tensor.to(device="cuda") initialises CUDA before dispatching; nothing here
    # touches a GPU (the recorder runs every op on the host), so skip that step
    lazy_init = torch.cuda._lazy_init
    torch.cuda._lazy_init = lambda: None
    try:
        with rec:
            bits, err, codes, scales = select_bits(w, calib, 0.0)
    finally:
        torch.cuda._lazy_init = lazy_init
    assert bits == 16 and codes is None, "threshold 0 must run every width"
    return {"rows": rows, "cols": cols, "samples": samples, "weight_tid": w.tid,
            "ops": rec.ops}


def main(tree: str) -> None:
    sys.path.insert(0, str(Path(tree).resolve()))
    ref_core = importlib.import_module("mlbricks.elasticbit.core")
    for rows, cols, samples in SHAPES:
        t = trace(ref_core._selectBitsTorch, rows, cols, samples)
        t["source"] = ("mlbricks/elasticbit/core.py:_selectBitsTorch (core.py:112-195), "
                       "recorded by tests/golden/make_selection_trace.py")
        out = HERE / f"selection_trace_{rows}x{cols}_s{samples}.json"
        out.write_text(json.dumps(t, separators=(",", ":")) + "\n")
        n_scalar = sum(1 for op in t["ops"] if op.get("scalar"))
        print(f"wrote {out.name}: {len(t['ops'])} ops, {n_scalar} host reads")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_selection_trace.py MLBRICKS_TREE")
    main(sys.argv[1])
