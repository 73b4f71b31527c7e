"""ebx_analyze_noalloc: the width analysis for callers that cannot allocate
device memory (their memory is owned by a host framework's fixed pool, or they
must not trigger the synchronisation cudaMalloc/cudaFree can cause).

It must give the same results as ebx_analyze with a caller workspace, on
consecutive calls that reuse the library's fixed scratch array, and refuse
problems larger than that array.  Kept in the last-collected file so a run that
stops at its first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from mlbricks_b200 import _ebx
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_TOL = 1e-12  # the analyzer tests' bar against the reference goldens


def _analyze_with_workspace(lib, w, c):
    rows, cols = w.shape
    wd = torch.from_numpy(w).cuda()
    cd = torch.from_numpy(c).cuda()
    nws = int(lib.ebx_analyze_workspace_bytes(rows, c.shape[0]))
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    hw = torch.empty(14, dtype=torch.float64, device="cuda")
    full = torch.empty(14, dtype=torch.float64, device="cuda")
    _ebx.check(lib.ebx_analyze(wd.data_ptr(), rows, cols, cd.data_ptr(), c.shape[0],
                               hw.data_ptr(), full.data_ptr(), ws.data_ptr(), nws,
                               _ebx.stream_ptr()))
    torch.cuda.synchronize()
    return hw.cpu().numpy(), full.cpu().numpy()


def _analyze_noalloc(lib, w, c):
    rows, cols = w.shape
    wd = torch.from_numpy(w).cuda()
    cd = torch.from_numpy(c).cuda()
    hw = torch.empty(14, dtype=torch.float64, device="cuda")
    full = torch.empty(14, dtype=torch.float64, device="cuda")
    _ebx.check(lib.ebx_analyze_noalloc(wd.data_ptr(), rows, cols, cd.data_ptr(), c.shape[0],
                                       hw.data_ptr(), full.data_ptr(), _ebx.stream_ptr()))
    torch.cuda.synchronize()
    return hw.cpu().numpy(), full.cpu().numpy()


def _close(a, b):
    return np.all(np.abs(a - b) <= REL_TOL * np.maximum(np.abs(b), 1e-300))


def test_noalloc_matches_workspace_analyzer_on_consecutive_calls(cuda_ok):
    lib = _ebx.load()
    cases = [
        (O.baseline_weights(1536, 384, seed=0), O.normal((32, 384), seed=1)),
        (O.baseline_weights(96, 128, seed=5), O.normal((12, 128), seed=6)),
        (O.baseline_weights(1024, 512, seed=7), O.normal((32, 512), seed=8)),
    ]
    for w, c in cases:  # consecutive calls: the second reuses what the first left
        ref_hw, ref_full = _analyze_with_workspace(lib, w, c)
        for _ in range(2):
            hw, full = _analyze_noalloc(lib, w, c)
            assert _close(hw, ref_hw) and _close(full, ref_full)


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_ok):
    lib = _ebx.load()
    w = torch.zeros((16384, 64), dtype=torch.float32, device="cuda")
    c = torch.zeros((64, 64), dtype=torch.float32, device="cuda")
    out = torch.zeros(28, dtype=torch.float64, device="cuda")
    st = lib.ebx_analyze_noalloc(w.data_ptr(), 16384, 64, c.data_ptr(), 64, out.data_ptr(),
                                 out.data_ptr() + 14 * 8, _ebx.stream_ptr())
    assert st == _ebx.EBX_ERR_INVALID
    assert "scratch" in _ebx.last_error()
    assert torch.count_nonzero(out).item() == 0  # nothing was launched
