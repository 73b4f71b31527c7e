"""Tensor-parallel host logic on CPU: shard slicing and the row/column
orchestration over a 2-rank gloo group, with a stand-in compute (x @ W16^T in
float64 from the oracle's exact dequantised weight) in place of libebx."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlbricks_b200.elasticbit import tensor_parallel as tp
from oracle import oracle as O


@pytest.mark.parametrize("total,world,align", [(4096, 8, 16), (14336, 8, 64), (128256, 8, 16),
                                               (100, 3, 16), (384, 2, 64)])
def test_shard_bounds_cover_and_align(total, world, align):
    prev = 0
    for r in range(world):
        lo, hi = tp.shard_bounds(total, world, r, align)
        assert lo == prev and hi >= lo
        if r < world - 1:
            assert hi % align == 0
        prev = hi
    assert prev == total


@pytest.mark.parametrize("mode", tp.MODES)
def test_shard_codes_reassemble(mode):
    q = np.arange(64 * 192, dtype=np.int16).reshape(64, 192) % 200
    s = np.arange(64, dtype=np.float32) + 1
    parts = [tp.shard_codes(q, s, mode, 3, r) for r in range(3)]
    if mode == "column":
        assert np.array_equal(np.concatenate([p[0] for p in parts], axis=0), q)
        assert np.array_equal(np.concatenate([p[1] for p in parts]), s)
    else:
        assert np.array_equal(np.concatenate([p[0] for p in parts], axis=1), q)
        assert all(np.array_equal(p[1], s) for p in parts)


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, K, bits = 96, 256, 9
        w = O.baseline_weights(N, K, seed=1)
        s = O.row_scales(w, bits)
        q = O.quantize(w, s, bits)
        bias = torch.from_numpy(O.normal((N,), seed=2, scale=0.1))
        x = torch.from_numpy(O.normal((5, K), seed=3)).to(torch.float16)
        coll = tp.Collectives.from_group()
        out = {}
        for mode in tp.MODES:
            qs, ss, bounds = tp.shard_codes(q, s, mode, world, rank)
            w16 = torch.from_numpy(O.dequantize_codes(qs, ss).astype(np.float64))

            def local(xx, fp32, w16=w16):
                y = xx.double() @ w16.T
                return y.float() if fp32 else y.to(torch.float16)

            lin = tp.ShardedLinear(None, mode, N, K, bounds, bias=bias, collectives=coll,
                                   local=local, gather=True)
            out[mode] = lin(x).float().numpy()
        result_q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_row_and_column_parallel_match_unsharded_on_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q_out.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    N, K, bits = 96, 256, 9
    w = O.baseline_weights(N, K, seed=1)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    x = O.normal((5, K), seed=3).astype(np.float16)
    bias = O.normal((N,), seed=2, scale=0.1)
    ref = O.linear_full(x, O.dequantize_codes(q, s).astype(np.float32), bias)
    for rank in range(world):
        for mode in tp.MODES:
            y = results[rank][mode]
            assert y.shape == (5, N)
            rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
            assert rel < 1e-3, (mode, rel)
            assert np.abs(y - ref).max() <= max(2e-3, float(np.abs(np.spacing(ref.astype(np.float16))).max()))


def test_interleave_by8_layout_numpy_and_torch():
    from mlbricks_b200.elasticbit.tensor_parallel import interleave_by8

    g = np.arange(16 * 3).reshape(16, 3)
    u = -np.arange(16 * 3).reshape(16, 3)
    out = interleave_by8(g, u)
    assert out.shape == (32, 3)
    assert np.array_equal(out[0:8], g[0:8]) and np.array_equal(out[8:16], u[0:8])
    assert np.array_equal(out[16:24], g[8:16]) and np.array_equal(out[24:32], u[8:16])
    tout = interleave_by8(torch.from_numpy(g), torch.from_numpy(u))
    assert np.array_equal(tout.numpy(), out)
    s = interleave_by8(np.arange(8.0), np.arange(8.0) + 100)
    assert np.array_equal(s, np.concatenate([np.arange(8.0), np.arange(8.0) + 100]))
    with pytest.raises(ValueError):
        interleave_by8(np.zeros((12, 2)), np.zeros((12, 2)))


def test_swiglu_module_large_batch_deinterleaves():
    """M > 16 path: ebx_linear's fp32 sums on the interleaved matrix, activation in
    torch in fp32, one rounding to fp16."""
    from mlbricks_b200.elasticbit.tensor_parallel import SwiGLULinear, interleave_by8

    rng = np.random.default_rng(0)
    I, K, M = 24, 10, 20
    wg = rng.standard_normal((I, K)).astype(np.float32)
    wu = rng.standard_normal((I, K)).astype(np.float32)
    w = torch.from_numpy(interleave_by8(wg, wu))

    class Stand:
        def linear(self, x, bias=None, out32=False):
            y32 = x.float() @ w.T
            return (y32.half(), y32) if out32 else y32.half()

    mod = SwiGLULinear(Stand(), I, K)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32))
    y = mod(x)
    assert y.dtype == torch.float16
    g = x @ torch.from_numpy(wg).T
    u = x @ torch.from_numpy(wu).T
    assert torch.equal(y, (torch.nn.functional.silu(g) * u).half())


def _argmax_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vocab = 1000
        g = torch.Generator().manual_seed(3)
        logits = torch.randn((5, vocab), generator=g).half()
        # ties across a shard boundary and inside one shard: the lowest index must win
        lo0, hi0 = tp.shard_bounds(vocab, world, 0, 16)
        logits[1, hi0] = 9.0
        logits[1, hi0 - 1] = 9.0
        logits[2, 7] = 9.0
        logits[2, 3] = 9.0
        lo, hi = tp.shard_bounds(vocab, world, rank, 16)
        ids = tp.greedy_argmax(logits[:, lo:hi], lo, tp.Collectives.from_group())
        result_q.put((rank, ids.tolist(), logits.float().argmax(dim=-1).tolist()))
    finally:
        dist.destroy_process_group()


def test_greedy_argmax_over_column_shards():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_argmax_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, ids, ref in res:
        assert ids == ref
