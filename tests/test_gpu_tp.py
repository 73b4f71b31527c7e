"""Tensor-parallel shards on 2+ GPUs over NCCL (libebx compute per rank) vs the
unsharded matrix on one GPU.  Skipped when fewer than two GPUs are visible."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, q_out):
    import datetime

    import torch.distributed as dist

    from mlbricks_b200.elasticbit import tensor_parallel as tp
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        N, K, bits = 512, 4096, 10
        w = O.baseline_weights(N, K, seed=11)
        s = O.row_scales(w, bits)
        q = O.quantize(w, s, bits)
        bias = torch.from_numpy(O.normal((N,), seed=12, scale=0.1)).cuda()
        coll = tp.Collectives.from_group()
        res = {}
        for M in (1, 16, 100):
            x = torch.from_numpy(O.normal((M, K), seed=M).astype(np.float16)).cuda()
            for mode in tp.MODES:
                lin = tp.build_sharded(q, s, bits, mode, world, rank, bias=bias,
                                       collectives=coll, gather=True)
                res[(M, mode)] = lin(x).float().cpu().numpy()
        q_out.put((rank, res))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_matches_single_gpu(cuda_ok):
    import torch.multiprocessing as mp

    from mlbricks_b200 import RuntimeMatrix
    from oracle import oracle as O

    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs at least two GPUs")
    world = min(world, 8)
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q_out.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    N, K, bits = 512, 4096, 10
    w = O.baseline_weights(N, K, seed=11)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    bias = torch.from_numpy(O.normal((N,), seed=12, scale=0.1)).cuda().half()
    full = RuntimeMatrix._compressSelectedCodes(q, s, bits, 0.0, 0.0, decodePolicy="fullPrecision")
    for M in (1, 16, 100):
        x = torch.from_numpy(O.normal((M, K), seed=M).astype(np.float16)).cuda()
        ref = full.linear(x, bias).float().cpu().numpy()
        for rank in range(world):
            for mode in ("column", "row"):
                y = results[rank][(M, mode)]
                ulp = np.spacing(np.abs(ref.astype(np.float16))).astype(np.float32)
                assert np.all(np.abs(y - ref) <= np.maximum(2e-3, ulp)), (M, mode, rank)
                if mode == "column":
                    assert np.array_equal(y, ref)  # same kernel, same rows: bit-identical
