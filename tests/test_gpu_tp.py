"""Tensor-parallel shards on 2+ GPUs (one process per GPU, NCCL for the host
plumbing, libebx compute) against the unsharded matrix on one GPU, for both
all-reduce routes of row-parallel layers: NCCL over fp32 partials, and the
libebx exchange (ebx_linear_allreduce).  Also: a rank that never joins an
exchange makes the others' finish kernel give up after its bounded wait and
report it through ebx_device_status, with the CUDA context still usable.
Skipped when fewer than two GPUs are visible."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPE = (512, 4096, 10)  # N, K, bits
MS = (1, 5, 16, 100)


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _case():
    from oracle import oracle as O

    N, K, bits = SHAPE
    w = O.baseline_weights(N, K, seed=11)
    s = O.row_scales(w, bits)
    q = O.quantize(w, s, bits)
    bias = O.normal((N,), seed=12, scale=0.1).astype(np.float16)
    xs = {M: O.normal((M, K), seed=M).astype(np.float16) for M in MS}
    return q, s, bits, bias, xs


def _init(rank, world, port):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return dist


def _worker(rank, world, port, q_out):
    dist = _init(rank, world, port)
    from mlbricks_b200.elasticbit import tensor_parallel as tp

    try:
        q, s, bits, bias, xs = _case()
        bias_t = torch.from_numpy(bias).cuda()
        coll = tp.Collectives.from_group()
        ex = tp.Exchange.from_group(128, 4096)  # M <= 16: fused decode; 16 < M <= 128: allreduce
        res = {}
        lin = {mode: tp.build_sharded(q, s, bits, mode, world, rank, bias=bias_t,
                                      collectives=coll, gather=True) for mode in tp.MODES}
        lin_x = tp.build_sharded(q, s, bits, "row", world, rank, bias=bias_t, collectives=coll,
                                 exchange=ex)
        for M in MS:
            x = torch.from_numpy(xs[M]).cuda()
            for mode in tp.MODES:
                res[(M, mode)] = lin[mode](x).float().cpu().numpy()
            for rep in range(3):  # successive epochs
                res[(M, "exchange", rep)] = lin_x(x).float().cpu().numpy()
            for protocol in ("broadcast", "two_phase"):  # both protocols, forced
                ex.set_protocol(protocol)
                res[(M, protocol)] = lin_x(x).float().cpu().numpy()
            ex.set_protocol("auto")
        torch.cuda.synchronize()
        import ctypes

        from mlbricks_b200 import _ebx
        lib = _ebx.load()
        v = ctypes.c_int32()
        _ebx.check(lib.ebx_device_status(rank, ctypes.byref(v), 0))
        res["status"] = int(v.value)
        dist.barrier()
        ex.close()
        q_out.put((rank, res))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _unsharded_reference():
    from mlbricks_b200 import RuntimeMatrix

    q, s, bits, bias, xs = _case()
    full = RuntimeMatrix._compressSelectedCodes(q, s, bits, 0.0, 0.0, decodePolicy="fullPrecision")
    b = torch.from_numpy(bias).cuda()
    return {M: full.linear(torch.from_numpy(xs[M]).cuda(), b).float().cpu().numpy() for M in MS}


def _spawn(target, world, timeout=300):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q_out.get(timeout=timeout) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


def test_tensor_parallel_matches_single_gpu(cuda_ok):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    results = _spawn(_worker, world)
    ref = _unsharded_reference()
    for M in MS:
        r16 = ref[M].astype(np.float16)
        tol = np.maximum(2e-3, np.spacing(np.abs(r16)).astype(np.float32))
        for rank in range(world):
            res = results[rank]
            assert res["status"] == 0
            for mode in ("column", "row"):
                y = res[(M, mode)]
                assert np.all(np.abs(y - ref[M]) <= tol), (M, mode, rank)
                if mode == "column":  # every rank gathers the same shards
                    assert np.array_equal(y, results[0][(M, mode)])
            if M <= 128:  # fused decode exchange (M <= 16) or ebx_exchange_allreduce
                y0 = res[(M, "exchange", 0)]
                assert np.all(np.abs(y0 - ref[M]) <= tol), (M, "exchange", rank)
                for rep in (1, 2):
                    assert np.array_equal(res[(M, "exchange", rep)], y0)
                # rank-order summation: every rank holds the same bits
                assert np.array_equal(y0, results[0][(M, "exchange", 0)])
                # broadcast and two-phase add the same words in the same order
                assert np.array_equal(res[(M, "broadcast")], y0)
                assert np.array_equal(res[(M, "two_phase")], y0)


SEQ_MS = (16, 1, 8, 1, 5, 16, 2, 16)  # back-to-back exchange calls of changing M
# and of changing protocol (every rank switches the same way before each call)
SEQ_PROTOCOLS = ("two_phase", "broadcast", "two_phase", "two_phase", "auto", "broadcast",
                 "two_phase", "auto")


def _seq_inputs():
    from oracle import oracle as O

    _, K, _ = SHAPE
    return [O.normal((M, K), seed=200 + i).astype(np.float16) for i, M in enumerate(SEQ_MS)]


def _sequence_worker(rank, world, port, q_out):
    """Exchange calls with a different M each, issued without any host
    synchronisation in between; every rank but 0 sleeps on the host before
    each launch, so rank 0 runs ahead and pushes the partials of call E + 1
    while its peers still read those of call E -- with the broadcast and the
    two-phase protocol mixed from call to call."""
    import ctypes
    import time

    dist = _init(rank, world, port)
    from mlbricks_b200 import _ebx
    from mlbricks_b200.elasticbit import tensor_parallel as tp

    try:
        q, s, bits, bias, _ = _case()
        bias_t = torch.from_numpy(bias).cuda()
        ex = tp.Exchange.from_group(16, 4096)
        lin = tp.build_sharded(q, s, bits, "row", world, rank, bias=bias_t, exchange=ex)
        xs = [torch.from_numpy(x).cuda() for x in _seq_inputs()]
        torch.cuda.synchronize()
        dist.barrier()
        outs = []
        for x, protocol in zip(xs, SEQ_PROTOCOLS):
            if rank != 0:
                time.sleep(0.05)
            ex.set_protocol(protocol)
            outs.append(lin(x))
        torch.cuda.synchronize()
        res = {"y": [o.float().cpu().numpy() for o in outs]}
        lib = _ebx.load()
        v = ctypes.c_int32()
        _ebx.check(lib.ebx_device_status(rank, ctypes.byref(v), 0))
        res["status"] = int(v.value)
        dist.barrier()
        ex.close()
        q_out.put((rank, res))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_exchange_back_to_back_changing_m(cuda_ok):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    results = _spawn(_sequence_worker, world)
    from mlbricks_b200 import RuntimeMatrix

    q, s, bits, bias, _ = _case()
    full = RuntimeMatrix._compressSelectedCodes(q, s, bits, 0.0, 0.0, decodePolicy="fullPrecision")
    b = torch.from_numpy(bias).cuda()
    for i, x in enumerate(_seq_inputs()):
        ref = full.linear(torch.from_numpy(x).cuda(), b).float().cpu().numpy()
        tol = np.maximum(2e-3, np.spacing(np.abs(ref.astype(np.float16))).astype(np.float32))
        for rank in range(world):
            assert results[rank]["status"] == 0, rank
            y = results[rank]["y"][i]
            assert np.all(np.abs(y - ref) <= tol), (i, SEQ_MS[i], rank)
            assert np.array_equal(y, results[0]["y"][i])


def _absent_rank_worker(rank, world, port, q_out):
    dist = _init(rank, world, port)
    import ctypes

    from mlbricks_b200 import _ebx
    from mlbricks_b200.elasticbit import tensor_parallel as tp

    try:
        q, s, bits, bias, xs = _case()
        ex = tp.Exchange.from_group(16, 4096)
        lin = tp.build_sharded(q, s, bits, "row", world, rank, exchange=ex)
        out = {}
        lib = _ebx.load()
        v = ctypes.c_int32()
        if rank == 0:
            # ranks >= 1 never join this exchange: the finish kernel's bounded wait
            # (about 2 s) gives up and records the failure
            x = torch.from_numpy(xs[1]).cuda()
            lin(x)
            torch.cuda.synchronize()
            _ebx.check(lib.ebx_device_status(rank, ctypes.byref(v), 1))
            out["status"] = int(v.value)
            # the context is still usable: a plain launch works and the status is clear
            y = lin.matrix.linear(x[:, : lin.bounds[1] - lin.bounds[0]].contiguous())
            torch.cuda.synchronize()
            out["after"] = bool(torch.isfinite(y.float()).all().item())
            _ebx.check(lib.ebx_device_status(rank, ctypes.byref(v), 0))
            out["status_after"] = int(v.value)
        dist.barrier()
        ex.close()  # out of step now: discarded, as the header says
        q_out.put((rank, out))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_exchange_reports_absent_rank(cuda_ok):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    results = _spawn(_absent_rank_worker, 2)
    assert results[0]["status"] == 0x7102
    assert results[0]["after"] and results[0]["status_after"] == 0
