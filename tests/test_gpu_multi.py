"""Column-sharded matmul with the all-gather fused into the epilogue, on 2
GPUs and on every visible GPU (one process per GPU, NCCL for the IPC-handle
exchange and the completion barrier).  Skipped when too few GPUs are
visible.  Each rank checks its full gathered output against the oracle, bit
for bit."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank(rank, world, port, q):
    import sys

    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import zyron_b200 as zb
    from oracle import oracle as O
    from zyron_b200.sharded import PeerOutputs, column_ranges, sharded_matmul_gathered

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        M, K, N = 640, 512, 2048
        rng = np.random.default_rng(11)
        x = rng.standard_normal((M, K)).astype(np.float32)
        w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        b, e = column_ranges(N, world)[rank]
        W = zb.quantize(torch.from_numpy(np.ascontiguousarray(w[:, b:e])).to(dev), zb.Type.Int8)
        out = PeerOutputs(M, N, dev)
        pay, sc = O.quantize_weights(w, O.INT8)  # per-column quantization: the shards' codes are the full matrix's
        xs = [x, rng.standard_normal((M, K)).astype(np.float32), rng.standard_normal((M, K)).astype(np.float32)]
        wants = [O.matmul(xi, O.INT8, pay, sc, N)[3] for xi in xs]
        # call 1, then call 2 issued before call 1's output is read: the
        # double-buffered outputs keep y1 intact while call 2 runs
        y1 = sharded_matmul_gathered(torch.from_numpy(xs[0]).to(dev), W, out)
        y2 = sharded_matmul_gathered(torch.from_numpy(xs[1]).to(dev), W, out)
        got1 = y1.cpu().numpy()
        got2 = y2.cpu().numpy()
        # call 3 reuses call 1's buffers
        y3 = sharded_matmul_gathered(torch.from_numpy(xs[2]).to(dev), W, out)
        got3 = y3.cpu().numpy()
        torch.cuda.synchronize(dev)
        ok = all(np.array_equal(g.view(np.uint32), wv.view(np.uint32)) for g, wv in zip((got1, got2, got3), wants))
        ok = ok and y3.data_ptr() == y1.data_ptr() and y2.data_ptr() != y1.data_ptr()
        q.put((rank, bool(ok), zb.device_error()))
        dist.barrier()
        out.close()
    finally:
        dist.destroy_process_group()


def _run_gathered(world):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    assert res == [(r, True, 0) for r in range(world)]


def test_gathered_matmul_two_gpus():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_gathered(2)


def test_gathered_matmul_all_gpus():
    """Every visible GPU (up to eight) as one rank: each rank's epilogue
    stores its columns into every peer's output."""
    import torch

    world = min(torch.cuda.device_count(), 8)
    if world < 3:
        pytest.skip("needs more than two GPUs")
    _run_gathered(world)


def _nccl_rank(rank, world, port, q):
    import sys

    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import zyron_b200 as zb
    from oracle import oracle as O
    from zyron_b200.sharded import NcclComm, column_ranges, nccl_sharded_matmul, shard_weight

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    comm = None
    try:
        comm = NcclComm(dev)
        ok = True
        for qt, M, K, N in ((1, 5, 700, 2047), (2, 300, 1000, 2047), (1, 1, 4096, 11008)):
            rng = np.random.default_rng(M + K + N + qt)
            x = rng.standard_normal((M, K)).astype(np.float32)
            w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
            bias = rng.standard_normal(N).astype(np.float32)
            pay, sc = O.quantize_weights(w, qt)
            W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
            shard = shard_weight(W, rank, world)
            b, e = column_ranges(N, world)[rank]
            y = nccl_sharded_matmul(torch.from_numpy(x).to(dev), shard, N, comm,
                                    bias_shard=torch.from_numpy(bias[b:e].copy()).to(dev))
            torch.cuda.synchronize(dev)
            want = O.matmul(x, qt, pay, sc, N, bias)[3]
            ok = ok and bool(np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32)))
        q.put((rank, ok, zb.device_error()))
        dist.barrier()
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_nccl_sharded_matmul_two_gpus():
    """zq_matmul_sharded over a 2-rank NCCL communicator, uneven split
    (2047 columns: 1024 + 1023), decode- and prefill-sized M, INT8 and INT4,
    with bias; every rank's full output equals the oracle bit for bit."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert res == [(0, True, 0), (1, True, 0)]
