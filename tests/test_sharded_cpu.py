"""Host logic of the column-sharded matmul on CPU: world-size-2 gloo process
group, per-rank compute done by the oracle (the CUDA kernels are covered by
the GPU tests).  The gathered result must equal the single-process matmul
bit for bit, for even and uneven column splits."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from zyron_b200.sharded import assemble_columns, column_ranges


def test_column_ranges():
    assert column_ranges(8, 2) == [(0, 4), (4, 8)]
    assert column_ranges(7, 3) == [(0, 3), (3, 5), (5, 7)]
    assert column_ranges(65536, 8)[-1] == (57344, 65536)
    with pytest.raises(ValueError):
        column_ranges(3, 4)


def test_c_shard_range_matches_column_ranges():
    """zq_shard_range (the C entry point the NCCL sharded matmul checks
    shards against) splits exactly as column_ranges does; pure host code."""
    import ctypes as C

    from zyron_b200 import _lib

    L = _lib.lib()
    for n in (1, 2, 3, 7, 8, 100, 2047, 11008, 65536, 65537):
        for world in (1, 2, 3, 4, 5, 7, 8):
            if n < world:
                b, e = C.c_size_t(), C.c_size_t()
                assert L.zq_shard_range(n, world, 0, C.byref(b), C.byref(e)) == 1
                assert b"fewer columns than ranks" in L.zq_last_error()
                continue
            got = []
            for r in range(world):
                b, e = C.c_size_t(), C.c_size_t()
                assert L.zq_shard_range(n, world, r, C.byref(b), C.byref(e)) == 0
                got.append((b.value, e.value))
            assert got == column_ranges(n, world)
    b, e = C.c_size_t(), C.c_size_t()
    assert L.zq_shard_range(8, 2, 2, C.byref(b), C.byref(e)) == 1
    assert L.zq_shard_range(8, 0, 0, C.byref(b), C.byref(e)) == 1
    assert L.zq_matmul_sharded_workspace_bytes(None, 4, 8, 2) == 0


def test_assemble_columns():
    r = column_ranges(5, 2)
    blocks = [torch.arange(6.).reshape(2, 3), torch.arange(4.).reshape(2, 2) + 100]
    out = assemble_columns(blocks, r)
    assert out.tolist() == [[0, 1, 2, 100, 101], [3, 4, 5, 102, 103]]


class OracleShard:
    """Stand-in for a QuantizedMatrix shard on the CPU (test only)."""

    def __init__(self, qtype, K, payload_codes, scales):
        self.qtype, self.K, self.codes, self.scales = qtype, K, payload_codes, scales

    def cols(self):
        return self.scales.shape[0]


def oracle_matmul(x, shard, bias=None):
    from oracle import oracle as O

    N = shard.cols()
    # repack this shard's codes into the reference INT8 layout for the oracle
    payload = shard.codes.astype(np.int8).reshape(-1).view(np.uint8)
    y = O.matmul(x.numpy(), O.INT8, payload, shard.scales, N, None if bias is None else bias.numpy())[3]
    return torch.from_numpy(y)


def _worker(rank, world, port, n_cols, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from oracle import oracle as O
    from zyron_b200.sharded import column_ranges, sharded_matmul

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)
        K, M = 40, 6
        x = rng.standard_normal((M, K)).astype(np.float32)
        w = (rng.standard_normal((K, n_cols)) * 0.02).astype(np.float32)
        payload, scales = O.quantize_weights(w, O.INT8)
        codes = O.unpack_codes(O.INT8, payload, K, n_cols)  # [N][K]
        b, e = column_ranges(n_cols, world)[rank]
        shard = OracleShard(O.INT8, K, codes[b:e], scales[b:e])
        y = sharded_matmul(torch.from_numpy(x), shard, n_cols, matmul_fn=oracle_matmul)
        full = O.matmul(x, O.INT8, payload, scales, n_cols)[3]
        q.put((rank, bool(np.array_equal(y.numpy().view(np.uint32), full.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_cols", [8, 7])
def test_sharded_matmul_gloo_world2(n_cols):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_cols, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(2))
    assert results == {0: True, 1: True}
