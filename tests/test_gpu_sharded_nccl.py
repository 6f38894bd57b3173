"""zq_matmul_sharded (the column-sharded matmul joined by an NCCL all-gather,
as a C entry point taking an ncclComm_t) on one GPU with a single-rank
communicator: the block matmul, the all-gather and the column join all run,
and the output must equal the oracle bit for bit.  The 2-GPU case with an
uneven split is in test_gpu_multi.py."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comm(cuda):
    import torch

    from zyron_b200.sharded import NcclComm

    c = NcclComm(torch.device("cuda", 0))
    yield c
    c.close()


@pytest.mark.parametrize("qt", [1, 2])
@pytest.mark.parametrize("M,K,N", [(1, 4096, 1000), (3, 129, 255), (6, 700, 129), (64, 512, 512), (300, 1000, 777)])
def test_sharded_single_rank_bit_exact(comm, qt, M, K, N):
    import torch

    import zyron_b200 as zb
    from zyron_b200.sharded import nccl_sharded_matmul

    rng = np.random.default_rng(M * 7 + K * 3 + N + qt)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    pay, sc = O.quantize_weights(w, qt)
    W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
    xd = torch.from_numpy(x).cuda()
    y = nccl_sharded_matmul(xd, W, N, comm, bias_shard=torch.from_numpy(b).cuda())
    torch.cuda.synchronize()
    want = O.matmul(x, qt, pay, sc, N, b)[3]
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert zb.device_error() == 0


def test_sharded_rejects_wrong_shard(comm):
    """A shard that is not this rank's zq_shard_range fails on the host,
    before any collective."""
    import torch

    import zyron_b200 as zb
    from zyron_b200 import _lib
    from zyron_b200.sharded import nccl_sharded_matmul

    W = zb.quantize(torch.randn(64, 32, device="cuda"), zb.Type.Int8)
    x = torch.randn(4, 64, device="cuda")
    with pytest.raises(_lib.ZQInvalidArgument, match=r"holds 32 columns, its shard of 40 is \[0, 40\)"):
        nccl_sharded_matmul(x, W, 40, comm)
    L = _lib.lib()
    y = torch.empty(4, 32, device="cuda")
    st = L.zq_matmul_sharded(W.handle, C.c_void_p(x.data_ptr()), 4, None, C.c_void_p(y.data_ptr()), 32, None, None,
                             0, None)
    assert st == 1 and b"null NCCL communicator" in L.zq_last_error()
