"""zq_matmul_noalloc -- the matmul entry point that allocates nothing.

Callers that cannot allocate device memory (or hand over a workspace) get
their scratch from a fixed array inside the library.  This file is collected
last on purpose, so a run that stops at the first failure has already run
every other test; it also passes on its own in a fresh process.  The check:
two calls in a row through the C ABI give exactly the same output as
zq_matmul with a caller workspace and as the oracle (the library's results
are bit-exact, so the tolerance is zero), and a request larger than the fixed
array is refused with a clear error.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qt,M,K,N", [(1, 1, 4096, 1000), (2, 8, 1000, 300), (1, 200, 1000, 300),
                                      (2, 130, 256, 520), (2, 512, 4096, 11008)])
def test_noalloc_matches_workspace_entry_point(cuda, qt, M, K, N):
    import torch

    import zyron_b200 as zb
    from zyron_b200 import _lib

    L = _lib.lib()
    rng = np.random.default_rng(100 + M + qt)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    pay, sc = O.quantize_weights(w, qt)
    W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
    bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).cuda()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    for call in range(2):  # two calls in a row, new inputs each time
        x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
        want = zb.matmul(x, W, bias=bias)
        got = torch.full((M, N), float("nan"), device="cuda")
        _lib.check(L.zq_matmul_noalloc(W.handle, C.c_void_p(x.data_ptr()), M, C.c_void_p(bias.data_ptr()),
                                       C.c_void_p(got.data_ptr()), sp))
        torch.cuda.synchronize()
        g = got.cpu().numpy().view(np.uint32)
        e = want.cpu().numpy().view(np.uint32)
        assert np.array_equal(g, e), f"call {call}: {(g != e).sum()} outputs differ from zq_matmul"
        o = O.matmul(x.cpu().numpy(), qt, pay, sc, N, bias.cpu().numpy())[3].view(np.uint32)
        assert np.array_equal(g, o), f"call {call}: {(g != o).sum()} outputs differ from the oracle"
    assert zb.device_error() == 0


def test_noalloc_rejects_oversize(cuda):
    import torch

    import zyron_b200 as zb
    from zyron_b200 import _lib

    L = _lib.lib()
    K, N = 4096, 64
    w = np.zeros((K, N), dtype=np.float32)
    pay, sc = O.quantize_weights(w, 1)
    W = zb.QuantizedMatrix.from_parts(1, K, N, sc, pay)
    M = 4096  # 4096 x 4096 codes = 16 MiB > the fixed array
    x = torch.zeros((M, K), device="cuda")
    y = torch.zeros((M, N), device="cuda")
    rc = L.zq_matmul_noalloc(W.handle, C.c_void_p(x.data_ptr()), M, None, C.c_void_p(y.data_ptr()), None)
    assert rc == _lib.ZQ_ERR_INVALID_ARGUMENT
    assert "zq_matmul_noalloc needs" in L.zq_last_error().decode()
