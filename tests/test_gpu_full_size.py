"""Parity at the workload sizes of the quantized-matmul benchmarks.

* INT8 M=64 K=512 N=512, INT4 M=128 K=2048 N=2048, and the decode GEMV
  M in {1, 8}, K=4096, N=11008 (INT8 and INT4): every output compared with
  the oracle bit for bit.
* The prefill GEMM M=8192 K=8192 N=65536 is too large for the oracle in
  full.  A row's activation codes depend only on that row, and an output
  column only on that column's codes and scale, so exact comparison on
  sampled rows x sampled column blocks is a complete check of those entries.
  The sample spans the first and last tiles in both dimensions and a random
  interior block.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("qt,M,K,N", [
    (1, 64, 512, 512),
    (2, 128, 2048, 2048),
    (1, 1, 4096, 11008), (1, 8, 4096, 11008),
    (2, 1, 4096, 11008), (2, 8, 4096, 11008),
])
def test_workload_shapes_exact(cuda, qt, M, K, N):
    import torch

    import zyron_b200 as zb

    rng = np.random.default_rng(1000 * qt + M)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    W = zb.quantize(torch.from_numpy(w).cuda(), zb.Type(qt))
    pay, sc = O.quantize_weights(w, qt)
    assert np.array_equal(W.payload(), pay)
    assert np.array_equal(bits(W.scales()), bits(sc))
    y = zb.matmul(torch.from_numpy(x).cuda(), W).cpu().numpy()
    yo = O.matmul(x, qt, pay, sc, N)[3]
    assert np.array_equal(bits(y), bits(yo))
    assert zb.device_error() == 0


def test_prefill_8192x8192x65536_sampled_exact(cuda):
    import torch

    import zyron_b200 as zb

    M, K, N = 8192, 8192, 65536
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    x = torch.randn((M, K), generator=g, device=dev)
    w = torch.randn((K, N), generator=g, device=dev).mul_(0.02)
    W = zb.quantize(w, zb.Type.Int8)
    del w
    torch.cuda.empty_cache()
    y = zb.matmul(x, W)
    assert zb.device_error() == 0

    rng = np.random.default_rng(9)
    rows = np.unique(np.concatenate([[0, 1, 127, 128, M - 1], rng.integers(0, M, 11)]))
    start = int(rng.integers(256, N - 768))
    col_blocks = [(0, 256), (start, start + 256), (N - 256, N)]
    xr = x[torch.from_numpy(rows).to(dev)].cpu().numpy()
    codes_r, scale_r = O.quantize_rows(xr)
    q_dev, s_dev = zb.quantize_rows(x[torch.from_numpy(rows).to(dev)])
    assert np.array_equal(q_dev.cpu().numpy(), codes_r)
    assert np.array_equal(bits(s_dev.cpu().numpy()), bits(scale_r))
    y_rows = y[torch.from_numpy(rows).to(dev)].cpu().numpy()
    for b, e in col_blocks:
        S = W.slice_cols(b, e)
        _, yo = O.matmul_codes(codes_r, scale_r, O.INT8, S.payload(), S.scales(), e - b)
        assert np.array_equal(bits(y_rows[:, b:e]), bits(yo)), (b, e)
