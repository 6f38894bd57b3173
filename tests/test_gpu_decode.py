"""Decode-sized matmuls (M <= 16 activation rows) bit for bit against the
oracle, through both decode kernels: the tcgen05 kernel (weights streamed by
TMA, work split evenly over the SMs with exact int32 partial sums) and the
dp4a warp-per-column GEMV (M <= 8).

The shapes stress the split: N not a multiple of the 64-column block, K not
a multiple of the 128-code k-block, one column block shared by 64 CTAs,
blocks of a single k-block, more CTAs than column blocks, and more column
blocks than CTAs (shared pieces streamed first, whole blocks after, each
shared block finished by its latest share).
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TENSOR_CORE, CUDA_CORE = 1, 2

DECODE_SHAPES = [
    (1, 1, 1), (1, 64, 7), (1, 4096, 1000), (2, 31, 33), (3, 129, 255), (4, 8192, 64), (5, 1000, 300),
    (7, 12288, 129), (8, 4096, 1100), (8, 33, 1), (9, 200, 130), (12, 3000, 777), (16, 4096, 2048),
    (16, 100, 5000), (8, 4096, 11008), (2, 384, 20000),
]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def assert_bits_equal(got, want, what):
    g, w = bits(got), bits(want)
    if not np.array_equal(g, w):
        bad = np.argwhere(g != w)
        i = tuple(bad[0])
        raise AssertionError(f"{what}: {len(bad)} mismatches, first at {i}: got {got[i]!r} want {want[i]!r}")


@pytest.fixture(scope="module")
def zb(cuda):
    import zyron_b200

    return zyron_b200


def _case(M, K, N, qt):
    rng = np.random.default_rng(M * 1009 + K * 13 + N * 7 + qt)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    if M > 1:
        x[1] = 0.0
    if M > 2:
        x[2, 0] = np.nan
    if M > 3:
        x[3, K // 2] = np.inf
    b = rng.standard_normal(N).astype(np.float32)
    return x, w, b


@pytest.mark.parametrize("kernel", [TENSOR_CORE, CUDA_CORE])
@pytest.mark.parametrize("qt", [1, 2])
@pytest.mark.parametrize("M,K,N", DECODE_SHAPES)
def test_decode_matmul_bit_exact(zb, kernel, qt, M, K, N):
    import torch

    if kernel == CUDA_CORE and M > 8:
        pytest.skip("the dp4a GEMV serves M <= 8")
    x, w, b = _case(M, K, N, qt)
    pay, sc = O.quantize_weights(w, qt)
    W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
    W.set_decode_kernel(kernel)
    xd = torch.from_numpy(x).cuda()
    y = zb.matmul(xd, W).cpu().numpy()
    _, _, _, yo = O.matmul(x, qt, pay, sc, N)
    assert_bits_equal(y, yo, f"matmul t{qt} {M}x{K}x{N}")
    yb = zb.matmul(xd, W, bias=torch.from_numpy(b).cuda()).cpu().numpy()
    _, _, _, ybo = O.matmul(x, qt, pay, sc, N, b)
    assert_bits_equal(yb, ybo, f"linear t{qt} {M}x{K}x{N}")
    assert zb.device_error() == 0


@pytest.mark.parametrize("qt", [1, 2])
def test_decode_codes_entry_reuses_workspace(zb, qt):
    """zq_matmul_codes (no quantizer before it) clears the kernel's tickets
    itself; repeated calls on one workspace, with a different weight in
    between, stay exact."""
    import torch

    L = zb._lib.lib()
    M, K = 6, 5000
    cases = []
    for N in (700, 129):
        x, w, b = _case(M, K, N, qt)
        pay, sc = O.quantize_weights(w, qt)
        W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
        W.set_decode_kernel(TENSOR_CORE)
        _, _, _, yo = O.matmul(x, qt, pay, sc, N, b)
        cases.append((x, b, W, yo, N))
    need = max(L.zq_matmul_workspace_bytes(W.handle, M) for _, _, W, _, _ in cases)
    ws = torch.empty(need + 256, dtype=torch.uint8, device="cuda")
    ws_ptr = (ws.data_ptr() + 255) & ~255
    for rep in range(3):
        for x, b, W, yo, N in cases:
            Kp = L.zq_weight_padded_k(W.handle)
            xd = torch.from_numpy(x).cuda()
            codes = torch.empty((M, Kp), dtype=torch.int8, device="cuda")
            rs = torch.empty((M,), dtype=torch.float32, device="cuda")
            zb._lib.check(L.zq_quantize_rows(C.c_void_p(xd.data_ptr()), M, K, C.c_void_p(codes.data_ptr()), Kp,
                                             C.c_void_p(rs.data_ptr()), None))
            y = torch.empty((M, N), dtype=torch.float32, device="cuda")
            bd = torch.from_numpy(b).cuda()
            zb._lib.check(L.zq_matmul_codes(W.handle, C.c_void_p(codes.data_ptr()), C.c_void_p(rs.data_ptr()), M,
                                            C.c_void_p(bd.data_ptr()), C.c_void_p(y.data_ptr()), C.c_void_p(ws_ptr),
                                            need, None))
            assert_bits_equal(y.cpu().numpy(), yo, f"codes entry t{qt} N={N} rep {rep}")
    assert zb.device_error() == 0


@pytest.mark.parametrize("qt", [1, 2])
@pytest.mark.parametrize("M,K,N", [(1, 4096, 1000), (3, 1024, 300), (4, 512, 64)])
def test_fused_gemv_unaligned_rows(zb, qt, M, K, N):
    """The fused quantizer+GEMV reads activation rows as float4 when they
    start on 16-byte boundaries and element by element otherwise: x handed to
    zq_matmul one float past an aligned base takes the second path, with the
    same bits as the oracle."""
    import torch

    L = zb._lib.lib()
    x, w, b = _case(M, K, N, qt)
    pay, sc = O.quantize_weights(w, qt)
    W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
    W.set_decode_kernel(CUDA_CORE)
    buf = torch.zeros(M * K + 4, dtype=torch.float32, device="cuda")
    assert buf.data_ptr() % 16 == 0
    buf[1:1 + M * K] = torch.from_numpy(x.ravel()).cuda()
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    bd = torch.from_numpy(b).cuda()
    need = L.zq_matmul_workspace_bytes(W.handle, M)
    ws = torch.empty(need + 256, dtype=torch.uint8, device="cuda")
    ws_ptr = (ws.data_ptr() + 255) & ~255
    zb._lib.check(L.zq_matmul(W.handle, C.c_void_p(buf.data_ptr() + 4), M, C.c_void_p(bd.data_ptr()),
                              C.c_void_p(y.data_ptr()), C.c_void_p(ws_ptr), need, None))
    _, _, _, yo = O.matmul(x, qt, pay, sc, N, b)
    assert_bits_equal(y.cpu().numpy(), yo, f"unaligned x t{qt} {M}x{K}x{N}")
    assert zb.device_error() == 0


@pytest.mark.parametrize("qt", [1, 2])
def test_bounded_wait_timeout_reports_and_recovers(zb, qt):
    """A bounded device wait that runs out: the decode kernel's finishers wait
    for one partial sum more than exists (zq_test_decode_wait_timeout, limit
    2 ms).  The kernel records the timeout and returns; zq_device_error
    reports ZQ_ERR_DEVICE_TIMEOUT with code 5 once and clears it; the next
    normal call on the same workspace is bit-exact."""
    import torch

    from zyron_b200 import _lib

    L = zb._lib.lib()
    M, K, N = 8, 4096, 11008  # 172 column blocks over the SMs: many are split
    x, w, b = _case(M, K, N, qt)
    pay, sc = O.quantize_weights(w, qt)
    W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
    W.set_decode_kernel(TENSOR_CORE)
    Kp = L.zq_weight_padded_k(W.handle)
    xd = torch.from_numpy(x).cuda()
    codes = torch.empty((M, Kp), dtype=torch.int8, device="cuda")
    rs = torch.empty((M,), dtype=torch.float32, device="cuda")
    zb._lib.check(L.zq_quantize_rows(C.c_void_p(xd.data_ptr()), M, K, C.c_void_p(codes.data_ptr()), Kp,
                                     C.c_void_p(rs.data_ptr()), None))
    need = L.zq_matmul_workspace_bytes(W.handle, M)
    ws = torch.empty(need + 256, dtype=torch.uint8, device="cuda")
    ws_ptr = (ws.data_ptr() + 255) & ~255
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    assert zb.device_error() == 0
    zb._lib.check(L.zq_test_decode_wait_timeout(W.handle, C.c_void_p(codes.data_ptr()), C.c_void_p(rs.data_ptr()),
                                                M, C.c_void_p(y.data_ptr()), C.c_void_p(ws_ptr), need, 2_000_000,
                                                None))
    code = C.c_uint32()
    assert L.zq_device_error(None, C.byref(code)) == _lib.ZQ_ERR_DEVICE_TIMEOUT
    assert code.value == 5
    assert L.zq_device_error(None, C.byref(code)) == _lib.ZQ_OK and code.value == 0
    # the context is healthy and the same workspace serves a normal call
    for _ in range(2):
        zb._lib.check(L.zq_matmul_codes(W.handle, C.c_void_p(codes.data_ptr()), C.c_void_p(rs.data_ptr()), M, None,
                                        C.c_void_p(y.data_ptr()), C.c_void_p(ws_ptr), need, None))
        _, _, _, yo = O.matmul(x, qt, pay, sc, N)
        assert_bits_equal(y.cpu().numpy(), yo, f"after timeout t{qt}")
    assert zb.device_error() == 0
    # limits outside [1e5, 1e9] ns are refused on the host
    assert L.zq_test_decode_wait_timeout(W.handle, C.c_void_p(codes.data_ptr()), C.c_void_p(rs.data_ptr()), M,
                                         C.c_void_p(y.data_ptr()), C.c_void_p(ws_ptr), need, 2_000_000_000,
                                         None) == _lib.ZQ_ERR_INVALID_ARGUMENT
