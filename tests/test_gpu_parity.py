"""GPU parity of the CUDA path against the oracle, through the C ABI.

Integer work (activation codes, weight codes, payloads) and the fp32 outputs
are compared BIT FOR BIT: the CUDA epilogue evaluates the reference's
float(acc) * s_row * s_col (+ bias) with the same three roundings, so any
difference is a bug.  The oracle (oracle/zq_oracle.c) is itself pinned to the
reference by tests/test_oracle.py.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def assert_bits_equal(got, want, what):
    g, w = bits(got), bits(want)
    if not np.array_equal(g, w):
        bad = np.argwhere(g != w)
        i = tuple(bad[0])
        raise AssertionError(f"{what}: {len(bad)} mismatches, first at {i}: got {got[i]!r} want {want[i]!r}")


def make(rng, M, K, N, edge=True):
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    if edge:
        if M > 1:
            x[1] = 0.0
        if M > 2:
            x[2, 0] = np.nan
        if M > 3:
            x[3, K // 2] = np.inf
        if N > 2:
            w[:, 1] = 0.0
    return x, w


@pytest.fixture(scope="module")
def zb(cuda):
    import zyron_b200

    return zyron_b200


def test_golden_vectors_through_cuda(zb, golden):
    import torch

    for ci, (M, K, N) in enumerate(golden["shapes"]):
        M, K, N = int(M), int(K), int(N)
        x = torch.from_numpy(golden[f"c{ci}_x"]).cuda()
        bias = torch.from_numpy(golden[f"c{ci}_bias"]).cuda()
        for qt in (1, 2):
            p = f"c{ci}_t{qt}"
            W = zb.QuantizedMatrix.from_parts(qt, K, N, golden[p + "_scales"], golden[p + "_payload"])
            assert_bits_equal(zb.matmul(x, W).cpu().numpy(), golden[p + "_y"], p + " matmul")
            assert_bits_equal(zb.matmul(x, W, bias=bias).cpu().numpy(), golden[p + "_ylin"], p + " linear")
            assert_bits_equal(W.dequantize().cpu().numpy(), golden[p + "_deq"], p + " dequantize")
            assert W.save_bytes() == golden[p + "_zyq"].tobytes(), p + " save"
            W2 = zb.QuantizedMatrix.load_bytes(golden[p + "_zyq"].tobytes())
            assert np.array_equal(W2.payload(), golden[p + "_payload"])
            # device quantize() == reference quantize()
            Wq = zb.quantize(torch.from_numpy(golden[f"c{ci}_w"]).cuda(), zb.Type(qt))
            assert np.array_equal(Wq.payload(), golden[p + "_payload"]), p + " device quantize payload"
            assert_bits_equal(Wq.scales(), golden[p + "_scales"], p + " device quantize scales")
    assert zb.device_error() == 0


@pytest.mark.parametrize("M,K", [(1, 1), (3, 17), (8, 4096), (37, 1000), (300, 2048), (2, 3)])
def test_quantize_rows_bit_exact(zb, M, K):
    import torch

    rng = np.random.default_rng(M * 7 + K)
    x, _ = make(rng, M, K, 1)
    if M > 4:
        x[4] = np.float32(1e-45) * rng.integers(-3, 4, K)  # denormals
    if M > 5 and K > 3:
        x[5] = 0.5
        x[5, 0] = 127.0
        x[5, 1] = -2.5
        x[5, 2] = 3.5
    q, s = zb.quantize_rows(torch.from_numpy(x).cuda())
    qo, so = O.quantize_rows(x)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert_bits_equal(s.cpu().numpy(), so, "row scales")


def _near_tie_rows(rng, M, K):
    """Rows whose quotients x / s sit within a few ulps of half-integers, where
    the kernels' multiply-by-reciprocal fast path must hand over to the exact
    division: each row's absmax fixes s = absmax / 127 (not a power of two),
    and the other values are (k + 1/2) * s, k in [-127, 126), moved by -3..3
    ulps; +-absmax give quotients at the clamp."""
    x = np.empty((M, K), dtype=np.float32)
    for r in range(M):
        amax = np.float32(rng.uniform(0.5, 300.0))
        s = np.float32(amax / np.float32(127.0))
        k = rng.integers(-127, 126, K).astype(np.float32) + np.float32(0.5)
        v = (k * s).astype(np.float32)
        nudge = rng.integers(-3, 4, K)
        toward = np.where(nudge > 0, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
        for step in range(3):
            v = np.where(np.abs(nudge) > step, np.nextafter(v, toward), v).astype(np.float32)
        v[0] = amax
        if K > 1:
            v[1] = -amax
        x[r] = v
    return x


@pytest.mark.parametrize("M,K", [(1, 4096), (4, 1000), (64, 3072)])
def test_quantize_near_ties_bit_exact(zb, M, K):
    """Near-tie quotients through the standalone quantizer, the 1-4-row GEMV
    that quantizes its rows itself, the GEMM path and the device weight
    quantizer, against the oracle."""
    import torch

    rng = np.random.default_rng(9000 + M + K)
    x = _near_tie_rows(rng, M, K)
    q, s = zb.quantize_rows(torch.from_numpy(x).cuda())
    qo, so = O.quantize_rows(x)
    assert np.array_equal(q.cpu().numpy(), qo), f"{(q.cpu().numpy() != qo).sum()} codes differ"
    assert_bits_equal(s.cpu().numpy(), so, "row scales")
    w = (rng.standard_normal((K, 96)) * 0.02).astype(np.float32)
    for qt in (1, 2):
        pay, sc = O.quantize_weights(w, qt)
        W = zb.QuantizedMatrix.from_parts(qt, K, 96, sc, pay)
        y = zb.matmul(torch.from_numpy(x).cuda(), W).cpu().numpy()
        assert_bits_equal(y, O.matmul(x, qt, pay, sc, 96)[3], f"matmul t{qt}")
        # the same values as weights: columns of x.T, device quantize()
        wt = np.ascontiguousarray(x.T)
        Wq = zb.quantize(torch.from_numpy(wt).cuda(), zb.Type(qt))
        pay_o, sc_o = O.quantize_weights(wt, qt)
        assert np.array_equal(Wq.payload(), pay_o), f"device quantize payload t{qt}"
        assert_bits_equal(Wq.scales(), sc_o, f"device quantize scales t{qt}")
    assert zb.device_error() == 0


SHAPES = [
    # decode GEMV sizes (M <= 8)
    (1, 64, 7), (1, 4096, 1000), (2, 31, 33), (3, 129, 255), (5, 1000, 300), (8, 4096, 1100), (8, 33, 1),
    # tcgen05 GEMM sizes: ragged M / N / K around the 128 x {64,128,256} tiles
    (9, 64, 130), (64, 512, 512), (127, 256, 64), (128, 128, 256), (129, 384, 257), (200, 1000, 100),
    (256, 2048, 520), (300, 17, 33), (513, 640, 1024), (1024, 256, 4096),
]


@pytest.mark.parametrize("qt", [1, 2])
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_matmul_bit_exact(zb, qt, M, K, N):
    import torch

    rng = np.random.default_rng(M * 131 + K * 7 + N + qt)
    x, w = make(rng, M, K, N)
    b = rng.standard_normal(N).astype(np.float32)
    pay, sc = O.quantize_weights(w, qt)
    W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
    xd = torch.from_numpy(x).cuda()
    y = zb.matmul(xd, W).cpu().numpy()
    _, _, _, yo = O.matmul(x, qt, pay, sc, N)
    assert_bits_equal(y, yo, f"matmul t{qt} {M}x{K}x{N}")
    yb = zb.matmul(xd, W, bias=torch.from_numpy(b).cuda()).cpu().numpy()
    _, _, _, ybo = O.matmul(x, qt, pay, sc, N, b)
    assert_bits_equal(yb, ybo, f"linear t{qt} {M}x{K}x{N}")
    assert zb.device_error() == 0


@pytest.mark.parametrize("qt", [1, 2])
def test_zero_rows(zb, qt):
    """An input with no rows gives an empty [0, N] output, as the
    reference's matmul does (its row loop runs zero times); device and host
    inputs both."""
    import torch

    K, N = 64, 48
    _, w = make(np.random.default_rng(5), 1, K, N)
    pay, sc = O.quantize_weights(w, qt)
    W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
    yo = O.matmul(np.zeros((0, K), np.float32), qt, pay, sc, N)[3]
    assert yo.shape == (0, N)
    y = zb.matmul(torch.empty((0, K), device="cuda"), W)
    assert tuple(y.shape) == (0, N)
    assert zb.matmul(np.zeros((0, K), np.float32), W).shape == (0, N)
    assert zb.device_error() == 0


@pytest.mark.parametrize("qt", [1, 2])
def test_host_entry_point(zb, qt):
    rng = np.random.default_rng(11 + qt)
    for M, K, N in [(1, 300, 70), (40, 96, 130)]:
        x, w = make(rng, M, K, N)
        b = rng.standard_normal(N).astype(np.float32)
        pay, sc = O.quantize_weights(w, qt)
        W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
        assert_bits_equal(zb.matmul(x, W, bias=b), O.matmul(x, qt, pay, sc, N, b)[3], "host matmul")
        # rank-3 input keeps its leading dims (quantization.cpp:192-196)
        y3 = zb.matmul(x.reshape(1, M, K), W)
        assert y3.shape == (1, M, N)


def test_quantized_linear_mirror(zb):
    """Mirror of the reference's test_quantized_linear (tests/test_phase5.cpp:129-155),
    with the tolerance check replaced by bit-exact comparison to the oracle."""
    import torch

    rng = np.random.default_rng(31)
    weight = rng.uniform(-0.5, 0.5, (16, 8)).astype(np.float32)
    bias = rng.uniform(-0.2, 0.2, 8).astype(np.float32)
    inp = rng.uniform(-1, 1, (4, 5, 16)).astype(np.float32)
    for qt in (zb.Type.Int8, zb.Type.Int4):
        lin = zb.QuantizedLinear(torch.from_numpy(weight).cuda(), bias, qt)
        out = lin(torch.from_numpy(inp).cuda()).cpu().numpy()
        assert out.shape == (4, 5, 8)
        pay, sc = O.quantize_weights(weight, int(qt))
        ref = O.matmul(inp.reshape(20, 16), int(qt), pay, sc, 8, bias)[3].reshape(4, 5, 8)
        assert_bits_equal(out, ref, "QuantizedLinear")
        fp = inp.reshape(20, 16) @ weight + bias
        assert np.max(np.abs(fp.reshape(4, 5, 8) - out)) < (0.2 if qt == zb.Type.Int8 else 0.6)


def test_slice_cols_and_odd_k_int4_roundtrip(zb):
    import torch

    rng = np.random.default_rng(5)
    for qt, K, N in [(2, 33, 9), (2, 31, 70), (1, 7, 5)]:
        _, w = make(rng, 2, K, N, edge=False)
        pay, sc = O.quantize_weights(w, qt)
        W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
        assert np.array_equal(W.payload(), pay)
        for c in range(N):
            for r in (0, K - 1):
                assert W.value(c, r) == int(O.unpack_codes(qt, pay, K, N)[c, r])
        S = W.slice_cols(2, N - 1)
        codes = O.unpack_codes(qt, pay, K, N)[2:N - 1]
        assert np.array_equal(O.unpack_codes(qt, S.payload(), K, N - 3), codes)
        assert_bits_equal(S.scales(), sc[2:N - 1], "slice scales")
        x = rng.standard_normal((3, K)).astype(np.float32)
        full = zb.matmul(torch.from_numpy(x).cuda(), W).cpu().numpy()
        part = zb.matmul(torch.from_numpy(x).cuda(), S).cpu().numpy()
        assert_bits_equal(part, full[:, 2:N - 1], "column shard")


@pytest.mark.parametrize("qt", [1, 2])
@pytest.mark.parametrize("M,K,N", [(2048, 256, 4864), (2000, 200, 4900)])
def test_pair_tile_gemm_bit_exact(zb, qt, M, K, N):
    """Shapes with >= 148 tiles of 256 x 256 select the 2-SM (cluster pair)
    GEMM; the second one is ragged in M, K and N."""
    import torch

    rng = np.random.default_rng(M + N + qt)
    x, w = make(rng, M, K, N)
    pay, sc = O.quantize_weights(w, qt)
    W = zb.QuantizedMatrix.from_parts(qt, K, N, sc, pay)
    b = rng.standard_normal(N).astype(np.float32)
    y = zb.matmul(torch.from_numpy(x).cuda(), W, bias=torch.from_numpy(b).cuda()).cpu().numpy()
    assert_bits_equal(y, O.matmul(x, qt, pay, sc, N, b)[3], f"pair gemm t{qt} {M}x{K}x{N}")
    assert zb.device_error() == 0


@pytest.mark.parametrize("M,K,N", [(1024, 8192, 9472), (1000, 4000, 9500)])
def test_int4_pair_gemm_equals_int8_on_same_codes(zb, M, K, N):
    """Long-K INT4 GEMMs on the 2-SM tile.  INT4 weights must give exactly the
    INT8 result for the same codes and scales (the integer dot and the
    epilogue are the same), so the INT8 kernel -- bit-exact against the
    oracle above -- checks the INT4 unpack at sizes where the CPU oracle
    would take minutes.  The second shape is ragged in M, K and N."""
    import torch

    rng = np.random.default_rng(M + K)
    x, w = make(rng, M, K, N)
    pay4, sc = O.quantize_weights(w, 2)
    codes = O.unpack_codes(2, pay4, K, N)
    W4 = zb.QuantizedMatrix.from_parts(2, K, N, sc, pay4)
    W8 = zb.QuantizedMatrix.from_parts(1, K, N, sc, codes.view(np.uint8).ravel())
    xd = torch.from_numpy(x).cuda()
    assert_bits_equal(zb.matmul(xd, W4).cpu().numpy(), zb.matmul(xd, W8).cpu().numpy(),
                      f"int4 vs int8 pair gemm {M}x{K}x{N}")
    assert zb.device_error() == 0


def test_host_entry_point_chunked(zb):
    """Host calls with > 64 MiB of input run in pipelined row chunks; the
    result must equal the device-pointer path bit for bit (ragged last
    chunk), with sampled rows checked against the oracle."""
    import torch

    rng = np.random.default_rng(77)
    M, K, N = 2500, 8192, 300
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    pay, sc = O.quantize_weights(w, 1)
    W = zb.QuantizedMatrix.from_parts(1, K, N, sc, pay)
    xp = torch.from_numpy(x).pin_memory()
    y_host = zb.matmul(xp.numpy(), W)
    y_dev = zb.matmul(torch.from_numpy(x).cuda(), W).cpu().numpy()
    assert_bits_equal(y_host, y_dev, "chunked host matmul")
    rows = [0, 1, 1249, 1250, M - 1]
    assert_bits_equal(y_host[rows], O.matmul(x[rows], 1, pay, sc, N)[3], "chunked host rows vs oracle")


@pytest.mark.parametrize("M,K,N,pair", [(300, 256, 200, False), (2048, 256, 4864, True)])
def test_matmul_multi_destinations(zb, M, K, N, pair):
    """The epilogue writes every output element to several buffers at a row
    stride and column offset (the gathered-output path); each buffer holds
    exactly the single-output result in its columns and nothing else
    changes.  The second shape selects the 2-SM kernel."""
    import ctypes as C

    import torch
    from zyron_b200 import _lib

    L = _lib.lib()
    rng = np.random.default_rng(M + 3)
    x, w = make(rng, M, K, N, edge=False)
    pay, sc = O.quantize_weights(w, 1)
    W = zb.QuantizedMatrix.from_parts(1, K, N, sc, pay)
    xd = torch.from_numpy(x).cuda()
    want = zb.matmul(xd, W).cpu().numpy()
    ldy, off = N + 36, 20
    outs = [torch.full((M, ldy), -7.0, device="cuda") for _ in range(3)]
    ptrs = (C.c_void_p * 3)(*[o.data_ptr() for o in outs])
    wsb = L.zq_matmul_workspace_bytes(W.handle, M)
    ws = torch.empty(wsb + 256, dtype=torch.uint8, device="cuda")
    wp = (ws.data_ptr() + 255) & ~255
    _lib.check(L.zq_matmul_multi(W.handle, C.c_void_p(xd.data_ptr()), M, None, ptrs, 3, ldy, off, C.c_void_p(wp), wsb,
                                 C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    for o in outs:
        h = o.cpu().numpy()
        assert_bits_equal(h[:, off:off + N], want, "multi-destination output")
        assert np.all(h[:, :off] == -7.0) and np.all(h[:, off + N:] == -7.0)
    assert zb.device_error() == 0
