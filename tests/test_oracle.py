"""The oracle (oracle/zq_oracle.c) pinned against the ZYRON reference.

* against the committed golden vectors, which the reference itself produced
  (tests/golden/make_golden.py), bit for bit;
* against the compiled reference (oracle/_ref) on fresh seeded inputs, when
  that library is present.
"""
import numpy as np
import pytest

from oracle import oracle as O


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def cases(golden):
    for ci, (M, K, N) in enumerate(golden["shapes"]):
        for qt in (O.INT8, O.INT4):
            yield ci, int(M), int(K), int(N), qt


def test_golden_quantize(golden):
    for ci, M, K, N, qt in cases(golden):
        p = f"c{ci}_t{qt}"
        payload, scales = O.quantize_weights(golden[f"c{ci}_w"], qt)
        assert np.array_equal(payload, golden[p + "_payload"]), p
        assert np.array_equal(bits(scales), bits(golden[p + "_scales"])), p


def test_golden_matmul_and_linear(golden):
    for ci, M, K, N, qt in cases(golden):
        p = f"c{ci}_t{qt}"
        pay, sc = golden[p + "_payload"], golden[p + "_scales"]
        _, _, _, y = O.matmul(golden[f"c{ci}_x"], qt, pay, sc, N)
        assert np.array_equal(bits(y), bits(golden[p + "_y"])), p
        _, _, _, yl = O.matmul(golden[f"c{ci}_x"], qt, pay, sc, N, golden[f"c{ci}_bias"])
        assert np.array_equal(bits(yl), bits(golden[p + "_ylin"])), p


def test_golden_dequantize_and_zyq(golden):
    for ci, M, K, N, qt in cases(golden):
        p = f"c{ci}_t{qt}"
        pay, sc = golden[p + "_payload"], golden[p + "_scales"]
        assert np.array_equal(bits(O.dequantize(qt, pay, sc, K, N)), bits(golden[p + "_deq"])), p
        assert O.zyq_bytes(qt, K, N, sc, pay) == golden[p + "_zyq"].tobytes(), p


def test_quantize_value_edges():
    # lround half away from zero, clamp, NaN -> -limit, bad scales -> 0
    q = O.lib().zo_quantize_value
    assert q(2.5, 1.0, 127) == 3 and q(-2.5, 1.0, 127) == -3
    assert q(0.49999997, 1.0, 127) == 0
    assert q(200.0, 1.0, 127) == 127 and q(-200.0, 1.0, 127) == -127
    assert q(9.0, 1.0, 7) == 7
    assert q(float("nan"), 1.0, 127) == -127
    assert q(1.0, 0.0, 127) == 0 and q(1.0, float("inf"), 127) == 0 and q(1.0, float("nan"), 127) == 0


@pytest.mark.skipif(not O.ref_available(), reason="compiled reference not built here")
@pytest.mark.parametrize("qt", [O.INT8, O.INT4])
@pytest.mark.parametrize("shape", [(5, 47, 13), (16, 256, 96), (1, 4096, 64), (33, 65, 2)])
def test_oracle_matches_compiled_reference(qt, shape):
    M, K, N = shape
    rng = np.random.default_rng(M * 1000 + K + N + qt)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    R = O.RefMatrix.quantize(w, qt)
    pay, sc = O.quantize_weights(w, qt)
    assert np.array_equal(R.payload(), pay)
    assert np.array_equal(bits(R.scales()), bits(sc))
    assert np.array_equal(bits(R.matmul(x)), bits(O.matmul(x, qt, pay, sc, N)[3]))
    assert np.array_equal(bits(R.linear(x, b)), bits(O.matmul(x, qt, pay, sc, N, b)[3]))
    assert np.array_equal(R.codes(), O.unpack_codes(qt, pay, K, N))


def test_int32_accumulators_are_exact():
    # the int32 accumulator equals an int64 reference sum (no wrap at these K)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 300)).astype(np.float32)
    w = (rng.standard_normal((300, 6)) * 0.02).astype(np.float32)
    pay, sc = O.quantize_weights(w, O.INT4)
    q, s, acc, _ = O.matmul(x, O.INT4, pay, sc, 6)
    codes = O.unpack_codes(O.INT4, pay, 300, 6).astype(np.int64)
    assert np.array_equal(acc.astype(np.int64), q.astype(np.int64) @ codes.T)
