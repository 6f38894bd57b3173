"""Generate the golden fixtures in tests/golden/ from the ZYRON reference itself.

The reference is compiled from its own sources by ``oracle/Makefile`` into
``oracle/_ref/libzyron_ref.so`` (``make -C oracle REF=<reference checkout>``).
This script feeds it seeded inputs and records what the reference's public
API returns -- quantize() payloads and scales, matmul() and
QuantizedLinear::forward() outputs, dequantize(), the .zyq bytes of save(),
and the exception messages of load() on damaged .zyq records.  The fixtures
are committed, so tests need neither the reference nor this script.

Inputs: numpy's PCG64 generator, x ~ N(0, 1), w ~ N(0, 0.02) (the shapes and
distributions of the quantized-matmul workloads), plus edge rows (all zeros,
NaN, +-inf, denormals, exact half-way quotients).

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

# (M, K, N): ragged sizes around tile edges, odd K (INT4 columns straddle
# bytes), single row / single column, and 64 rows x K=512 of the matmul workload.
SHAPES = [
    (1, 1, 1), (1, 17, 9), (3, 33, 5), (7, 32, 24), (2, 31, 7), (5, 129, 3),
    (9, 64, 130), (4, 100, 257), (64, 512, 40),
]


def edge_rows(x, rng):
    M, K = x.shape
    if M >= 2:
        x[1] = 0.0                                   # all-zero row -> scale 1.0
    if M >= 3:
        x[2, 0] = np.nan                             # NaN skipped by absmax, code -127
    if M >= 4:
        x[3, K // 2] = np.inf                        # inf -> scale inf, all codes 0
    if M >= 5:
        x[4] = np.float32(1e-45) * rng.integers(-3, 4, K)  # denormals; scale underflows
    if M >= 6 and K >= 4:
        # exact half-way quotients: absmax 127 -> scale 1.0, x = k + 0.5
        x[5, :] = 0.5
        x[5, 0] = 127.0
        x[5, 1] = -2.5
        x[5, 2] = 3.5
    return x


def damaged_zyq(good: bytes):
    """Damaged .zyq records paired with the reference's exception text."""
    cases = []
    b = bytearray(good)
    cases.append(("empty", b""))
    cases.append(("short_magic", bytes(b[:3])))
    bad = bytearray(b); bad[0] ^= 0xFF
    cases.append(("bad_magic", bytes(bad)))
    bad = bytearray(b); bad[4] = 2
    cases.append(("bad_version", bytes(bad)))
    cases.append(("short_version", bytes(b[:6])))
    bad = bytearray(b); bad[8] = 3
    cases.append(("bad_type", bytes(bad)))
    bad = bytearray(b); bad[12:20] = (0).to_bytes(8, "little")
    cases.append(("zero_rows", bytes(bad)))
    bad = bytearray(b); bad[20:28] = (0).to_bytes(8, "little")
    cases.append(("zero_cols", bytes(bad)))
    bad = bytearray(b); bad[12:20] = (1 << 40).to_bytes(8, "little"); bad[20:28] = (1 << 40).to_bytes(8, "little")
    cases.append(("overflow", bytes(bad)))
    bad = bytearray(b); bad[28:36] = (1).to_bytes(8, "little")
    cases.append(("bad_scale_count", bytes(bad)))
    bad = bytearray(b); bad[36:40] = np.array([-1.0], dtype="<f4").tobytes()
    cases.append(("negative_scale", bytes(bad)))
    bad = bytearray(b); bad[36:40] = np.array([np.nan], dtype="<f4").tobytes()
    cases.append(("nan_scale", bytes(bad)))
    bad = bytearray(b); bad[36:40] = np.array([np.inf], dtype="<f4").tobytes()
    cases.append(("inf_scale", bytes(bad)))
    cases.append(("short_scales", bytes(b[:38])))
    ncols = int.from_bytes(b[20:28], "little")
    poff = 36 + 4 * ncols
    bad = bytearray(b); bad[poff:poff + 8] = (7).to_bytes(8, "little")
    cases.append(("bad_payload_size", bytes(bad)))
    cases.append(("short_payload", bytes(b[:-1])))
    out = []
    for name, data in cases:
        try:
            O.RefMatrix.load_bytes(data if data else b"\0")  # ref needs a non-null buffer
            if not data:
                raise AssertionError
            out.append((name, data, 0, ""))
        except O.RefError as e:
            out.append((name, data, e.code, str(e)))
        except AssertionError:
            out.append((name, data, 0, ""))
    # The empty case must be fed as a zero-length stream.
    fixed = []
    for name, data, code, msg in out:
        if name == "empty":
            try:
                buf = np.zeros(1, dtype=np.uint8)
                h = O.C.c_void_p()
                rc = O.ref().ref_load_zyq(O.C.c_void_p(buf.ctypes.data), 0, O.C.byref(h))
                msg = O.ref().ref_last_error().decode() if rc else ""
                code = rc
            except Exception as e:  # pragma: no cover
                raise e
        fixed.append((name, data, code, msg))
    return fixed


def main():
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libzyron_ref.so is missing: run make -C oracle REF=<reference>")
    rng = np.random.default_rng(20261201)
    arrays = {}
    index = []
    for ci, (M, K, N) in enumerate(SHAPES):
        x = edge_rows(rng.standard_normal((M, K)).astype(np.float32), rng)
        w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        if N >= 3:
            w[:, 1] = 0.0                                 # all-zero column -> scale 1.0
        bias = rng.standard_normal(N).astype(np.float32)
        arrays[f"c{ci}_x"] = x
        arrays[f"c{ci}_w"] = w
        arrays[f"c{ci}_bias"] = bias
        for qt in (O.INT8, O.INT4):
            R = O.RefMatrix.quantize(w, qt)
            p = f"c{ci}_t{qt}"
            arrays[p + "_payload"] = R.payload()
            arrays[p + "_scales"] = R.scales()
            arrays[p + "_y"] = R.matmul(x)
            arrays[p + "_ylin"] = R.linear(x, bias)
            arrays[p + "_deq"] = R.dequantize()
            arrays[p + "_zyq"] = np.frombuffer(R.save_bytes(), dtype=np.uint8)
        index.append((M, K, N))
    arrays["shapes"] = np.array(index, dtype=np.int64)

    R = O.RefMatrix.quantize(arrays["c2_w"], O.INT4)
    cases = damaged_zyq(R.save_bytes())
    arrays["zyq_bad_names"] = np.array([c[0] for c in cases])
    arrays["zyq_bad_codes"] = np.array([c[2] for c in cases], dtype=np.int32)
    arrays["zyq_bad_msgs"] = np.array([c[3] for c in cases])
    for name, data, _, _ in cases:
        arrays[f"zyq_bad_{name}"] = np.frombuffer(data, dtype=np.uint8)

    out = os.path.join(HERE, "quantization_golden.npz")
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({os.path.getsize(out)} bytes, {len(SHAPES)} shapes, {len(cases)} damaged records)")


if __name__ == "__main__":
    main()
