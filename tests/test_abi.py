"""The C ABI boundary without a GPU: the library loads, exports every entry
point include/zq.h declares, and rejects bad arguments and damaged .zyq
records on the host with the reference's status and message before any
device work."""
import ctypes as C

import numpy as np
import pytest

from zyron_b200 import _lib


def test_library_exports_every_header_symbol(native_lib):
    declared = _lib.header_symbols()
    assert declared, "no entry points parsed from include/zq.h"
    for name in declared:
        assert hasattr(native_lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(declared)
    assert native_lib.zq_abi_version() == 1


def _create(qtype, rows, cols, scales, payload):
    h = C.c_void_p()
    rc = _lib.lib().zq_weight_create(qtype, rows, cols, scales.ctypes.data_as(C.c_void_p),
                                     payload.ctypes.data_as(C.c_void_p), payload.size, None, C.byref(h))
    return rc, _lib.lib().zq_last_error().decode()


def test_weight_create_validation(native_lib):
    s = np.ones(4, dtype=np.float32)
    p = np.zeros(16, dtype=np.uint8)
    assert _create(3, 4, 4, s, p) == (_lib.ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: unsupported type")
    assert _create(1, 0, 4, s, p) == (_lib.ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty")
    assert _create(1, 4, 0, s, p) == (_lib.ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: weights are empty")
    assert _create(1, 4, 4, s, p[:15]) == (_lib.ZQ_ERR_INVALID_ARGUMENT,
                                           "ZYRON quantization: invalid payload size")
    assert _create(2, 4, 4, s, p) == (_lib.ZQ_ERR_INVALID_ARGUMENT, "ZYRON quantization: invalid payload size")
    assert _create(1, 1 << 33, 1 << 33, s, p)[0] == _lib.ZQ_ERR_OVERFLOW


def test_null_weight_is_empty(native_lib):
    L = native_lib
    assert L.zq_matmul(None, None, 1, None, None, None, 0, None) == _lib.ZQ_ERR_INVALID_ARGUMENT
    assert L.zq_last_error().decode() == "ZYRON quantization: weights are empty"
    assert L.zq_dequantize(None, None, None) == _lib.ZQ_ERR_INVALID_ARGUMENT
    assert L.zq_matmul_workspace_bytes(None, 8) == 0
    assert L.zq_weight_destroy(None) == _lib.ZQ_OK


def test_damaged_zyq_matches_reference_messages(native_lib, golden):
    L = native_lib
    for name, code, msg in zip(golden["zyq_bad_names"], golden["zyq_bad_codes"], golden["zyq_bad_msgs"]):
        data = golden[f"zyq_bad_{name}"]
        buf = np.ascontiguousarray(data, dtype=np.uint8)
        h = C.c_void_p()
        used = C.c_size_t()
        rc = L.zq_weight_load_zyq(buf.ctypes.data_as(C.c_void_p) if buf.size else None, buf.size,
                                  C.byref(used), None, C.byref(h))
        # reference exception class -> status: 3 overflow_error, 4 runtime_error
        assert rc == int(code), (name, rc, L.zq_last_error())
        assert L.zq_last_error().decode() == str(msg), name


def test_python_mirror_errors(native_lib):
    import zyron_b200 as zb

    empty = zb.QuantizedMatrix()
    assert empty.empty() and empty.bytes() == 0 and empty.compression_ratio() == 0.0
    with pytest.raises(ValueError, match="ZYRON quantization: input rank must be >= 2"):
        zb.matmul(np.zeros(4, dtype=np.float32), empty)
    with pytest.raises(ValueError, match="ZYRON quantization: weights are empty"):
        zb.matmul(np.zeros((1, 4), dtype=np.float32), empty)
    with pytest.raises(RuntimeError, match="ZYRON quantization: cannot save empty matrix"):
        empty.save_bytes()
    with pytest.raises(IndexError, match="ZYRON quantization: matrix index out of range"):
        empty.value(0, 0)
    with pytest.raises(RuntimeError, match="ZYRON quantization: failed to open"):
        zb.QuantizedMatrix.load("/nonexistent/dir/w.zyq")


def test_device_layout_constants():
    # The panel layout pads K to whole 128-code k-blocks for both types;
    # workspace sizes follow from it.  Restated here from csrc/zq_kernels.h.
    def padded(t, k):
        return (k + 127) // 128 * 128

    assert padded(1, 1) == 128 and padded(1, 128) == 128 and padded(1, 129) == 256
    assert padded(2, 1) == 128 and padded(2, 4096) == 4096 and padded(2, 11008) == 11008
