"""Python mirror of ZYRON's ``zyron::quantization`` API over the C ABI.

Names, argument meaning and error behaviour follow the reference:
``Type``, ``QuantizedMatrix`` (include/zyron/quantization/quantization.hpp:
13-52), ``quantize`` / ``matmul`` (54-58) and ``QuantizedLinear``
(include/zyron/quantization/quantized_linear.hpp:10-31).  Exceptions map
std::invalid_argument -> ValueError, std::out_of_range -> IndexError,
std::overflow_error -> OverflowError, std::runtime_error -> RuntimeError
(the ZQError subclasses in ``_lib``), with the reference's messages.

Weights live in device memory (one upload); activations may be torch CUDA
tensors (the result stays on the device) or numpy arrays (host in, host out,
through ``zq_matmul_host``).
"""
from __future__ import annotations

import ctypes as C
import enum
import threading

import numpy as np

from . import _lib
from ._lib import check, lib


class Type(enum.IntEnum):
    Int8 = 1
    Int4 = 2


def _torch():
    import torch

    return torch


def _stream_ptr(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _payload_bytes(qtype, rows, cols):
    e = rows * cols
    return e if qtype == Type.Int8 else (e + 1) // 2


class QuantizedMatrix:
    """Device-resident quantized weight with the reference's accessors."""

    def __init__(self, handle=None):
        self._h = handle
        self._host_cache = None
        if handle is not None:
            t = C.c_int()
            r, c, p = C.c_size_t(), C.c_size_t(), C.c_size_t()
            d = C.c_int()
            check(lib().zq_weight_info(handle, C.byref(t), C.byref(r), C.byref(c), C.byref(p), C.byref(d)))
            self._type, self._rows, self._cols, self._device = Type(t.value), r.value, c.value, d.value
        else:
            self._type, self._rows, self._cols, self._device = Type.Int8, 0, 0, -1

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib._lib is not None:
            _lib._lib.zq_weight_destroy(h)
            self._h = None

    # ---- construction ------------------------------------------------------
    @classmethod
    def from_parts(cls, qtype, rows, cols, scales, payload, stream=None):
        """Upload scales + payload given in the reference's storage layout."""
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        payload = np.ascontiguousarray(payload, dtype=np.uint8)
        h = C.c_void_p()
        check(lib().zq_weight_create(int(qtype), rows, cols, scales.ctypes.data_as(C.c_void_p),
                                     payload.ctypes.data_as(C.c_void_p), payload.size,
                                     _stream_ptr(stream), C.byref(h)))
        return cls(h)

    @classmethod
    def load_bytes(cls, data: bytes, stream=None):
        buf = np.frombuffer(data, dtype=np.uint8)
        h = C.c_void_p()
        used = C.c_size_t()
        check(lib().zq_weight_load_zyq(buf.ctypes.data_as(C.c_void_p), len(data), C.byref(used),
                                       _stream_ptr(stream), C.byref(h)))
        return cls(h)

    @classmethod
    def load(cls, path, stream=None):
        try:
            with open(path, "rb") as f:
                data = f.read()
        except OSError:
            raise _lib.ZQRuntimeError(f"ZYRON quantization: failed to open: {path}")
        return cls.load_bytes(data, stream)

    def save_bytes(self, stream=None) -> bytes:
        if self.empty():
            raise _lib.ZQRuntimeError("ZYRON quantization: cannot save empty matrix")
        n = C.c_size_t()
        check(lib().zq_weight_save_zyq(self._h, None, 0, C.byref(n), _stream_ptr(stream)))
        buf = np.zeros(n.value, dtype=np.uint8)
        check(lib().zq_weight_save_zyq(self._h, buf.ctypes.data_as(C.c_void_p), n.value, C.byref(n),
                                       _stream_ptr(stream)))
        return buf.tobytes()

    def save(self, path, stream=None):
        data = self.save_bytes(stream)
        try:
            with open(path, "wb") as f:
                f.write(data)
        except OSError:
            raise _lib.ZQRuntimeError(f"ZYRON quantization: failed to open: {path}")

    # ---- accessors (quantization.hpp:22-33) ---------------------------------
    def type(self):
        return self._type

    def rows(self):
        return self._rows

    def cols(self):
        return self._cols

    def elements(self):
        return 0 if self.empty() else self._rows * self._cols

    def empty(self):
        return self._rows == 0 or self._cols == 0

    def bytes(self):
        if self.empty():
            return 0
        return _payload_bytes(self._type, self._rows, self._cols) + 4 * self._cols

    def float_bytes(self):
        return self.elements() * 4

    def compression_ratio(self):
        b = self.bytes()
        return 0.0 if b == 0 else self.float_bytes() / b

    def _download(self):
        if self._host_cache is None:
            scales = np.zeros(self._cols, dtype=np.float32)
            payload = np.zeros(_payload_bytes(self._type, self._rows, self._cols), dtype=np.uint8)
            check(lib().zq_weight_download(self._h, scales.ctypes.data_as(C.c_void_p),
                                           payload.ctypes.data_as(C.c_void_p), _stream_ptr()))
            self._host_cache = (scales, payload)
        return self._host_cache

    def scales(self):
        if self.empty():
            return np.zeros(0, dtype=np.float32)
        return self._download()[0].copy()

    def payload(self):
        """Raw payload in the reference's column-major storage."""
        return self._download()[1].copy()

    def value(self, column, row):
        """Code at (column, row) (quantization.cpp:89-97)."""
        if column >= self._cols or row >= self._rows or column < 0 or row < 0:
            raise _lib.ZQOutOfRange("ZYRON quantization: matrix index out of range")
        lin = column * self._rows + row
        payload = self._download()[1]
        if self._type == Type.Int8:
            return int(payload.view(np.int8)[lin])
        b = int(payload[lin >> 1])
        nib = (b >> 4) if (lin & 1) else (b & 0x0F)
        return nib if nib < 8 else nib - 16

    def dequantize(self):
        """fp32 [rows, cols] torch tensor on the weight's device."""
        torch = _torch()
        if self.empty():
            return torch.zeros((self._rows, self._cols), dtype=torch.float32)
        out = torch.empty((self._rows, self._cols), dtype=torch.float32, device=f"cuda:{self._device}")
        check(lib().zq_dequantize(self._h, C.c_void_p(out.data_ptr()), _stream_ptr()))
        return out

    def slice_cols(self, begin, end, stream=None):
        h = C.c_void_p()
        check(lib().zq_weight_slice_cols(self._h, begin, end, _stream_ptr(stream), C.byref(h)))
        return QuantizedMatrix(h)

    def set_option(self, option: int, value: int) -> int:
        """zq_weight_set_option on this weight (ZQ_OPT_* of include/zq.h);
        returns the old value.  Results never depend on the options."""
        prev = C.c_int()
        check(lib().zq_weight_set_option(self._h, int(option), int(value), C.byref(prev)))
        return prev.value

    def set_decode_kernel(self, kind: int) -> int:
        """Kernel for this weight's matmuls with few rows: 0 automatic,
        1 tcgen05 decode kernel, 2 dp4a GEMV (ZQ_DECODE_*)."""
        return self.set_option(1, kind)  # ZQ_OPT_DECODE_KERNEL

    @property
    def handle(self):
        return self._h


def quantize(weights, qtype=Type.Int8, stream=None):
    """quantize() (quantization.cpp:121-162).  ``weights`` is an fp32 [K, N]
    torch CUDA tensor (quantized on the device) or numpy array (uploaded
    first)."""
    torch = _torch()
    if isinstance(weights, np.ndarray):
        if weights.ndim != 2:
            raise _lib.ZQInvalidArgument("ZYRON quantization: weights must be rank-2")
        weights = torch.from_numpy(np.ascontiguousarray(weights, dtype=np.float32)).cuda()
    if weights.dim() != 2:
        raise _lib.ZQInvalidArgument("ZYRON quantization: weights must be rank-2")
    if not weights.is_contiguous():
        raise _lib.ZQInvalidArgument("ZYRON quantization: weights must be contiguous")
    if weights.dtype != torch.float32:
        raise _lib.ZQInvalidArgument("zyron_b200: weights must be float32")
    if int(qtype) not in (1, 2):
        raise _lib.ZQInvalidArgument("ZYRON quantization: unsupported type")
    h = C.c_void_p()
    with torch.cuda.device(weights.device):
        check(lib().zq_weight_quantize(C.c_void_p(weights.data_ptr()), weights.shape[0], weights.shape[1],
                                       int(qtype), _stream_ptr(stream), C.byref(h)))
    return QuantizedMatrix(h)


class _Workspaces(threading.local):
    def __init__(self):
        self.bufs = {}


_ws = _Workspaces()


def workspace(weights, m, device, stream_key):
    """Per-thread, per-(device, stream) cached device scratch for zq_matmul."""
    torch = _torch()
    need = lib().zq_matmul_workspace_bytes(weights.handle, m)
    key = (device, stream_key)
    buf = _ws.bufs.get(key)
    if buf is None or buf.numel() < need:
        buf = torch.empty(max(need, 256) + 256, dtype=torch.uint8, device=device)
        _ws.bufs[key] = buf
    base = buf.data_ptr()
    aligned = (base + 255) & ~255
    return aligned, buf.numel() - (aligned - base)


def matmul(input, weights: QuantizedMatrix, bias=None, out=None, stream=None):
    """quantization::matmul (quantization.cpp:177-238); with ``bias`` it is
    QuantizedLinear::forward (quantized_linear.cpp:33-50).

    torch CUDA input -> torch CUDA output; numpy input -> numpy output.
    """
    ndim = input.ndim if isinstance(input, np.ndarray) else input.dim()
    if ndim < 2:
        raise _lib.ZQInvalidArgument("ZYRON quantization: input rank must be >= 2")
    if weights is None or weights.empty():
        raise _lib.ZQInvalidArgument("ZYRON quantization: weights are empty")
    if input.shape[-1] != weights.rows():
        raise _lib.ZQInvalidArgument("ZYRON quantization: input/weight dimension mismatch")
    out_shape = tuple(input.shape[:-1]) + (weights.cols(),)

    if isinstance(input, np.ndarray):
        x = np.ascontiguousarray(input, dtype=np.float32).reshape(-1, weights.rows())
        y = np.empty((x.shape[0], weights.cols()), dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        check(lib().zq_matmul_host(weights.handle, x.ctypes.data_as(C.c_void_p), x.shape[0],
                                   None if b is None else b.ctypes.data_as(C.c_void_p),
                                   y.ctypes.data_as(C.c_void_p), _stream_ptr(stream)))
        return y.reshape(out_shape)

    torch = _torch()
    if input.dtype != torch.float32:
        raise _lib.ZQInvalidArgument("zyron_b200: input must be float32")
    x = input.contiguous().reshape(-1, weights.rows())
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, weights.cols()), dtype=torch.float32, device=x.device)
    s = stream if stream is not None else torch.cuda.current_stream(x.device)
    with torch.cuda.device(x.device):
        ws, ws_bytes = workspace(weights, m, x.device, s.cuda_stream)
        check(lib().zq_matmul(weights.handle, C.c_void_p(x.data_ptr()), m,
                              None if bias is None else C.c_void_p(bias.data_ptr()),
                              C.c_void_p(out.data_ptr()), C.c_void_p(ws), ws_bytes, C.c_void_p(s.cuda_stream)))
    return out.reshape(out_shape)


def quantize_rows(x, stream=None):
    """The per-row activation quantizer alone: (codes int8 [M,K], scales fp32 [M])."""
    torch = _torch()
    x = x.contiguous()
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        check(lib().zq_quantize_rows(C.c_void_p(x.data_ptr()), m, k, C.c_void_p(q.data_ptr()), k,
                                     C.c_void_p(s.data_ptr()), _stream_ptr(stream)))
    return q, s


def device_error(stream=None):
    """Synchronise and raise ZQDeviceTimeout if a bounded device wait gave up."""
    code = C.c_uint32()
    check(lib().zq_device_error(_stream_ptr(stream), C.byref(code)))
    return code.value


class QuantizedLinear:
    """Inference-only linear layer (quantized_linear.cpp:8-50)."""

    def __init__(self, weight, bias=None, qtype=Type.Int8):
        torch = _torch()
        if isinstance(weight, QuantizedMatrix):
            if weight.empty():
                raise _lib.ZQInvalidArgument("ZYRON QuantizedLinear: weight cannot be empty")
            self._w = weight
            if bias is not None:
                b = torch.as_tensor(bias, dtype=torch.float32)
                if b.numel() != 0 and (b.dim() != 1 or b.numel() != weight.cols()):
                    raise _lib.ZQInvalidArgument("ZYRON QuantizedLinear: bias shape mismatch")
                bias = b if b.numel() else None
        else:
            self._w = quantize(weight, qtype)
            if weight.ndim != 2:
                raise _lib.ZQInvalidArgument("ZYRON QuantizedLinear: weight must be rank-2")
            if bias is not None:
                b = torch.as_tensor(bias, dtype=torch.float32)
                if b.dim() != 1 or b.shape[0] != weight.shape[1]:
                    raise _lib.ZQInvalidArgument("ZYRON QuantizedLinear: bias shape mismatch")
                bias = b
        self._b = None if bias is None else bias.to(f"cuda:{self._w._device}").contiguous()

    def in_features(self):
        return self._w.rows()

    def out_features(self):
        return self._w.cols()

    def type(self):
        return self._w.type()

    def weight(self):
        return self._w

    def bias(self):
        return self._b

    def forward(self, input, out=None, stream=None):
        ndim = input.ndim if isinstance(input, np.ndarray) else input.dim()
        if ndim < 2:
            raise _lib.ZQInvalidArgument("ZYRON QuantizedLinear: input rank must be >= 2")
        if input.shape[-1] != self.in_features():
            raise _lib.ZQInvalidArgument("ZYRON QuantizedLinear: input feature mismatch")
        bias = self._b
        if isinstance(input, np.ndarray) and bias is not None:
            bias = bias.cpu().numpy()
        return matmul(input, self._w, bias=bias, out=out, stream=stream)

    __call__ = forward
