"""zyron_b200 -- B200-native (sm_100a) implementation of ZYRON's quantized
inference matmul path behind the reference's ``zyron::quantization`` API.

The compute path is hand-written CUDA in ``csrc/`` reached through the C ABI
declared in ``include/zq.h``; this package is a thin Python mirror of the
reference API used by the tests and the bench.  The C++20 drop-in lives in
``cpp/``.
"""
from ._lib import (ZQCudaError, ZQDeviceTimeout, ZQError, ZQInvalidArgument, ZQOutOfRange, ZQOverflow,
                   ZQRuntimeError, lib)
from .quantization import (QuantizedLinear, QuantizedMatrix, Type, device_error, matmul, quantize,
                           quantize_rows)

__all__ = [
    "Type", "QuantizedMatrix", "QuantizedLinear", "quantize", "matmul", "quantize_rows", "device_error",
    "ZQError", "ZQInvalidArgument", "ZQOutOfRange", "ZQOverflow", "ZQRuntimeError", "ZQCudaError",
    "ZQDeviceTimeout", "lib",
]
