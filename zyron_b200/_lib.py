"""ctypes binding of the C ABI in include/zq.h (libzyron_b200.so).

The library is built in-tree (``python -m zyron_b200.build``).  There is no
fallback: if the shared library is missing, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libzyron_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "zq.h")

ZQ_OK = 0
ZQ_ERR_INVALID_ARGUMENT = 1
ZQ_ERR_OUT_OF_RANGE = 2
ZQ_ERR_OVERFLOW = 3
ZQ_ERR_RUNTIME = 4
ZQ_ERR_CUDA = 5
ZQ_ERR_DEVICE_TIMEOUT = 6


class ZQError(Exception):
    """Base class; ``status`` is the zq_status code."""

    status = -1


class ZQInvalidArgument(ZQError, ValueError):
    """std::invalid_argument in the reference."""

    status = ZQ_ERR_INVALID_ARGUMENT


class ZQOutOfRange(ZQError, IndexError):
    """std::out_of_range in the reference."""

    status = ZQ_ERR_OUT_OF_RANGE


class ZQOverflow(ZQError, OverflowError):
    """std::overflow_error in the reference."""

    status = ZQ_ERR_OVERFLOW


class ZQRuntimeError(ZQError, RuntimeError):
    """std::runtime_error in the reference (format / I/O)."""

    status = ZQ_ERR_RUNTIME


class ZQCudaError(ZQError, RuntimeError):
    status = ZQ_ERR_CUDA


class ZQDeviceTimeout(ZQError, RuntimeError):
    status = ZQ_ERR_DEVICE_TIMEOUT


_ERRORS = {
    ZQ_ERR_INVALID_ARGUMENT: ZQInvalidArgument,
    ZQ_ERR_OUT_OF_RANGE: ZQOutOfRange,
    ZQ_ERR_OVERFLOW: ZQOverflow,
    ZQ_ERR_RUNTIME: ZQRuntimeError,
    ZQ_ERR_CUDA: ZQCudaError,
    ZQ_ERR_DEVICE_TIMEOUT: ZQDeviceTimeout,
}

_lib = None
_lock = threading.Lock()

vp = C.c_void_p
sz = C.c_size_t
st = C.c_int

# name -> (restype, argtypes); must match include/zq.h
SIGNATURES = {
    "zq_last_error": (C.c_char_p, []),
    "zq_abi_version": (C.c_int, []),
    "zq_weight_create": (st, [C.c_int, sz, sz, vp, vp, sz, vp, C.POINTER(vp)]),
    "zq_weight_quantize": (st, [vp, sz, sz, C.c_int, vp, C.POINTER(vp)]),
    "zq_weight_quantize_host": (st, [vp, sz, sz, C.c_int, vp, C.POINTER(vp)]),
    "zq_dequantize_host": (st, [vp, vp, vp]),
    "zq_weight_load_zyq": (st, [vp, sz, C.POINTER(sz), vp, C.POINTER(vp)]),
    "zq_weight_save_zyq": (st, [vp, vp, sz, C.POINTER(sz), vp]),
    "zq_weight_info": (st, [vp, C.POINTER(C.c_int), C.POINTER(sz), C.POINTER(sz), C.POINTER(sz),
                            C.POINTER(C.c_int)]),
    "zq_weight_download": (st, [vp, vp, vp, vp]),
    "zq_weight_slice_cols": (st, [vp, sz, sz, vp, C.POINTER(vp)]),
    "zq_weight_destroy": (st, [vp]),
    "zq_matmul_workspace_bytes": (sz, [vp, sz]),
    "zq_quantize_rows": (st, [vp, sz, sz, vp, sz, vp, vp]),
    "zq_weight_padded_k": (sz, [vp]),
    "zq_matmul_codes": (st, [vp, vp, vp, sz, vp, vp, vp, sz, vp]),
    "zq_matmul": (st, [vp, vp, sz, vp, vp, vp, sz, vp]),
    "zq_matmul_noalloc": (st, [vp, vp, sz, vp, vp, vp]),
    "zq_matmul_multi": (st, [vp, vp, sz, vp, vp, C.c_int, sz, sz, vp, sz, vp]),
    "zq_shard_range": (st, [sz, C.c_int, C.c_int, C.POINTER(sz), C.POINTER(sz)]),
    "zq_nccl_get_unique_id": (st, [vp]),
    "zq_nccl_comm_init": (st, [C.c_int, vp, C.c_int, C.POINTER(vp)]),
    "zq_nccl_comm_destroy": (st, [vp]),
    "zq_matmul_sharded_workspace_bytes": (sz, [vp, sz, sz, C.c_int]),
    "zq_matmul_sharded": (st, [vp, vp, sz, vp, vp, sz, vp, vp, sz, vp]),
    "zq_matmul_host": (st, [vp, vp, sz, vp, vp, vp]),
    "zq_dequantize": (st, [vp, vp, vp]),
    "zq_device_error": (st, [vp, C.POINTER(C.c_uint32)]),
    "zq_weight_set_option": (st, [vp, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "zq_test_decode_wait_timeout": (st, [vp, vp, vp, sz, vp, vp, sz, C.c_uint64, vp]),
    "zq_lm_set_option": (st, [vp, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "zq_ipc_export": (st, [vp, vp]),
    "zq_ipc_import": (st, [vp, C.POINTER(vp)]),
    "zq_ipc_close": (st, [vp]),
    "zq_lm_load": (st, [vp, sz, vp, C.POINTER(vp)]),
    "zq_lm_get_info": (st, [vp, vp]),
    "zq_lm_generate_greedy": (st, [vp, vp, sz, sz, vp, sz, C.POINTER(sz), vp, vp]),
    "zq_lm_generate": (st, [vp, vp, sz, vp, vp, sz, C.POINTER(sz), vp, vp]),
    "zq_lm_destroy": (st, [vp]),
    "zq_quantize_checkpoint": (st, [vp, sz, C.c_int, vp, C.POINTER(vp), C.POINTER(sz), C.POINTER(C.c_double)]),
    "zq_lm_init_image": (st, [vp, C.c_uint32, C.c_int, vp, C.POINTER(vp), C.POINTER(sz), C.POINTER(C.c_double)]),
    "zq_free_buffer": (None, [vp]),
    "zq_sampler_create": (st, [C.c_uint32, C.POINTER(vp)]),
    "zq_sampler_destroy": (st, [vp]),
    "zq_sample_next": (st, [vp, vp, sz, vp, sz, vp, C.POINTER(C.c_int64)]),
}


class GenerationConfigC(C.Structure):
    """zq_generation_config (include/zq.h)."""

    _fields_ = [("max_new_tokens", C.c_size_t), ("temperature", C.c_float), ("top_k", C.c_size_t),
                ("top_p", C.c_float), ("repetition_penalty", C.c_float), ("no_repeat_ngram_size", C.c_size_t),
                ("seed", C.c_uint32)]


class LmConfigC(C.Structure):
    """zq_lm_config (include/zq.h)."""

    _fields_ = [("vocab_size", C.c_size_t), ("hidden_size", C.c_size_t), ("num_layers", C.c_size_t),
                ("num_heads", C.c_size_t), ("num_kv_heads", C.c_size_t), ("intermediate_size", C.c_size_t),
                ("max_sequence_length", C.c_size_t), ("norm_eps", C.c_float), ("use_rms_norm", C.c_int),
                ("causal", C.c_int), ("use_rope", C.c_int), ("tie_word_embeddings", C.c_int),
                ("rope_theta", C.c_float), ("dropout", C.c_float), ("use_qat", C.c_int), ("qat_bits", C.c_size_t)]


class IpcHandle(C.Structure):
    """zq_ipc_handle (include/zq.h)."""

    _fields_ = [("handle", C.c_ubyte * 64), ("offset", C.c_uint64), ("device", C.c_int), ("pad", C.c_int)]


class LmInfo(C.Structure):
    """zq_lm_info (include/zq.h)."""

    _fields_ = [(n, C.c_size_t) for n in ("vocab_size", "hidden_size", "num_layers", "num_heads", "num_kv_heads",
                                          "intermediate_size", "max_sequence_length")] + [
        ("norm_eps", C.c_float), ("use_rms_norm", C.c_int), ("causal", C.c_int), ("use_rope", C.c_int),
        ("tie_word_embeddings", C.c_int), ("rope_theta", C.c_float), ("type", C.c_int),
        ("quantized_bytes", C.c_size_t), ("float_reference_bytes", C.c_size_t)]


def header_symbols():
    """Entry points declared in include/zq.h."""
    with open(HEADER) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(zq_[a-z0-9_]+)\s*\(", text)))


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"zyron_b200 native library not built: {LIB_PATH} is missing "
                        "(run `python -m zyron_b200.build`)")
                L = C.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(status):
    if status != ZQ_OK:
        msg = lib().zq_last_error().decode(errors="replace")
        raise _ERRORS.get(status, ZQError)(msg)
