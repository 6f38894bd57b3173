"""ctypes front end to the checkers (TEST INFRASTRUCTURE ONLY).

Two checkers live under oracle/:

* ``liboracle.so`` -- the C restatement of ZYRON's quantized matmul path
  (``zq_oracle.c``; each function cites the reference file:line it follows).
* ``_ref/libzyron_ref.so`` -- the reference itself, compiled from its own
  sources by ``oracle/Makefile`` together with ``ref_harness.cpp``.  It is
  present wherever it was built (it travels with the repository snapshot as a
  built artefact); :func:`ref_available` says whether it can be loaded.

Only tests/, the smoke check and bench.py's CPU-baseline / reference arm import
this module.  The product package (zyron_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
INT8, INT4 = 1, 2

_lib = None
_ref = None


def _f32p(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _vp(a):
    return C.c_void_p(a.ctypes.data) if a is not None else None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError("oracle/liboracle.so is not built (run make -C oracle)")
        L = C.CDLL(path)
        sz = C.c_size_t
        L.zo_quantize_value.restype = C.c_int8
        L.zo_quantize_value.argtypes = [C.c_float, C.c_float, C.c_int]
        L.zo_payload_bytes.restype = sz
        L.zo_payload_bytes.argtypes = [C.c_int, sz, sz]
        L.zo_quantize_weights.argtypes = [C.c_void_p, sz, sz, C.c_int, C.c_void_p, C.c_void_p]
        L.zo_quantize_rows.argtypes = [C.c_void_p, sz, sz, C.c_void_p, C.c_void_p]
        L.zo_matmul_codes.argtypes = [C.c_void_p, C.c_void_p, sz, sz, C.c_int, C.c_void_p,
                                      C.c_void_p, sz, C.c_void_p, C.c_void_p, C.c_void_p]
        L.zo_dequantize.argtypes = [C.c_int, C.c_void_p, C.c_void_p, sz, sz, C.c_void_p]
        _lib = L
    return _lib


def payload_bytes(qtype, K, N):
    return K * N if qtype == INT8 else (K * N + 1) // 2


def quantize_weights(w, qtype):
    """quantize(): w fp32 row-major [K][N] -> (payload uint8, scales fp32[N])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    K, N = w.shape
    payload = np.zeros(payload_bytes(qtype, K, N), dtype=np.uint8)
    scales = np.zeros(N, dtype=np.float32)
    lib().zo_quantize_weights(_vp(w), K, N, qtype, _vp(payload), _vp(scales))
    return payload, scales


def quantize_rows(x):
    """Per-row dynamic activation quantizer -> (codes int8 [M][K], scales fp32[M])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    q = np.zeros((M, K), dtype=np.int8)
    s = np.zeros(M, dtype=np.float32)
    lib().zo_quantize_rows(_vp(x), M, K, _vp(q), _vp(s))
    return q, s


def matmul_codes(q, row_scale, qtype, payload, col_scale, N, bias=None):
    q = np.ascontiguousarray(q, dtype=np.int8)
    M, K = q.shape
    row_scale = np.ascontiguousarray(row_scale, dtype=np.float32)
    col_scale = np.ascontiguousarray(col_scale, dtype=np.float32)
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    acc = np.zeros((M, N), dtype=np.int32)
    y = np.zeros((M, N), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().zo_matmul_codes(_vp(q), _vp(row_scale), M, K, qtype, _vp(payload), _vp(col_scale), N,
                          _vp(b), _vp(acc), _vp(y))
    return acc, y


def matmul(x, qtype, payload, col_scale, N, bias=None):
    """quantization::matmul (+ bias as QuantizedLinear::forward) ->
    (codes, row scales, int32 acc, fp32 y)."""
    q, s = quantize_rows(x)
    acc, y = matmul_codes(q, s, qtype, payload, col_scale, N, bias)
    return q, s, acc, y


def dequantize(qtype, payload, col_scale, K, N):
    out = np.zeros((K, N), dtype=np.float32)
    lib().zo_dequantize(qtype, _vp(np.ascontiguousarray(payload, dtype=np.uint8)),
                        _vp(np.ascontiguousarray(col_scale, dtype=np.float32)), K, N, _vp(out))
    return out


def unpack_codes(qtype, payload, K, N):
    """Column-major payload -> int8 codes [N][K]."""
    payload = np.asarray(payload, dtype=np.uint8)
    if qtype == INT8:
        return payload.view(np.int8).reshape(N, K).copy()
    lo = (payload & 0x0F).astype(np.int16)
    hi = (payload >> 4).astype(np.int16)
    nib = np.empty(payload.size * 2, dtype=np.int16)
    nib[0::2] = lo
    nib[1::2] = hi
    nib = nib[: K * N]
    nib = np.where(nib < 8, nib, nib - 16).astype(np.int8)
    return nib.reshape(N, K)


# ---------------------------------------------------------------------------
# .zyq byte format (quantization.cpp:240-311): restated for the checker.
# ---------------------------------------------------------------------------
ZYQ_MAGIC = 0x315A5951
ZYQ_VERSION = 1


def zyq_bytes(qtype, K, N, scales, payload):
    hdr = np.array([ZYQ_MAGIC, ZYQ_VERSION, qtype], dtype="<u4").tobytes()
    hdr += np.array([K, N, N], dtype="<u8").tobytes()
    body = np.asarray(scales, dtype="<f4").tobytes()
    body += np.array([len(payload)], dtype="<u8").tobytes()
    body += np.asarray(payload, dtype=np.uint8).tobytes()
    return hdr + body


# ---------------------------------------------------------------------------
# The compiled reference (oracle/_ref/libzyron_ref.so)
# ---------------------------------------------------------------------------

def ref_path():
    return os.path.join(HERE, "_ref", "libzyron_ref.so")


def ref_available():
    return os.path.exists(ref_path())


def ref():
    global _ref
    if _ref is None:
        R = C.CDLL(ref_path())
        sz = C.c_size_t
        vp = C.c_void_p
        R.ref_last_error.restype = C.c_char_p
        R.ref_set_threads.argtypes = [sz]
        R.ref_num_threads.restype = sz
        R.ref_quantize.argtypes = [vp, sz, sz, C.c_int, C.POINTER(vp)]
        R.ref_free.argtypes = [vp]
        R.ref_save_zyq.argtypes = [vp, vp, sz, C.POINTER(sz)]
        R.ref_load_zyq.argtypes = [vp, sz, C.POINTER(vp)]
        R.ref_scales.argtypes = [vp, vp]
        R.ref_codes.argtypes = [vp, vp]
        R.ref_bytes.argtypes = [vp]
        R.ref_bytes.restype = sz
        R.ref_matmul.argtypes = [vp, vp, sz, sz, vp]
        R.ref_linear_forward.argtypes = [vp, vp, vp, sz, sz, vp]
        R.ref_dequantize.argtypes = [vp, vp]
        R.ref_qlm_create.argtypes = [sz, sz, sz, sz, sz, sz, sz, C.c_int, C.c_int, C.c_int,
                                     C.c_uint32, C.c_int, C.POINTER(vp)]
        R.ref_qlm_free.argtypes = [vp]
        R.ref_qlm_save.argtypes = [vp, C.c_char_p]
        R.ref_qlm_load.argtypes = [C.c_char_p, C.POINTER(vp)]
        R.ref_qlm_forward.argtypes = [vp, vp, sz, vp]
        R.ref_qlm_generate_greedy.argtypes = [vp, vp, sz, sz, vp, C.POINTER(sz)]
        R.ref_checkpoint_save.argtypes = [C.c_char_p, sz, sz, sz, sz, sz, sz, sz, C.c_int, C.c_int, C.c_int,
                                          C.c_uint32]
        R.ref_qlm_generate.argtypes = [vp, vp, sz, sz, C.c_float, sz, C.c_float, C.c_float, sz, C.c_uint32, vp,
                                       C.POINTER(sz)]
        _ref = R
    return _ref


class RefError(Exception):
    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def _chk(rc):
    if rc != 0:
        raise RefError(rc, ref().ref_last_error().decode())


class RefMatrix:
    """A reference zyron::quantization::QuantizedMatrix."""

    def __init__(self, handle, K, N, qtype):
        self.h, self.K, self.N, self.qtype = handle, K, N, qtype

    @classmethod
    def quantize(cls, w, qtype):
        w = np.ascontiguousarray(w, dtype=np.float32)
        K, N = w.shape
        h = C.c_void_p()
        _chk(ref().ref_quantize(_vp(w), K, N, qtype, C.byref(h)))
        return cls(h, K, N, qtype)

    @classmethod
    def load_bytes(cls, data: bytes):
        buf = np.frombuffer(data, dtype=np.uint8)
        h = C.c_void_p()
        _chk(ref().ref_load_zyq(_vp(buf), len(data), C.byref(h)))
        K, N = np.frombuffer(data[12:28], dtype="<u8")
        qtype = int(np.frombuffer(data[8:12], dtype="<u4")[0])
        return cls(h, int(K), int(N), qtype)

    def __del__(self):
        if getattr(self, "h", None) and _ref is not None:
            _ref.ref_free(self.h)
            self.h = None

    def save_bytes(self) -> bytes:
        n = C.c_size_t()
        _chk(ref().ref_save_zyq(self.h, None, 0, C.byref(n)))
        buf = np.zeros(n.value, dtype=np.uint8)
        _chk(ref().ref_save_zyq(self.h, _vp(buf), n.value, C.byref(n)))
        return buf.tobytes()

    def scales(self):
        s = np.zeros(self.N, dtype=np.float32)
        _chk(ref().ref_scales(self.h, _vp(s)))
        return s

    def codes(self):
        c = np.zeros((self.N, self.K), dtype=np.int8)
        _chk(ref().ref_codes(self.h, _vp(c)))
        return c

    def payload(self):
        data = self.save_bytes()
        off = 4 * 3 + 8 * 3 + 4 * self.N + 8
        return np.frombuffer(data[off:], dtype=np.uint8).copy()

    def matmul(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        M = x.shape[0]
        y = np.zeros((M, self.N), dtype=np.float32)
        _chk(ref().ref_matmul(self.h, _vp(x), M, self.K, _vp(y)))
        return y

    def linear(self, x, bias=None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        M = x.shape[0]
        y = np.zeros((M, self.N), dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        _chk(ref().ref_linear_forward(self.h, _vp(b), _vp(x), M, self.K, _vp(y)))
        return y

    def dequantize(self):
        out = np.zeros((self.K, self.N), dtype=np.float32)
        _chk(ref().ref_dequantize(self.h, _vp(out)))
        return out


def ref_set_threads(n):
    ref().ref_set_threads(n)
    return int(ref().ref_num_threads())


class RefQlm:
    """A reference zyron::model::QuantizedLanguageModel (quantized_language_model.hpp)."""

    def __init__(self, handle, vocab):
        self.h, self.vocab = handle, vocab

    @classmethod
    def create(cls, vocab, hidden, layers, heads, kv_heads, ffn, max_seq, use_rope=True, use_rms_norm=True,
               tie=True, seed=0, qtype=INT8):
        """LanguageModel(config, seed) quantized to ``qtype``."""
        h = C.c_void_p()
        _chk(ref().ref_qlm_create(vocab, hidden, layers, heads, kv_heads, ffn, max_seq, int(use_rope),
                                  int(use_rms_norm), int(tie), seed, qtype, C.byref(h)))
        return cls(h, vocab)

    @classmethod
    def load(cls, path, vocab):
        h = C.c_void_p()
        _chk(ref().ref_qlm_load(str(path).encode(), C.byref(h)))
        return cls(h, vocab)

    def __del__(self):
        if getattr(self, "h", None) is not None and _ref is not None:
            _ref.ref_qlm_free(self.h)
            self.h = None

    def save(self, path):
        _chk(ref().ref_qlm_save(self.h, str(path).encode()))

    def forward(self, ids):
        """Logits [T][vocab] of forward(ids)."""
        a = np.ascontiguousarray(ids, dtype=np.uint64)
        out = np.zeros((a.size, self.vocab), dtype=np.float32)
        _chk(ref().ref_qlm_forward(self.h, _vp(a), a.size, _vp(out)))
        return out

    def generate(self, ids, max_new_tokens, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0,
                 no_repeat_ngram_size=0, seed=0):
        """generate(ids, GenerationConfig{...}) -> prompt + new tokens."""
        a = np.ascontiguousarray(ids, dtype=np.uint64)
        out = np.zeros(a.size + max_new_tokens + 1, dtype=np.uint64)
        n = C.c_size_t()
        _chk(ref().ref_qlm_generate(self.h, _vp(a), a.size, max_new_tokens, temperature, top_k, top_p,
                                    repetition_penalty, no_repeat_ngram_size, seed, _vp(out), C.byref(n)))
        return [int(t) for t in out[: n.value]]


def ref_tool_path():
    """The reference's zyron_quantize executable, built by oracle/Makefile."""
    return os.path.join(HERE, "_ref", "zyron_quantize")


def ref_checkpoint_save(path, vocab, hidden, layers, heads, kv_heads, ffn, max_seq, use_rope=True,
                        use_rms_norm=True, tie=True, seed=0):
    """A reference .zyron checkpoint with non-trivial parameter values
    (ref_harness.cpp: ref_checkpoint_save)."""
    _chk(ref().ref_checkpoint_save(str(path).encode(), vocab, hidden, layers, heads, kv_heads, ffn, max_seq,
                                   int(use_rope), int(use_rms_norm), int(tie), seed))


def ref_quantize_tool(checkpoint, output, bits=8):
    """Run the reference's zyron_quantize: (exit code, stdout, stderr)."""
    import subprocess

    p = subprocess.run([ref_tool_path(), "--checkpoint", str(checkpoint), "--output", str(output), "--bits",
                        str(bits)], capture_output=True, text=True, timeout=600)
    return p.returncode, p.stdout, p.stderr
