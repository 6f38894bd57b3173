"""Python mirror of ZYRON's ``QuantizedLanguageModel`` over the device decode
loop (``zq_lm_*`` in include/zq.h).

``QuantizedLanguageModel.load(path)`` reads the reference's ``.zyqmodel``
format (src/model/quantized_language_model.cpp:615-642) and keeps weights,
KV cache and activations on the GPU; ``generate(ids, config)`` is the
reference's generate (496-547) for every GenerationConfig.

``init_zyqmodel(config, seed)`` builds the ``.zyqmodel`` image of the
reference's ``LanguageModel(config, seed)`` quantized with
``QuantizedLanguageModel(model, type)``: the parameters are drawn with the
reference's generator, seeds and order (src/model/language_model.cpp:52-75),
so the image equals the reference's byte for byte.  ``random_zyqmodel``
builds one of the same shapes and init ranges -- Xavier-uniform linears with
bias 0 (src/nn/linear.cpp:13-44), U(-0.02, 0.02) embedding, unit norm
weights, an lm_head tied to the transposed embedding -- from numpy draws.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import struct

import numpy as np

from . import _lib
from ._lib import check, lib
from .quantization import Type, _stream_ptr, quantize

MODEL_MAGIC = 0x4D4C5A51  # "QZLM"
MODEL_VERSION = 1


@dataclasses.dataclass
class Config:
    """transformer::Config (include/zyron/transformer/config.hpp:10-25)."""

    vocab_size: int = 260
    hidden_size: int = 128
    num_layers: int = 2
    num_heads: int = 4
    num_kv_heads: int = 0
    intermediate_size: int = 512
    max_sequence_length: int = 128
    norm_eps: float = 1e-5
    use_rms_norm: bool = True
    causal: bool = True
    use_rope: bool = True
    tie_word_embeddings: bool = True
    rope_theta: float = 10000.0
    dropout: float = 0.0
    use_qat: bool = False
    qat_bits: int = 8

    def resolved_num_kv_heads(self):
        return self.num_heads if self.num_kv_heads == 0 else self.num_kv_heads


@dataclasses.dataclass
class GenerationConfig:
    """GenerationConfig (include/zyron/model/generation.hpp:12-20)."""

    max_new_tokens: int = 32
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    no_repeat_ngram_size: int = 0
    seed: int = 0


class QuantizedLanguageModel:
    def __init__(self, handle):
        self._h = handle
        info = _lib.LmInfo()
        check(lib().zq_lm_get_info(handle, C.byref(info)))
        self._info = info

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib._lib is not None:
            _lib._lib.zq_lm_destroy(h)
            self._h = None

    @classmethod
    def load_bytes(cls, data: bytes, stream=None):
        buf = np.frombuffer(data, dtype=np.uint8)
        h = C.c_void_p()
        check(lib().zq_lm_load(buf.ctypes.data_as(C.c_void_p) if buf.size else None, len(data),
                               _stream_ptr(stream), C.byref(h)))
        return cls(h)

    @classmethod
    def load(cls, path, stream=None):
        try:
            with open(path, "rb") as f:
                data = f.read()
        except OSError:
            raise _lib.ZQRuntimeError(f"ZYRON quantized model: failed to open: {path}")
        return cls.load_bytes(data, stream)

    def config(self):
        i = self._info
        return Config(vocab_size=i.vocab_size, hidden_size=i.hidden_size, num_layers=i.num_layers,
                      num_heads=i.num_heads, num_kv_heads=i.num_kv_heads, intermediate_size=i.intermediate_size,
                      max_sequence_length=i.max_sequence_length, norm_eps=i.norm_eps,
                      use_rms_norm=bool(i.use_rms_norm), causal=bool(i.causal), use_rope=bool(i.use_rope),
                      tie_word_embeddings=bool(i.tie_word_embeddings), rope_theta=i.rope_theta)

    def type(self):
        return Type(self._info.type)

    def set_persistent(self, on: bool) -> bool:
        """Greedy decoding as one persistent cooperative kernel (True) or the
        graph-replayed kernel chain (False, default); returns the old value."""
        prev = C.c_int()
        check(lib().zq_lm_set_option(self._h, 1, int(bool(on)), C.byref(prev)))  # ZQ_LM_OPT_PERSISTENT
        return bool(prev.value)

    def quantized_bytes(self):
        return self._info.quantized_bytes

    def float_reference_bytes(self):
        return self._info.float_reference_bytes

    def compression_ratio(self):
        q = self.quantized_bytes()
        return 0.0 if q == 0 else self.float_reference_bytes() / q

    def generate(self, input_ids, config: GenerationConfig = GenerationConfig(), stream=None, return_logits=False):
        """QuantizedLanguageModel::generate (496-547) for any GenerationConfig.
        Returns the prompt plus the new tokens; with ``return_logits`` also
        the [new, vocab] logits each new token was chosen from.  Greedy
        decoding (top_k == 1, with or without repetition penalty and n-gram
        block) runs entirely on the device; other configurations sample each
        step's logits on the host with the reference's sampler."""
        ids = np.ascontiguousarray(np.asarray(input_ids, dtype=np.int64))
        cap = ids.size + max(config.max_new_tokens, 0) + 1
        out = np.zeros(cap, dtype=np.int64)
        n = C.c_size_t()
        logits = None
        if return_logits:
            logits = np.zeros((max(config.max_new_tokens, 1), self._info.vocab_size), dtype=np.float32)
        cfg = _config_c(config)
        check(lib().zq_lm_generate(self._h, ids.ctypes.data_as(C.c_void_p) if ids.size else None, ids.size,
                                   C.byref(cfg), out.ctypes.data_as(C.c_void_p), cap, C.byref(n),
                                   None if logits is None else logits.ctypes.data_as(C.c_void_p),
                                   None if stream is None else C.c_void_p(stream.cuda_stream)))
        toks = [int(t) for t in out[: n.value]]
        if return_logits:
            return toks, logits[: n.value - ids.size]
        return toks


def _config_c(cfg: GenerationConfig):
    if cfg.max_new_tokens < 0 or cfg.top_k < 0 or cfg.no_repeat_ngram_size < 0:
        raise _lib.ZQInvalidArgument("zyron_b200: negative GenerationConfig count")
    return _lib.GenerationConfigC(int(cfg.max_new_tokens), float(cfg.temperature), int(cfg.top_k), float(cfg.top_p),
                                  float(cfg.repetition_penalty), int(cfg.no_repeat_ngram_size),
                                  int(cfg.seed) & 0xFFFFFFFF)


class Sampler:
    """sample_next (quantized_language_model.cpp:82-174) on the host, with the
    std::mt19937(seed) state that generate keeps across steps (520)."""

    def __init__(self, seed: int = 0):
        h = C.c_void_p()
        check(lib().zq_sampler_create(int(seed) & 0xFFFFFFFF, C.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib._lib is not None:
            _lib._lib.zq_sampler_destroy(h)
            self._h = None

    def next(self, logits, history, config: GenerationConfig) -> int:
        row = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1)
        hist = np.ascontiguousarray(np.asarray(history, dtype=np.int64))
        tok = C.c_int64()
        cfg = _config_c(config)
        check(lib().zq_sample_next(self._h, row.ctypes.data_as(C.c_void_p), row.size,
                                   hist.ctypes.data_as(C.c_void_p) if hist.size else None, hist.size, C.byref(cfg),
                                   C.byref(tok)))
        return int(tok.value)


# ---------------------------------------------------------------------------
# .zyqmodel writer (format of QuantizedLanguageModel::save, 615-625)
# ---------------------------------------------------------------------------

def _u32(v):
    return struct.pack("<I", int(v))


def _u64(v):
    return struct.pack("<Q", int(v))


def _f32(v):
    return struct.pack("<f", float(v))


def _tensor(a):
    if a is None or np.asarray(a).size == 0:
        return _u64(0) + _u64(0)
    a = np.ascontiguousarray(a, dtype="<f4")
    return _u64(a.ndim) + b"".join(_u64(d) for d in a.shape) + _u64(a.size) + a.tobytes()


def _config(c: Config):
    return (_u64(c.vocab_size) + _u64(c.hidden_size) + _u64(c.num_layers) + _u64(c.num_heads) +
            _u64(c.num_kv_heads) + _u64(c.intermediate_size) + _u64(c.max_sequence_length) + _f32(c.norm_eps) +
            _u32(c.use_rms_norm) + _u32(c.causal) + _u32(c.use_rope) + _u32(c.tie_word_embeddings) +
            _f32(c.rope_theta) + _f32(c.dropout) + _u32(c.use_qat) + _u64(c.qat_bits))


def init_zyqmodel(config: Config, seed: int = 42, qtype: Type = Type.Int8, stream=None) -> bytes:
    """QuantizedLanguageModel(LanguageModel(config, seed), qtype).save() as
    bytes: the parameters drawn as the reference's constructors draw them
    (language_model.cpp:52-75, tensor.cpp:165-172), weights quantized on the
    GPU (quantized_language_model.cpp:178-269).  See ``zq_lm_init_image``."""
    c = config
    cfg = _lib.LmConfigC(c.vocab_size, c.hidden_size, c.num_layers, c.num_heads, c.num_kv_heads,
                         c.intermediate_size, c.max_sequence_length, c.norm_eps, int(c.use_rms_norm), int(c.causal),
                         int(c.use_rope), int(c.tie_word_embeddings), c.rope_theta, c.dropout, int(c.use_qat),
                         c.qat_bits)
    L = lib()
    out = C.c_void_p()
    n = C.c_size_t()
    st = None if stream is None else C.c_void_p(stream.cuda_stream)
    check(L.zq_lm_init_image(C.byref(cfg), int(seed) & 0xFFFFFFFF, int(qtype), st, C.byref(out), C.byref(n), None))
    try:
        return C.string_at(out, n.value)
    finally:
        L.zq_free_buffer(out)


def random_zyqmodel(config: Config, seed: int = 0, qtype: Type = Type.Int8) -> bytes:
    """A .zyqmodel image of a randomly initialised model (see module doc).
    Weights are quantized on the GPU with the library's quantize()."""
    import torch

    c = config
    rng = np.random.default_rng(seed)
    H, V, F = c.hidden_size, c.vocab_size, c.intermediate_size
    kvh = c.resolved_num_kv_heads()
    hd = H // c.num_heads

    def q(w):
        return quantize(torch.from_numpy(np.ascontiguousarray(w, dtype=np.float32)).cuda(), qtype).save_bytes()

    def xavier(i, o):
        lim = np.float32(np.sqrt(np.float32(6.0) / np.float32(i + o)))
        return rng.uniform(-lim, lim, size=(i, o)).astype(np.float32)

    emb = rng.uniform(-0.02, 0.02, size=(V, H)).astype(np.float32)
    parts = [_u32(MODEL_MAGIC), _u32(MODEL_VERSION), _u32(int(qtype)), _config(c), q(emb)]
    pe = None
    if not c.use_rope:
        pe = np.zeros((c.max_sequence_length, H), dtype=np.float32)
        for pos in range(c.max_sequence_length):
            for i in range(0, H, 2):
                ang = np.float32(pos) / np.power(np.float32(10000.0), np.float32(i) / np.float32(H))
                pe[pos, i] = np.sin(ang)
                if i + 1 < H:
                    pe[pos, i + 1] = np.cos(ang)
    parts += [_tensor(pe), _tensor(np.ones(H, dtype=np.float32)), _u64(c.num_layers)]
    zeros = lambda n: np.zeros(n, dtype=np.float32)  # noqa: E731
    for _ in range(c.num_layers):
        nb = None if c.use_rms_norm else zeros(H)
        parts += [_u32(c.use_rms_norm), _tensor(np.ones(H, dtype=np.float32)), _tensor(nb),
                  _u32(c.use_rms_norm), _tensor(np.ones(H, dtype=np.float32)), _tensor(nb)]
        for (i, o) in [(H, H), (H, kvh * hd), (H, kvh * hd), (H, H), (H, F), (F, H)]:
            parts += [q(xavier(i, o)), _tensor(zeros(o))]
    head = np.ascontiguousarray(emb.T) if c.tie_word_embeddings else xavier(H, V)
    parts += [q(head), _tensor(zeros(V))]
    return b"".join(parts)
