"""Generate tests/golden/qlm_golden.npz from the ZYRON reference itself.

For a few small model configurations the compiled reference
(oracle/_ref/libzyron_ref.so, built by oracle/Makefile from the reference's
sources) builds LanguageModel(config, seed), converts it to a
QuantizedLanguageModel and saves the .zyqmodel image.  Recorded per model:
the image, a prompt, the reference's greedy generation
(generate with top_k = 1), and the last-row logits of forward() on every
prefix that chose a new token.  Also recorded: damaged .zyqmodel images with
the exception message the reference's load() raises on each.

Usage: python tests/golden/make_golden_qlm.py
"""
from __future__ import annotations

import ctypes as C
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

# name: (vocab, hidden, layers, heads, kv_heads, ffn, max_seq, rope, rms, seed, type)
MODELS = {
    "rope_gqa_int8": (96, 64, 2, 4, 2, 128, 48, 1, 1, 77, 1),
    "rope_gqa_int4": (96, 64, 2, 4, 2, 128, 48, 1, 1, 78, 2),
    "pe_layernorm_mha_int8": (80, 32, 2, 4, 4, 64, 40, 0, 0, 79, 1),
    "rope_mqa_odd_int8": (101, 48, 3, 6, 1, 96, 40, 1, 1, 80, 1),
}
N_NEW = 12


def ref_model(spec):
    vocab, hidden, layers, heads, kv, ffn, max_seq, rope, rms, seed, qt = spec
    h = C.c_void_p()
    rc = O.ref().ref_qlm_create(vocab, hidden, layers, heads, kv, ffn, max_seq, rope, rms, 1, seed, qt,
                                C.byref(h))
    if rc:
        raise RuntimeError(O.ref().ref_last_error().decode())
    return h


def save_bytes(h):
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.zyqmodel")
        if O.ref().ref_qlm_save(h, p.encode()):
            raise RuntimeError(O.ref().ref_last_error().decode())
        return open(p, "rb").read()


def load_message(data: bytes):
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.zyqmodel")
        open(p, "wb").write(data)
        h = C.c_void_p()
        rc = O.ref().ref_qlm_load(p.encode(), C.byref(h))
        if rc == 0:
            O.ref().ref_qlm_free(h)
            return 0, ""
        return rc, O.ref().ref_last_error().decode()


def forward_last(h, ids, vocab):
    ids = np.asarray(ids, dtype=np.uint64)
    out = np.zeros((ids.size, vocab), dtype=np.float32)
    rc = O.ref().ref_qlm_forward(h, C.c_void_p(ids.ctypes.data), ids.size, C.c_void_p(out.ctypes.data))
    if rc:
        raise RuntimeError(O.ref().ref_last_error().decode())
    return out[-1]


def generate(h, prompt, n_new):
    ids = np.asarray(prompt, dtype=np.uint64)
    out = np.zeros(ids.size + n_new + 1, dtype=np.uint64)
    n = C.c_size_t()
    rc = O.ref().ref_qlm_generate_greedy(h, C.c_void_p(ids.ctypes.data), ids.size, n_new,
                                         C.c_void_p(out.ctypes.data), C.byref(n))
    if rc:
        raise RuntimeError(O.ref().ref_last_error().decode())
    return out[: n.value].astype(np.int64)


def damaged(good: bytes):
    b = bytearray(good)
    cases = [("empty", b""), ("short", bytes(b[:10]))]
    x = bytearray(b); x[0] ^= 0xFF; cases.append(("bad_magic", bytes(x)))
    x = bytearray(b); x[4] = 9; cases.append(("bad_version", bytes(x)))
    x = bytearray(b); x[8] = 5; cases.append(("bad_type", bytes(x)))
    # config starts at 12: vocab, hidden, layers, heads, kv, ffn, max_seq (u64 each)
    x = bytearray(b); x[12 + 8:12 + 16] = (30).to_bytes(8, "little"); cases.append(("hidden_not_divisible", bytes(x)))
    x = bytearray(b); x[12 + 32:12 + 40] = (3).to_bytes(8, "little"); cases.append(("kv_heads_bad", bytes(x)))
    x = bytearray(b); x[12:20] = (0).to_bytes(8, "little"); cases.append(("zero_vocab", bytes(x)))
    cases.append(("truncated_mid", bytes(b[: len(b) // 2])))
    cases.append(("truncated_tail", bytes(b[:-3])))
    out = []
    for name, data in cases:
        code, msg = load_message(data)
        out.append((name, data, code, msg))
    return out


def main():
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libzyron_ref.so is missing: run make -C oracle REF=<reference>")
    O.ref_set_threads(os.cpu_count() or 1)
    arrays = {}
    rng = np.random.default_rng(4242)
    for name, spec in MODELS.items():
        vocab = spec[0]
        h = ref_model(spec)
        img = save_bytes(h)
        prompt = rng.integers(0, vocab, size=7).astype(np.int64)
        toks = generate(h, prompt, N_NEW)
        logits = np.stack([forward_last(h, toks[: prompt.size + i], vocab) for i in range(toks.size - prompt.size)])
        arrays[f"{name}_model"] = np.frombuffer(img, dtype=np.uint8)
        arrays[f"{name}_prompt"] = prompt
        arrays[f"{name}_tokens"] = toks
        arrays[f"{name}_logits"] = logits
        O.ref().ref_qlm_free(h)
    arrays["models"] = np.array(list(MODELS))
    h = ref_model(MODELS["rope_gqa_int8"])
    cases = damaged(save_bytes(h))
    O.ref().ref_qlm_free(h)
    arrays["bad_names"] = np.array([c[0] for c in cases])
    arrays["bad_codes"] = np.array([c[2] for c in cases], dtype=np.int32)
    arrays["bad_msgs"] = np.array([c[3] for c in cases])
    for name, data, _, _ in cases:
        arrays[f"bad_{name}"] = np.frombuffer(data, dtype=np.uint8)
    out = os.path.join(HERE, "qlm_golden.npz")
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({os.path.getsize(out)} bytes)")
    for c in cases:
        print(c[0], c[2], c[3])


if __name__ == "__main__":
    main()
