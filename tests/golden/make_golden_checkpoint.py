"""Writes tests/golden/checkpoint_golden.npz: .zyron checkpoints written by
the compiled reference (oracle/_ref, Checkpoint::save through
ref_harness.cpp) and what the reference's own zyron_quantize tool
(tools/zyron_quantize.cpp, built unmodified by oracle/Makefile) makes of them.

Cases:
  ok_*      valid checkpoints -> the tool's .zyqmodel bytes and printed ratio;
            two model configurations x INT8/INT4, plus the older checkpoint
            versions 1-3 (the same file rewritten without the fields those
            versions lack, checkpoint.cpp:43-71);
  bad_*     damaged checkpoints -> the tool's exit code and error message;
            the damaged bytes are not stored: damaged_cases() rebuilds them
            from the rope_rms_tied_gqa checkpoint.

Run from the repository root after `make -C oracle ref`:
    python tests/golden/make_golden_checkpoint.py
"""
import os
import struct
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

# (vocab, hidden, layers, heads, kv_heads, ffn, max_seq, rope, rms, tie, seed)
MODELS = {
    "rope_rms_tied_gqa": (40, 16, 2, 2, 1, 32, 16, True, True, True, 3),
    # odd vocabulary (INT4 columns straddle bytes), LayerNorm, sinusoidal PE,
    # untied lm_head; kv_heads == heads so the file also reads as version 1
    "pe_layernorm_untied": (37, 24, 1, 3, 3, 40, 12, False, False, False, 5),
}


def split_v4(b):
    """(config fields, rest) of a version-4 checkpoint (checkpoint.cpp:28-42)."""
    assert struct.unpack_from("<II", b, 0) == (0x4E52595A, 4)
    off = 8
    f = {}
    for name, fmt in [("vocab", "Q"), ("hidden", "Q"), ("layers", "Q"), ("heads", "Q"), ("ffn", "Q"),
                      ("max_seq", "Q"), ("eps", "f"), ("rms", "I"), ("causal", "I"), ("kv", "Q"), ("rope", "I"),
                      ("tie", "I"), ("theta", "f"), ("dropout", "f"), ("qat", "I"), ("qat_bits", "Q")]:
        f[name] = struct.unpack_from("<" + fmt, b, off)[0]
        off += struct.calcsize("<" + fmt)
    return f, b[off:]


def join(f, rest, version):
    out = struct.pack("<II", 0x4E52595A, version)
    out += struct.pack("<QQQQQQfII", f["vocab"], f["hidden"], f["layers"], f["heads"], f["ffn"], f["max_seq"],
                       f["eps"], f["rms"], f["causal"])
    if version >= 2:
        out += struct.pack("<QIIf", f["kv"], f["rope"], f["tie"], f["theta"])
        if version >= 3:
            out += struct.pack("<f", f["dropout"])
            if version >= 4:
                out += struct.pack("<IQ", f["qat"], f["qat_bits"])
    return out + rest


def header_offsets():
    """Byte offsets of the training state after a version-4 config (the config
    ends at byte 104; checkpoint.cpp:121-130)."""
    base = 8 + 96
    return {"lr": base + 16, "beta1": base + 20, "warmup": base + 48, "total": base + 56, "params": base + 68}


def vector_offsets(b):
    """Offsets of the parameter, first-moment and second-moment tensor vectors
    and of the tokenizer length field."""
    off = header_offsets()["params"]
    starts = []
    for _ in range(3):
        starts.append(off)
        n = struct.unpack_from("<Q", b, off)[0]
        off += 8
        for _ in range(n):
            rank = struct.unpack_from("<Q", b, off)[0]
            off += 8 + 8 * rank
            cnt = struct.unpack_from("<Q", b, off)[0]
            off += 8 + 4 * cnt
    return starts, off


def damaged_cases(a):
    """Damaged variants of the version-4 checkpoint `a` (whose first
    parameter, the embedding, is [40, 16])."""
    fa, resta = split_v4(a)
    offs = header_offsets()
    (p0, m0, _), to = vector_offsets(a)

    def patched(*edits):
        b = bytearray(a)
        for off, fmt, value in edits:
            struct.pack_into("<" + fmt, b, off, value)
        return bytes(b)

    tb = a[to + 8:]
    pad_len = struct.unpack_from("<I", tb, 16)[0]  # after magic, version, vocab size, merge count
    tb2 = tb[:16] + struct.pack("<I", 0) + tb[20 + pad_len:]
    return {
        "empty": b"",
        "magic": patched((0, "I", 0x12345678)),
        "version5": patched((4, "I", 5)),
        "truncated_header": a[:60],
        "truncated_params": a[: offs["params"] + 400],
        "truncated_tokenizer": a[:-10],
        "heads_not_dividing": join(dict(fa, heads=5), resta, 4),
        "qat_bits": join(dict(fa, qat_bits=6), resta, 4),
        "adam_lr": patched((offs["lr"], "f", -1.0)),
        "adam_beta1": patched((offs["beta1"], "f", 1.0)),
        "scheduler_warmup": patched((offs["warmup"], "Q", 500)),
        "tensor_size": patched((p0 + 16, "Q", 16)),
        "param_shape": patched((p0 + 16, "Q", 16), (p0 + 24, "Q", 40)),
        "moment_shape": patched((m0 + 16, "Q", 16), (m0 + 24, "Q", 40)),
        "config_vs_params": join(dict(fa, tie=0), resta, 4),
        "tokenizer_missing": a[:to] + struct.pack("<Q", 0),
        "tokenizer_magic": a[:to + 8] + b"XXXX" + tb[4:],
        "tokenizer_special_empty": a[:to] + struct.pack("<Q", len(tb2)) + tb2,
    }


def case_checkpoint(g, tag):
    """The checkpoint bytes of case `tag` of the fixture `g`."""
    if tag.startswith("bad_"):
        return damaged_cases(case_checkpoint(g, "ok_rope_rms_tied_gqa_int8"))[tag[4:]]
    if tag.startswith("ok_version"):
        f, rest = split_v4(case_checkpoint(g, "ok_pe_layernorm_untied_int8"))
        return join(f, rest, int(tag[len("ok_version"):]))
    return g[f"{tag.replace('_int4', '_int8')}_checkpoint"].tobytes()


def main():
    if not O.ref_available() or not os.path.exists(O.ref_tool_path()):
        raise SystemExit("build the reference first: make -C oracle ref")
    out = {}
    tmp = tempfile.mkdtemp()
    ck = {}
    for name, (V, H, L, nh, kv, F, T, rope, rms, tie, seed) in MODELS.items():
        p = os.path.join(tmp, name + ".zyron")
        O.ref_checkpoint_save(p, V, H, L, nh, kv, F, T, rope, rms, tie, seed)
        ck[name] = open(p, "rb").read()

    def run(tag, data, bits):
        src = os.path.join(tmp, tag + ".zyron")
        dst = os.path.join(tmp, tag + ".zyqmodel")
        with open(src, "wb") as fh:
            fh.write(data)
        if os.path.exists(dst):
            os.remove(dst)
        rc, so, se = O.ref_quantize_tool(src, dst, bits)
        out[f"{tag}_checkpoint"] = np.frombuffer(data, dtype=np.uint8)
        out[f"{tag}_bits"] = np.array(bits)
        out[f"{tag}_rc"] = np.array(rc)
        out[f"{tag}_stdout"] = np.array(so.replace(dst, "<output>"))
        out[f"{tag}_stderr"] = np.array(se)
        if rc == 0:
            out[f"{tag}_zyqmodel"] = np.frombuffer(open(dst, "rb").read(), dtype=np.uint8)
        return rc, se

    ok = []
    for name, data in ck.items():
        for bits in (8, 4):
            tag = f"ok_{name}_int{bits}"
            assert run(tag, data, bits)[0] == 0, tag
            ok.append(tag)
    f, rest = split_v4(ck["pe_layernorm_untied"])
    for v in (1, 2, 3):
        tag = f"ok_version{v}"
        rc, se = run(tag, join(f, rest, v), 8)
        assert rc == 0, (tag, se)
        ok.append(tag)

    a = ck["rope_rms_tied_gqa"]
    assert struct.unpack_from("<QQ", a, vector_offsets(a)[0][0] + 16) == (40, 16)
    names = []
    for k, v in damaged_cases(a).items():
        tag = f"bad_{k}"
        rc, se = run(tag, v, 8)
        assert rc != 0, k
        del out[f"{tag}_checkpoint"]  # rebuilt from ok_rope_rms_tied_gqa by damaged_cases()
        names.append(tag)
    for name in MODELS:  # stored once, under the INT8 case
        del out[f"ok_{name}_int4_checkpoint"]
    for v in (1, 2, 3):  # rebuilt from pe_layernorm_untied by case_checkpoint()
        del out[f"ok_version{v}_checkpoint"]
    out["ok_names"] = np.array(ok)
    out["bad_names"] = np.array(names)
    dst = os.path.join(ROOT, "tests", "golden", "checkpoint_golden.npz")
    np.savez_compressed(dst, **out)
    for n in names:
        print(n, repr(str(out[f"{n}_stderr"])))
    print("wrote", dst, os.path.getsize(dst), "bytes")


if __name__ == "__main__":
    main()
