"""zyron_quantize: a .zyron training checkpoint to a .zyqmodel quantized model.

Command-line mirror of the reference tool (tools/zyron_quantize.cpp:15-48):
same arguments, messages and exit codes, with the conversion done by the
library's ``zq_quantize_checkpoint`` (every weight quantized on the GPU,
output byte-identical to the reference tool's).

    python -m zyron_b200.zyron_quantize --checkpoint train.zyron --output model.zyqmodel [--bits 4|8]
"""
from __future__ import annotations

import ctypes as C
import sys

USAGE = "zyron_quantize --checkpoint <train.zyron> --output <model.zyqmodel> [--bits 4|8]\n"


class _ArgError(Exception):
    pass


def _parse(argv):
    """parse (zyron_quantize.cpp:17-31): same checks and messages."""
    inp = out = ""
    qtype = 1
    i = 0
    while i < len(argv):
        arg = argv[i]

        def need(name):
            nonlocal i
            if i + 1 >= len(argv):
                raise _ArgError(f"missing value for {name}")
            i += 1
            return argv[i]

        if arg == "--checkpoint":
            inp = need("--checkpoint")
        elif arg == "--output":
            out = need("--output")
        elif arg == "--bits":
            v = need("--bits")
            try:
                bits = int(v)
            except ValueError:
                raise _ArgError("stoull")
            if bits == 8:
                qtype = 1
            elif bits == 4:
                qtype = 2
            else:
                raise _ArgError("--bits must be 4 or 8")
        elif arg == "--help":
            sys.stdout.write(USAGE)
            raise SystemExit(0)
        else:
            raise _ArgError(f"unknown argument: {arg}")
        i += 1
    if not inp or not out:
        raise _ArgError("--checkpoint and --output are required")
    return inp, out, qtype


def quantize_checkpoint_bytes(data: bytes, qtype: int = 1, stream=None):
    """The .zyqmodel image of a .zyron checkpoint and its compression ratio."""
    from . import _lib

    L = _lib.lib()
    buf = C.create_string_buffer(data, len(data)) if data else None
    out = C.c_void_p()
    n = C.c_size_t()
    ratio = C.c_double()
    _lib.check(L.zq_quantize_checkpoint(buf, len(data), qtype, stream, C.byref(out), C.byref(n), C.byref(ratio)))
    try:
        return C.string_at(out, n.value), ratio.value
    finally:
        L.zq_free_buffer(out)


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    try:
        inp, outp, qtype = _parse(argv)
        try:
            with open(inp, "rb") as f:
                data = f.read()
        except OSError:
            raise _ArgError(f"ZYRON checkpoint: failed to open: {inp}")
        image, ratio = quantize_checkpoint_bytes(data, qtype)
        try:
            with open(outp, "wb") as f:
                f.write(image)
        except OSError:
            raise _ArgError(f"ZYRON quantized model: failed to open: {outp}")
        sys.stdout.write(f"ZYRON quantized model saved: {outp}\ncompression={ratio:g}x\n")
        return 0
    except Exception as e:  # the reference catches std::exception and prints what()
        sys.stderr.write(f"zyron_quantize error: {e}\n")
        return 1


if __name__ == "__main__":
    raise SystemExit(main())
