"""zyron_quantize parity: .zyron training checkpoint -> .zyqmodel.

The fixture (tests/golden/make_golden_checkpoint.py) holds checkpoints written
by the compiled reference's Checkpoint::save and what the reference's own
zyron_quantize tool (tools/zyron_quantize.cpp) made of them: the .zyqmodel
bytes and printed compression ratio of valid checkpoints (two model
configurations x INT8/INT4, checkpoint versions 1-3), and the error message of
damaged ones.

Damaged checkpoints are rejected on the host before any device work, so those
cases run without a GPU; converting a valid checkpoint quantizes every weight
on the GPU and must give the reference tool's bytes exactly.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
from make_golden_checkpoint import case_checkpoint  # noqa: E402


@pytest.fixture(scope="module")
def cgold():
    return np.load(os.path.join(ROOT, "tests", "golden", "checkpoint_golden.npz"))


def _message(stderr):
    prefix = "zyron_quantize error: "
    assert stderr.startswith(prefix), stderr
    return stderr[len(prefix):].rstrip("\n")


def test_damaged_checkpoints_match_reference_messages(native_lib, cgold):
    from zyron_b200 import _lib
    from zyron_b200.zyron_quantize import quantize_checkpoint_bytes

    names = [str(n) for n in cgold["bad_names"]]
    assert len(names) >= 15
    for tag in names:
        data = case_checkpoint(cgold, tag)
        want = _message(str(cgold[f"{tag}_stderr"]))
        with pytest.raises(_lib.ZQError) as e:
            quantize_checkpoint_bytes(data, 1)
        assert str(e.value) == want, tag


def test_cli_arguments_and_errors_match_reference(native_lib, cgold, tmp_path):
    """The command line: argument errors and a damaged checkpoint give the
    reference tool's messages on stderr and exit code 1."""
    src = tmp_path / "bad.zyron"
    src.write_bytes(case_checkpoint(cgold, "bad_adam_lr"))
    out = tmp_path / "o.zyqmodel"

    def cli(*args):
        p = subprocess.run([sys.executable, "-m", "zyron_b200.zyron_quantize", *args], cwd=ROOT,
                           capture_output=True, text=True, timeout=300)
        return p.returncode, p.stdout, p.stderr

    rc, so, se = cli("--checkpoint", str(src), "--output", str(out), "--bits", "8")
    assert (rc, so, se) == (1, "", str(cgold["bad_adam_lr_stderr"]))
    assert cli("--checkpoint", str(src), "--output", str(out), "--bits", "5") == (
        1, "", "zyron_quantize error: --bits must be 4 or 8\n")
    assert cli("--checkpoint", str(src)) == (1, "", "zyron_quantize error: --checkpoint and --output are required\n")
    assert cli("--bogus") == (1, "", "zyron_quantize error: unknown argument: --bogus\n")
    assert cli("--output") == (1, "", "zyron_quantize error: missing value for --output\n")
    missing = str(tmp_path / "none.zyron")
    assert cli("--checkpoint", missing, "--output", str(out)) == (
        1, "", f"zyron_quantize error: ZYRON checkpoint: failed to open: {missing}\n")
    assert not out.exists()


def test_init_image_rejects_bad_config(native_lib):
    """zq_lm_init_image validates the config as Config::validate does
    (config.hpp:32-66), with its messages, before any device work."""
    from zyron_b200 import _lib
    from zyron_b200.qlm import Config, init_zyqmodel

    with pytest.raises(_lib.ZQInvalidArgument, match="num_kv_heads must divide num_heads"):
        init_zyqmodel(Config(num_heads=4, num_kv_heads=3))
    with pytest.raises(_lib.ZQInvalidArgument, match="dimensions must be > 0"):
        init_zyqmodel(Config(num_layers=0))
    with pytest.raises(_lib.ZQInvalidArgument, match="RoPE requires an even attention head dimension"):
        init_zyqmodel(Config(hidden_size=12, num_heads=4))
    with pytest.raises(_lib.ZQInvalidArgument, match="type must be INT8 or INT4"):
        init_zyqmodel(Config(), qtype=3)


@pytest.mark.gpu
def test_quantized_model_bytes_match_reference_tool(cuda, cgold, tmp_path):
    from zyron_b200.zyron_quantize import quantize_checkpoint_bytes

    names = [str(n) for n in cgold["ok_names"]]
    assert len(names) == 7
    for tag in names:
        data = case_checkpoint(cgold, tag)
        qtype = 1 if int(cgold[f"{tag}_bits"]) == 8 else 2
        got, ratio = quantize_checkpoint_bytes(data, qtype)
        want = cgold[f"{tag}_zyqmodel"].tobytes()
        assert len(got) == len(want), tag
        assert got == want, f"{tag}: first difference at byte {next(i for i in range(len(got)) if got[i] != want[i])}"
        assert str(cgold[f"{tag}_stdout"]) == f"ZYRON quantized model saved: <output>\ncompression={ratio:g}x\n"


@pytest.mark.gpu
def test_cli_end_to_end_and_device_decode(cuda, cgold, tmp_path):
    """The command line writes the reference tool's file, and the device
    decode loop runs it with the reference's greedy tokens."""
    from oracle import oracle as O
    from zyron_b200.qlm import GenerationConfig, QuantizedLanguageModel

    for tag in ("ok_rope_rms_tied_gqa_int8", "ok_pe_layernorm_untied_int4"):
        src = tmp_path / f"{tag}.zyron"
        src.write_bytes(case_checkpoint(cgold, tag))
        dst = tmp_path / f"{tag}.zyqmodel"
        bits = str(int(cgold[f"{tag}_bits"]))
        p = subprocess.run([sys.executable, "-m", "zyron_b200.zyron_quantize", "--checkpoint", str(src), "--output",
                            str(dst), "--bits", bits], cwd=ROOT, capture_output=True, text=True, timeout=300)
        assert p.returncode == 0, p.stderr
        assert p.stdout == str(cgold[f"{tag}_stdout"]).replace("<output>", str(dst))
        assert dst.read_bytes() == cgold[f"{tag}_zyqmodel"].tobytes()
        lm = QuantizedLanguageModel.load(dst)
        prompt = [1, 5, 2, 7]
        got = lm.generate(prompt, GenerationConfig(max_new_tokens=6, top_k=1))
        if O.ref_available():
            ref = O.RefQlm.load(dst, lm.config().vocab_size)
            assert got == ref.generate(prompt, 6, top_k=1)
