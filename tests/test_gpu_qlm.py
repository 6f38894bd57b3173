"""Device decode loop of QuantizedLanguageModel against the reference.

Fixtures (tests/golden/make_golden_qlm.py) hold .zyqmodel images written by
the reference's QuantizedLanguageModel::save, the reference's greedy
generation and the logits each new token was chosen from.  The quantized
matmuls are exact, but norms, softmax, GELU and attention sums are fp32 in a
different order (parallel reductions, CUDA's tanhf/expf), so logits are
compared with a tolerance and the greedy tokens must agree.
"""
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

# max |logit difference| allowed, relative to the logit range of the step
LOGIT_RTOL = 2e-3


@pytest.fixture(scope="module")
def qgold():
    return np.load(os.path.join(ROOT, "tests", "golden", "qlm_golden.npz"))


@pytest.fixture(params=["kernel_chain", "persistent"])
def decode_path(request, monkeypatch):
    """Both device decode loops: the chain of per-phase kernels replayed from
    CUDA graphs (default) and the persistent cooperative kernel
    (ZQ_LM_PERSISTENT=1)."""
    if request.param == "persistent":
        monkeypatch.setenv("ZQ_LM_PERSISTENT", "1")
    else:
        monkeypatch.delenv("ZQ_LM_PERSISTENT", raising=False)
    return request.param


@pytest.mark.parametrize("name", ["rope_gqa_int8", "rope_gqa_int4", "pe_layernorm_mha_int8", "rope_mqa_odd_int8"])
def test_greedy_generation_matches_reference(cuda, qgold, name, decode_path):
    from zyron_b200.qlm import GenerationConfig, QuantizedLanguageModel

    lm = QuantizedLanguageModel.load_bytes(qgold[f"{name}_model"].tobytes())
    prompt = qgold[f"{name}_prompt"]
    want = qgold[f"{name}_tokens"]
    ref_logits = qgold[f"{name}_logits"]
    n_new = want.size - prompt.size
    cfg = GenerationConfig(max_new_tokens=n_new, top_k=1)
    toks, logits = lm.generate(prompt.tolist(), cfg, return_logits=True)
    span = float(ref_logits.max() - ref_logits.min())
    err = float(np.abs(logits - ref_logits).max())
    assert err <= LOGIT_RTOL * span, f"{name}: max logit error {err:.3g} (range {span:.3g})"
    assert toks == want.tolist(), f"{name}: {toks} vs {want.tolist()}"
    # without per-step logits (graph replay in the kernel chain) the same tokens
    assert lm.generate(prompt.tolist(), cfg) == want.tolist()


def test_generation_stops_at_context(cuda, qgold, decode_path):
    from zyron_b200.qlm import GenerationConfig, QuantizedLanguageModel

    lm = QuantizedLanguageModel.load_bytes(qgold["rope_gqa_int8_model"].tobytes())
    max_seq = lm.config().max_sequence_length
    prompt = list(range(max_seq - 3))
    out = lm.generate(prompt, GenerationConfig(max_new_tokens=50, top_k=1))
    assert len(out) == max_seq
    full = list(range(max_seq))
    out2 = lm.generate(full, GenerationConfig(max_new_tokens=5, top_k=1))
    assert len(out2) == max_seq + 1  # the reference appends one token before stopping
    with pytest.raises(ValueError, match="prompt exceeds context"):
        lm.generate(full + [1], GenerationConfig(max_new_tokens=1, top_k=1))
    with pytest.raises(IndexError, match="token id out of range"):
        lm.generate([10**6], GenerationConfig(max_new_tokens=1, top_k=1))


def test_random_model_image_loads_in_reference(cuda, tmp_path):
    """The writer's .zyqmodel is the reference's format: the reference loads
    it and greedy decoding agrees with the device loop."""
    import ctypes as C

    from oracle import oracle as O
    from zyron_b200.qlm import Config, GenerationConfig, QuantizedLanguageModel, random_zyqmodel

    if not O.ref_available():
        pytest.skip("compiled reference not present")
    cfg = Config(vocab_size=128, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2, intermediate_size=128,
                 max_sequence_length=32)
    img = random_zyqmodel(cfg, seed=3)
    p = tmp_path / "r.zyqmodel"
    p.write_bytes(img)
    h = C.c_void_p()
    assert O.ref().ref_qlm_load(str(p).encode(), C.byref(h)) == 0, O.ref().ref_last_error()
    prompt = np.array([5, 9, 17, 3], dtype=np.uint64)
    out = np.zeros(prompt.size + 8, dtype=np.uint64)
    n = C.c_size_t()
    assert O.ref().ref_qlm_generate_greedy(h, C.c_void_p(prompt.ctypes.data), prompt.size, 8,
                                           C.c_void_p(out.ctypes.data), C.byref(n)) == 0
    O.ref().ref_qlm_free(h)
    lm = QuantizedLanguageModel.load_bytes(img)
    got = lm.generate(prompt.astype(np.int64).tolist(), GenerationConfig(max_new_tokens=8, top_k=1))
    assert got == out[: n.value].astype(np.int64).tolist()
