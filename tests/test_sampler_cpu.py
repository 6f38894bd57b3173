"""The host sampler (zq_sample_next, zq_sample.cpp) against the compiled
reference, without a GPU.

The reference's generate (src/model/quantized_language_model.cpp:503-547)
calls forward() on the whole sequence and sample_next (82-174) on the last
row's logits each step, with one std::mt19937(seed) for the whole call.  Here
the same loop runs with the reference's own forward() for the logits and the
library's sampler for the choice; the token streams must be identical to the
reference's generate for every GenerationConfig, which pins the sampler bit
for bit: repetition penalty, n-gram block (including the fall back to the raw
logits when every token is blocked), softmax, sort order, top-k, top-p and
the draws.
"""
import numpy as np
import pytest

from oracle import oracle as O

if not O.ref_available():
    pytest.skip("compiled reference (oracle/_ref) not present", allow_module_level=True)

CONFIGS = [
    dict(top_k=1, repetition_penalty=1.3),
    dict(top_k=1, no_repeat_ngram_size=2),
    dict(top_k=1, repetition_penalty=1.5, no_repeat_ngram_size=3),
    dict(top_k=8, top_p=0.9, seed=5),
    dict(top_k=0, top_p=1.0, seed=3),
    dict(top_k=40, top_p=0.5, repetition_penalty=1.2, no_repeat_ngram_size=3, seed=7),
    dict(top_k=0, top_p=0.95, repetition_penalty=2.0, no_repeat_ngram_size=1, seed=11),
    dict(top_k=3, top_p=1.0, temperature=0.7, seed=4294967295),
]


@pytest.fixture(scope="module")
def ref_models():
    return {
        "rope_gqa": (O.RefQlm.create(101, 64, 2, 4, 2, 128, 48, seed=7), [5, 17, 3, 99, 42, 8, 8, 61]),
        # 8-token vocabulary: no_repeat_ngram_size = 1 blocks every token after
        # a few steps, which takes the reference's raw-logits fall-back
        "tiny_vocab": (O.RefQlm.create(8, 32, 1, 2, 1, 64, 40, seed=2), [1, 2, 3]),
    }


def _replay(model, prompt, n_new, cfg):
    from zyron_b200.qlm import GenerationConfig, Sampler

    gc = GenerationConfig(max_new_tokens=n_new, **cfg)
    s = Sampler(gc.seed)
    toks = list(prompt)
    for _ in range(n_new):
        logits = model.forward(toks)[-1]
        toks.append(s.next(logits, toks, gc))
    return toks


@pytest.mark.parametrize("model", ["rope_gqa", "tiny_vocab"])
@pytest.mark.parametrize("cfg", CONFIGS, ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
def test_sampler_matches_reference_generate(native_lib, ref_models, model, cfg):
    m, prompt = ref_models[model]
    if cfg.get("top_k", 0) > m.vocab:
        pytest.skip("top_k above the vocabulary")
    n_new = 16
    want = m.generate(prompt, n_new, **cfg)
    got = _replay(m, prompt, n_new, cfg)
    assert got == want


def test_sampler_blocked_everything_falls_back_to_raw_logits(native_lib):
    """Every token blocked: the raw logits decide (sample_next 120-128)."""
    from zyron_b200.qlm import GenerationConfig, Sampler

    logits = np.array([0.5, 2.0, -1.0, 1.5], dtype=np.float32)
    cfg = GenerationConfig(top_k=1, repetition_penalty=3.0, no_repeat_ngram_size=1)
    # history holds every id: all blocked, and the penalty is not applied
    assert Sampler(0).next(logits, [0, 1, 2, 3], cfg) == 1


def test_sampler_non_finite_logits_choose_token_zero(native_lib):
    """A NaN logit or a +inf maximum makes the softmax denominator non-finite:
    the reference returns token 0 (136)."""
    from zyron_b200.qlm import GenerationConfig, Sampler

    cfg = GenerationConfig(top_k=0, seed=1)
    assert Sampler(0).next(np.array([1.0, np.nan, 3.0], np.float32), [0], cfg) == 0
    assert Sampler(0).next(np.array([1.0, np.inf, 3.0], np.float32), [0], cfg) == 0
    assert Sampler(0).next(np.array([-np.inf] * 3, np.float32), [0], cfg) == 0
    # -inf logits alone are fine: they get probability 0
    assert Sampler(0).next(np.array([-np.inf, 2.0, -np.inf], np.float32), [0], GenerationConfig(top_k=1)) == 1
