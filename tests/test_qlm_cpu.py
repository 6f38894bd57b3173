"""QuantizedLanguageModel load on the host: damaged .zyqmodel images are
rejected with the reference's status and message before any device work
(fixtures from tests/golden/make_golden_qlm.py)."""
import ctypes as C
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def qgold():
    return np.load(os.path.join(ROOT, "tests", "golden", "qlm_golden.npz"))


def test_damaged_zyqmodel_matches_reference(native_lib, qgold):
    L = native_lib
    for name, code, msg in zip(qgold["bad_names"], qgold["bad_codes"], qgold["bad_msgs"]):
        data = np.ascontiguousarray(qgold[f"bad_{name}"], dtype=np.uint8)
        h = C.c_void_p()
        rc = L.zq_lm_load(data.ctypes.data_as(C.c_void_p) if data.size else None, data.size, None, C.byref(h))
        assert rc == int(code), (name, rc, L.zq_last_error())
        assert L.zq_last_error().decode() == str(msg), name


def test_generation_config_validation(native_lib):
    """validate_generation_config (quantized_language_model.cpp:71-80) and the
    top_k check (517) run in the C library, with the reference's messages."""
    from zyron_b200.qlm import GenerationConfig, Sampler

    s = Sampler(0)
    row = np.zeros(10, dtype=np.float32)
    for cfg, msg in [(GenerationConfig(temperature=0.0), "invalid temperature"),
                     (GenerationConfig(temperature=float("inf")), "invalid temperature"),
                     (GenerationConfig(top_p=1.5), "invalid top_p"),
                     (GenerationConfig(top_p=0.0), "invalid top_p"),
                     (GenerationConfig(repetition_penalty=0.5), "invalid repetition_penalty"),
                     (GenerationConfig(repetition_penalty=float("nan")), "invalid repetition_penalty"),
                     (GenerationConfig(top_k=11), "top_k exceeds vocabulary")]:
        with pytest.raises(ValueError, match=msg):
            s.next(row, [1, 2], cfg)
