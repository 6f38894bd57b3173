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


def test_generation_config_validation():
    from zyron_b200 import _lib
    from zyron_b200.qlm import GenerationConfig, _validate_generation

    info = _lib.LmInfo()
    info.vocab_size = 10
    with pytest.raises(ValueError, match="invalid temperature"):
        _validate_generation(GenerationConfig(temperature=0.0), info)
    with pytest.raises(ValueError, match="invalid top_p"):
        _validate_generation(GenerationConfig(top_p=1.5), info)
    with pytest.raises(ValueError, match="invalid repetition_penalty"):
        _validate_generation(GenerationConfig(repetition_penalty=0.5), info)
    with pytest.raises(ValueError, match="top_k exceeds vocabulary"):
        _validate_generation(GenerationConfig(top_k=11), info)
