"""Runs the C++20 drop-in's own test program (tests/cpp/test_quantization_api.cpp)
on the GPU: the zyron::quantization API over the C ABI, checked bit for bit
against the oracle."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def test_cpp_drop_in(cuda, tmp_path):
    from zyron_b200 import build

    build.build()
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), os.path.join(ROOT, "oracle", "liboracle.so")],
                   check=True, capture_output=True)
    exe = tmp_path / "test_quantization_api"
    pkg = os.path.join(ROOT, "zyron_b200")
    subprocess.run(["g++", "-std=c++20", "-O1", "-I", os.path.join(pkg, "cpp", "include"),
                    "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "cpp", "test_quantization_api.cpp"),
                    "-o", str(exe), "-L", pkg, "-lzyron_quant", "-lzyron_b200", "-L", os.path.join(ROOT, "oracle"),
                    "-loracle", f"-Wl,-rpath,{pkg}:{os.path.join(ROOT, 'oracle')}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout


@pytest.mark.parametrize("program,banner", [("test_phase5", "ZYRON Phase 5 tests: PASS"),
                                            ("test_final", "ZYRON final tests: PASS")])
def test_reference_tests_over_drop_in(cuda, program, banner):
    """The reference's own test programs (tests/test_phase5.cpp: quantize,
    matmul, QuantizedLinear, QuantizedLanguageModel; tests/test_final.cpp:
    .zyqmodel round trip, quantized batch generation), compiled unmodified
    with the reference's QuantizedLanguageModel and the rest of its sources,
    but with src/quantization replaced by the C++ drop-in (oracle/Makefile,
    target dropin): every quantized matmul they run goes through
    libzyron_b200.so on the GPU."""
    exe = os.path.join(ROOT, "oracle", "_ref", "dropin", program)
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/dropin not built (needs the reference sources)")
    ldd = subprocess.run(["ldd", exe], capture_output=True, text=True).stdout
    assert os.path.join("zyron_b200", "libzyron_b200.so") in ldd, ldd
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert banner in r.stdout
