"""Build the in-tree native libraries of zyron_b200.

* ``zyron_b200/libzyron_b200.so`` -- the CUDA kernels + C ABI (include/zq.h),
  compiled for sm_100a only.
* ``zyron_b200/libzyron_quant.so`` -- the C++20 drop-in of
  ``zyron::quantization`` (zyron_b200/cpp) over that C ABI.

nvcc cross-compiles without a GPU, so this runs on any machine with CUDA 12.9.
Usage: ``python -m zyron_b200.build [--force]``.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
CPP = os.path.join(HERE, "cpp")
LIB = os.path.join(HERE, "libzyron_b200.so")
QLIB = os.path.join(HERE, "libzyron_quant.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

CU_SOURCES = ["zq_api.cu", "zq_quant.cu", "zq_gemv.cu", "zq_gemm_sm100.cu", "zq_skinny_sm100.cu", "zq_noalloc.cu",
              "zq_lm.cu", "zq_sharded.cu"]
CU_HEADERS = ["zq_common.cuh", "zq_dot.cuh", "zq_tcgen05.cuh", "zq_kernels.h", "zq_internal.h"]
# Host-only C++ of the library, built by g++ with the reference's own Release
# flags (-std=c++20 -O3 -DNDEBUG): zq_sample.cpp restates the reference's
# token sampler, whose std::sort order and std::mt19937 draws come from the
# C++ standard library, and zq_checkpoint.cpp writes the sinusoidal position
# table with the same libm calls as the reference.
HOST_SOURCES = ["zq_sample.cpp", "zq_checkpoint.cpp"]
HOST_FLAGS = ["-std=c++20", "-O3", "-DNDEBUG", "-fPIC"]
CPP_SOURCES = ["src/quantization.cpp", "src/quantized_linear.cpp", "src/tensor.cpp"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-Xptxas", "-O3",
    # exact IEEE arithmetic: no fast-math, keep denormals, correctly rounded div
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true",
]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_cuda(force=False):
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES]
    hsrcs = [os.path.join(CSRC, s) for s in HOST_SOURCES]
    deps = srcs + hsrcs + [os.path.join(CSRC, h) for h in CU_HEADERS] + [os.path.join(ROOT, "include", "zq.h")]
    if not force and not _newer(LIB, deps):
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for s in srcs:
        o = os.path.join(objdir, os.path.basename(s) + ".o")
        _run([NVCC, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-c", s, "-o", o])
        objs.append(o)
    for s in hsrcs:
        o = os.path.join(objdir, os.path.basename(s) + ".o")
        _run(["g++", *HOST_FLAGS, "-I", os.path.join(ROOT, "include"), "-c", s, "-o", o])
        objs.append(o)
    _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs, "-cudart", "static",
          "-ldl"])
    return LIB


def build_cpp(force=False):
    srcs = [os.path.join(CPP, s) for s in CPP_SOURCES]
    if not all(os.path.exists(s) for s in srcs):
        return None
    hdr_root = os.path.join(CPP, "include")
    deps = srcs + [os.path.join(ROOT, "include", "zq.h"), LIB]
    for d, _, fs in os.walk(hdr_root):
        deps += [os.path.join(d, f) for f in fs]
    if not force and not _newer(QLIB, deps):
        return QLIB
    _run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-I", hdr_root, "-I", os.path.join(ROOT, "include"),
          *srcs, "-o", QLIB, "-L", HERE, "-lzyron_b200", "-Wl,-rpath,$ORIGIN"])
    return QLIB


def build(force=False):
    build_cuda(force)
    build_cpp(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
