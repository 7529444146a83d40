"""Build the native parts of winnex-madhava-b200 in-tree.

Produces, inside winnex-madhava_b200/winnex_madhava/:
  * libwinnex_madhava_b200.so   -- CUDA kernels + C ABI (sm_100a), from csrc/*.cu
  * _winnex_madhava<ext>.so     -- pybind11 module over the C ABI (py_module.cpp)

Usage: python winnex-madhava_b200/build.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "winnex_madhava")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(PKG, "libwinnex_madhava_b200.so")
EXT = os.path.join(PKG, "_winnex_madhava" + sysconfig.get_config_var("EXT_SUFFIX"))

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CU_SOURCES = ["capi.cu", "index.cu", "scan_simt.cu", "select.cu", "scan_tc.cu", "scan_tc2.cu", "scan_stream.cu", "scan_tc_bf16.cu", "ivf.cu", "ivf_f32.cu", "noalloc.cu", "persist.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INCLUDE, "-I" + CSRC,
                     "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force: bool = False) -> None:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(INCLUDE, "winnex_madhava_b200.h"))
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        if force or _stale(o, [s] + headers):
            _run([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o])
        objs.append(o)
    if force or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-Xlinker", "-soname=libwinnex_madhava_b200.so"])
    import pybind11

    py_src = os.path.join(CSRC, "py_module.cpp")
    if force or _stale(EXT, [py_src, LIB] + headers):
        _run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I" + pybind11.get_include(),
              "-I" + sysconfig.get_paths()["include"], "-I" + INCLUDE, py_src, "-o", EXT,
              "-L" + PKG, "-lwinnex_madhava_b200", "-Wl,-rpath,$ORIGIN"])


if __name__ == "__main__":
    build(force="--force" in sys.argv)
