"""Builds the engine in place (no pip install, no JIT cache):

  ns_fps_b200/libnsfps.so                      CUDA kernels + C ABI (nvcc, sm_100a)
  ns_fps_b200/yuezu_fps_module<EXT_SUFFIX>     pybind11 drop-in over the C ABI

Run ``python -m ns_fps_b200.build`` (or ``__graft_entry__.build()``).  Objects
are rebuilt only when a source or header is newer than the target.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")

LIB = os.path.join(HERE, "libnsfps.so")
EXT = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
MODULE = os.path.join(HERE, "yuezu_fps_module" + EXT)

CU_SOURCES = ["nsfps_setup.cu", "nsfps_loop.cu", "nsfps_rounds.cu", "nsfps_static.cu",
              "nsfps_group.cu", "nsfps_capi.cu"]
HEADERS = ["nsfps_internal.cuh", "nsfps_kernels.h", "nsfps_device.cuh"]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    # bit-exact float semantics: no multiply-add contraction anywhere
    "-fmad=false", "-Xcompiler", "-ffp-contract=off",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I" + INCLUDE, "-I" + CSRC,
]


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_lib(verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "nsfps.h")]
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if verbose_ptxas or _newer(o, [s] + headers):
            cmd = [NVCC, *NVCC_FLAGS, "-c", s, "-o", o]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd)
        objs.append(o)
    if _newer(LIB, objs):
        # only the extern "C" API (nsfps_*) is exported
        vs = os.path.join(BUILD, "exports.map")
        with open(vs, "w") as f:
            f.write("{ global: nsfps_*; local: *; };\n")
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs,
              "-Xlinker", "--version-script=" + vs,
              "-lcudart_static", "-lrt", "-lpthread", "-ldl"])
    return LIB


def build_module() -> str:
    src = os.path.join(CSRC, "yuezu_fps_module.cpp")
    if _newer(MODULE, [src, os.path.join(INCLUDE, "nsfps.h"), LIB]):
        import pybind11
        cxx = os.environ.get("CXX", "g++")
        _run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
              "-I" + pybind11.get_include(), "-I" + sysconfig.get_paths()["include"],
              "-I" + INCLUDE, src, "-o", MODULE, "-L" + HERE, "-lnsfps",
              "-Wl,-rpath,$ORIGIN"])
    return MODULE


def build(verbose_ptxas: bool = False) -> None:
    build_lib(verbose_ptxas)
    build_module()


if __name__ == "__main__":
    build(verbose_ptxas="-v" in sys.argv)
