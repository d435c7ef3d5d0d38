"""Builds the native parts of subq_audio in place (sm_100a only).

  subq_audio/libsubq_b200.so      C ABI (include/kernels.hpp): scan kernels,
                                  C++ engine, arena and safetensors loader
  subq_audio/_C<ext-suffix>       pybind11 module over the engine

Usage: python build.py [--force]
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
PKG = os.path.join(HERE, "subq_audio")
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

LIB = os.path.join(PKG, "libsubq_b200.so")
EXT = os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-diag-suppress", "177"]


def _sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    cpp = [os.path.join(CSRC, "engine", f) for f in ("arena.cpp", "engine.cpp", "safetensors.cpp")]
    return cu, cpp


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
            glob.glob(os.path.join(INCLUDE, "*.hpp")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_lib(force=False, verbose=False) -> str:
    cu, cpp = _sources()
    if force or _stale(LIB, cu + cpp + _headers() + [__file__]):
        tmp = LIB + ".tmp"
        cmd = [NVCC, *ARCH_FLAGS, *NVCC_FLAGS, "-shared", "-I", INCLUDE, "-I", CSRC, *cu]
        cmd += [x for f in cpp for x in ("-x", "cu", f)]
        cmd += ["-o", tmp]
        _run(cmd, verbose)
        os.replace(tmp, LIB)
    return LIB


def build_ext(force=False, verbose=False) -> str:
    import pybind11

    src = os.path.join(CSRC, "engine", "bindings.cpp")
    if force or _stale(EXT, [src, LIB] + _headers() + [__file__]):
        tmp = EXT + ".tmp"
        cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC",
               "-I", INCLUDE, "-I", pybind11.get_include(), "-I", sysconfig.get_paths()["include"],
               "-I", os.path.join(CUDA_HOME, "include"), src, "-o", tmp,
               "-L", PKG, "-lsubq_b200", "-Wl,-rpath,$ORIGIN",
               # static CUDA runtime: loading a second shared libcudart next to
               # torch's own copy breaks torch's library preloading
               # (its symbols stay private to this module)
               "-L", os.path.join(CUDA_HOME, "lib64"), "-l:libcudart_static.a", "-ldl", "-lrt", "-lpthread",
               "-Wl,--exclude-libs,ALL"]
        _run(cmd, verbose)
        os.replace(tmp, EXT)
    return EXT


def build(force=False, verbose=False) -> None:
    build_lib(force, verbose)
    build_ext(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
