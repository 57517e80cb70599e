"""In-tree build of the decode engine.

Produces, next to the sources (so the files travel with the repository):
  lib/libgqa_decode_b200.so   the CUDA kernels + C ABI (nvcc, sm_100a only)
  _build/gqa_decode_ext.so    the PyTorch binding (torch.utils.cpp_extension)

The reference JIT-builds its extension for sm_90a at import
(python/binding.py:11-23); this build targets sm_100a and can be run ahead
of time (``python mla-decode-kernels_b200/python/gqa_build.py``) or on first import.
"""

import ctypes
import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC_DIR = os.path.join(PKG_DIR, "csrc")
PY_DIR = os.path.join(PKG_DIR, "python")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libgqa_decode_b200.so")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
EXT_NAME = "gqa_decode_ext"
EXT_PATH = os.path.join(BUILD_DIR, EXT_NAME + ".so")

CU_SOURCES = ["gqa_scan.cu", "gqa_simt.cu", "gqa_api.cu", "gqa_cxx_abi.cu", "gqa_noalloc.cu",
              "mla_decode.cu", "dsa_decode.cu"]
CU_HEADERS = ["gqa_internal.h", "gqa_ptx.cuh", "gqa_merge.cuh", "umma_ptx.cuh", "device_once.h"]
PUBLIC_HEADERS = ["gqa_decode.h", "mla_decode.h", "dsa_decode.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xlinker", "-soname=libgqa_decode_b200.so",
]


def _nvcc():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_lib(force=False, verbose=False, extra_flags=()):
    """Compile the CUDA sources into lib/libgqa_decode_b200.so."""
    srcs = [os.path.join(CSRC_DIR, s) for s in CU_SOURCES]
    deps = srcs + [os.path.join(CSRC_DIR, h) for h in CU_HEADERS]
    deps += [os.path.join(INCLUDE_DIR, h) for h in PUBLIC_HEADERS]
    if not force and not _newer(LIB_PATH, deps):
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, *extra_flags, "-I" + INCLUDE_DIR, "-I" + CSRC_DIR, *srcs, "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def preload_lib():
    """dlopen the C-ABI library globally so the binding resolves against it."""
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python {os.path.abspath(__file__)}`")
    return ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)


def build_ext(force=False, verbose=False):
    """Compile python/gqa_decode_ext.cpp against the C ABI into _build/."""
    src = os.path.join(PY_DIR, "gqa_decode_ext.cpp")
    deps = [src, LIB_PATH] + [os.path.join(INCLUDE_DIR, h) for h in PUBLIC_HEADERS]
    if not force and not _newer(EXT_PATH, deps):
        return EXT_PATH
    preload_lib()
    from torch.utils.cpp_extension import load

    os.makedirs(BUILD_DIR, exist_ok=True)
    load(
        name=EXT_NAME,
        sources=[src],
        build_directory=BUILD_DIR,
        extra_include_paths=[INCLUDE_DIR],
        extra_cflags=["-O3"],
        extra_ldflags=[f"-L{LIB_DIR}", "-lgqa_decode_b200"],
        with_cuda=True,
        verbose=verbose,
    )
    os.utime(EXT_PATH, None)
    return EXT_PATH


def build_all(force=False, verbose=False):
    build_lib(force=force, verbose=verbose)
    build_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
    print(LIB_PATH)
    print(EXT_PATH)
