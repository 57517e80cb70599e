"""CPU: a C++ caller written against the reference's header links unchanged.

The reference declares gqa_decode_v0/v1/v2_launch with C++ linkage
(include/gqa_decode.h:6-23 of the reference), so an object compiled against
that header references the C++-mangled names.  These tests build such
callers and link them against lib/libgqa_decode_b200.so:

* a small C++ program carrying the reference's three prototypes, linked with
  --no-undefined and run: every call is made with an invalid batch size, so
  nothing touches a GPU, and the error each one records is read back
  through gqa_decode_last_error();
* when a reference checkout is available (GQA_REFERENCE_DIR, else the
  reference_path in BASELINE.json), the reference's own, unmodified
  python/gqa_decode_ext.cpp compiled against its own header into a PyTorch
  extension linked to this library, and imported (the loader resolves every
  symbol at import).
"""

import os
import subprocess
import textwrap

import pytest

import gqa_build as pkg_build
import oracle

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

CALLER = textwrap.dedent(r"""
    #include <cstdio>
    #include <cuda_bf16.h>
    #include <cuda_runtime_api.h>

    // The reference's prototypes (C++ linkage), as its header declares them.
    void gqa_decode_v0_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                              const __nv_bfloat16* v_cache, const int* block_table,
                              const int* seq_lens, __nv_bfloat16* out, int B, int Hq,
                              int Hkv, int block_size, int max_blocks, float scale,
                              cudaStream_t stream);
    void gqa_decode_v1_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                              const __nv_bfloat16* v_cache, const int* block_table,
                              const int* seq_lens, __nv_bfloat16* out, int B, int Hq,
                              int Hkv, int block_size, int max_blocks, float scale,
                              cudaStream_t stream);
    void gqa_decode_v2_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                              const __nv_bfloat16* v_cache, const int* block_table,
                              const int* seq_lens, __nv_bfloat16* out, int B, int Hq,
                              int Hkv, int block_size, int max_blocks, float scale,
                              int num_splits, float* ws_acc, float* ws_m, float* ws_l,
                              cudaStream_t stream);
    // This library's error channel for the void launchers (C linkage).
    extern "C" cudaError_t gqa_decode_last_error(void);

    int main() {
      // B = -1 is rejected before any device access.
      gqa_decode_v0_launch(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, -1, 32, 8, 16,
                           1, 0.1f, nullptr);
      const int e0 = gqa_decode_last_error();
      gqa_decode_v1_launch(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, -1, 32, 8, 16,
                           1, 0.1f, nullptr);
      const int e1 = gqa_decode_last_error();
      gqa_decode_v2_launch(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, -1, 32, 8, 16,
                           1, 0.1f, 8, nullptr, nullptr, nullptr, nullptr);
      const int e2 = gqa_decode_last_error();
      const int after = gqa_decode_last_error();  // reading resets it
      std::printf("%d %d %d %d\n", e0, e1, e2, after);
      return 0;
    }
""")


@pytest.fixture(scope="module")
def libpath():
    if not os.path.exists(pkg_build.LIB_PATH):
        pkg_build.build_lib()
    return pkg_build.LIB_PATH


def test_cxx_caller_of_reference_prototypes_links_and_runs(tmp_path, libpath):
    src = tmp_path / "caller.cpp"
    src.write_text(CALLER)
    exe = tmp_path / "caller"
    libdir = os.path.dirname(libpath)
    subprocess.run(["g++", "-std=c++17", str(src), "-I" + os.path.join(CUDA_HOME, "include"),
                    "-L" + libdir, "-lgqa_decode_b200", "-Wl,-rpath," + libdir,
                    "-Wl,--no-undefined", "-o", str(exe)], check=True)
    # the executable's undefined launcher references are the mangled names
    undef = subprocess.run(["nm", "-u", str(exe)], capture_output=True, text=True,
                           check=True).stdout
    assert "_Z20gqa_decode_v2_launch" in undef
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    # cudaErrorInvalidValue (1) from each launcher, then cudaSuccess after the reset
    assert out == ["1", "1", "1", "0"]


REF = oracle.reference_checkout()


@pytest.mark.skipif(REF is None, reason="no reference checkout (GQA_REFERENCE_DIR)")
def test_reference_extension_source_links_unchanged(tmp_path, libpath):
    import torch.utils.cpp_extension as ext

    src = os.path.join(REF, "python", "gqa_decode_ext.cpp")
    libdir = os.path.dirname(libpath)
    pkg_build.preload_lib()
    mod = ext.load(name="ref_gqa_decode_ext", sources=[src], build_directory=str(tmp_path),
                   extra_include_paths=[os.path.join(REF, "include")], extra_cflags=["-O0"],
                   extra_ldflags=[f"-L{libdir}", "-lgqa_decode_b200", f"-Wl,-rpath,{libdir}"],
                   with_cuda=True, verbose=False)
    for name in ("gqa_decode_v0", "gqa_decode_v1", "gqa_decode_v2"):
        assert hasattr(mod, name)
    so = [f for f in os.listdir(tmp_path) if f.endswith(".so")][0]
    undef = subprocess.run(["nm", "-u", os.path.join(tmp_path, so)], capture_output=True,
                           text=True, check=True).stdout
    assert "_Z20gqa_decode_v0_launch" in undef  # resolved against this library at import
