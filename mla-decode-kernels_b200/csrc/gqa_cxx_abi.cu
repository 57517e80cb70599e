// C++-linkage exports of the three reference launchers.
//
// The reference declares gqa_decode_v0/v1/v2_launch in include/gqa_decode.h
// (lines 6-23) without extern "C", so an object compiled against that header
// (for example the reference's python/gqa_decode_ext.cpp) references their
// C++-mangled names.  This translation unit defines exactly those symbols -
// same names, same parameter types (__nv_bfloat16 pointers, int dims, float
// scale, cudaStream_t) - and forwards to the shared launcher bodies, so such
// an object links against this library unchanged.  It deliberately does not
// include this library's gqa_decode.h, whose declarations of the same names
// have C linkage; the C-linkage symbols (gqa_api.cu) stay exported beside
// these for C, cgo, JNI and ctypes callers.
#include <cuda_bf16.h>
#include <cuda_runtime_api.h>

#include "gqa_internal.h"

// The reference's prototypes, C++ linkage.
void gqa_decode_v0_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                          const __nv_bfloat16* v_cache, const int* block_table,
                          const int* seq_lens, __nv_bfloat16* out, int B, int Hq, int Hkv,
                          int block_size, int max_blocks, float scale, cudaStream_t stream);
void gqa_decode_v1_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                          const __nv_bfloat16* v_cache, const int* block_table,
                          const int* seq_lens, __nv_bfloat16* out, int B, int Hq, int Hkv,
                          int block_size, int max_blocks, float scale, cudaStream_t stream);
void gqa_decode_v2_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                          const __nv_bfloat16* v_cache, const int* block_table,
                          const int* seq_lens, __nv_bfloat16* out, int B, int Hq, int Hkv,
                          int block_size, int max_blocks, float scale, int num_splits,
                          float* ws_acc, float* ws_m, float* ws_l, cudaStream_t stream);

__attribute__((visibility("default"))) void gqa_decode_v0_launch(
    const __nv_bfloat16* q, const __nv_bfloat16* k_cache, const __nv_bfloat16* v_cache,
    const int* block_table, const int* seq_lens, __nv_bfloat16* out, int B, int Hq, int Hkv,
    int block_size, int max_blocks, float scale, cudaStream_t stream) {
  gqa::compat_v0_launch(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv, block_size,
                        max_blocks, scale, stream);
}

__attribute__((visibility("default"))) void gqa_decode_v1_launch(
    const __nv_bfloat16* q, const __nv_bfloat16* k_cache, const __nv_bfloat16* v_cache,
    const int* block_table, const int* seq_lens, __nv_bfloat16* out, int B, int Hq, int Hkv,
    int block_size, int max_blocks, float scale, cudaStream_t stream) {
  gqa::compat_v1_launch(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv, block_size,
                        max_blocks, scale, stream);
}

__attribute__((visibility("default"))) void gqa_decode_v2_launch(
    const __nv_bfloat16* q, const __nv_bfloat16* k_cache, const __nv_bfloat16* v_cache,
    const int* block_table, const int* seq_lens, __nv_bfloat16* out, int B, int Hq, int Hkv,
    int block_size, int max_blocks, float scale, int num_splits, float* ws_acc, float* ws_m,
    float* ws_l, cudaStream_t stream) {
  gqa::compat_v2_launch(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv, block_size,
                        max_blocks, scale, num_splits, ws_acc, ws_m, ws_l, stream);
}
