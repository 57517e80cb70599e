// C-linkage forwarders to the reference's own launchers (reference
// include/gqa_decode.h:6-23 declares them with C++ linkage), so the tests can
// run the reference kernels, built from their sources for sm_100a by
// `make ref`, through ctypes as an independent GPU-side checker.
// TEST INFRASTRUCTURE ONLY.
#include "gqa_decode.h"  // the reference's header (-I<reference>/include)

extern "C" {

int ref_gqa_decode_v1(const void* q, const void* k, const void* v, const int* bt, const int* sl,
                      void* out, int B, int Hq, int Hkv, int bs, int max_blocks, float scale,
                      void* stream) {
  gqa_decode_v1_launch(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                       static_cast<const __nv_bfloat16*>(v), bt, sl,
                       static_cast<__nv_bfloat16*>(out), B, Hq, Hkv, bs, max_blocks, scale,
                       static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}

int ref_gqa_decode_v2(const void* q, const void* k, const void* v, const int* bt, const int* sl,
                      void* out, int B, int Hq, int Hkv, int bs, int max_blocks, float scale,
                      int num_splits, float* ws_acc, float* ws_m, float* ws_l, void* stream) {
  gqa_decode_v2_launch(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                       static_cast<const __nv_bfloat16*>(v), bt, sl,
                       static_cast<__nv_bfloat16*>(out), B, Hq, Hkv, bs, max_blocks, scale,
                       num_splits, ws_acc, ws_m, ws_l, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
