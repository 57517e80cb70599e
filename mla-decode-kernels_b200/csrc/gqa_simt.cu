// v0 rung: a plain CUDA-core grouped scan, kept as the ablation baseline for
// the pipelined tensor-core scan and as an independent implementation for
// cross-checks.  One CTA per (request b, kv head hk), 4 warps; warp w walks
// tokens w, w+4, ... (the warp-strided chains of
// kernels/gqa_decode/v1_vectorized.cu:31) but, unlike the reference, one K/V
// row load serves up to 8 q heads of the group at a time.  Lane = 4 dims.
// The 4 per-warp states are merged through shared memory with the
// online-softmax identity (kernels/gqa_decode/v1_vectorized.cu:51-70).
#include <math.h>

#include "gqa_internal.h"

namespace gqa {

namespace {
constexpr unsigned kFull = 0xffffffffu;
constexpr int kWarps = 4;
constexpr int kHeadsPerPass = 8;
}  // namespace

__global__ void __launch_bounds__(128) gqa_decode_simt_kernel(const SimtParams p) {
  const int G = p.Hq / p.Hkv;
  const int b = blockIdx.x / p.Hkv;
  const int hk = blockIdx.x - b * p.Hkv;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long cap = static_cast<long long>(p.max_blocks) * p.bs;
  long long S64 = p.seq_lens[b];
  if (S64 < 0) S64 = 0;
  if (S64 > cap) S64 = cap;
  const int S = static_cast<int>(S64);

  __shared__ float sm_m[kWarps][kHeadsPerPass];
  __shared__ float sm_l[kWarps][kHeadsPerPass];
  __shared__ float4 sm_acc[kWarps][kHeadsPerPass][32];

  const int* bt_row = p.block_table + static_cast<size_t>(b) * p.max_blocks;
  for (int j0 = 0; j0 < G; j0 += kHeadsPerPass) {
    const int cnt = min(kHeadsPerPass, G - j0);
    float qv[kHeadsPerPass][4];
    #pragma unroll
    for (int j = 0; j < kHeadsPerPass; ++j) {
      if (j < cnt) {
        const __nv_bfloat16* qp =
            p.q + (static_cast<size_t>(b) * p.Hq + hk * G + j0 + j) * kHeadDim + 4 * lane;
        const uint2 raw = *reinterpret_cast<const uint2*>(qp);
        const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
        const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
        qv[j][0] = __low2float(lo);
        qv[j][1] = __high2float(lo);
        qv[j][2] = __low2float(hi);
        qv[j][3] = __high2float(hi);
      } else {
        qv[j][0] = qv[j][1] = qv[j][2] = qv[j][3] = 0.f;
      }
    }
    float m[kHeadsPerPass], l[kHeadsPerPass], acc[kHeadsPerPass][4];
    #pragma unroll
    for (int j = 0; j < kHeadsPerPass; ++j) {
      m[j] = -INFINITY;
      l[j] = 0.f;
      acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    }
    for (int t = w; t < S; t += kWarps) {
      const int lb = t / p.bs;
      const int sl = t - lb * p.bs;
      const int page = __ldg(bt_row + lb);
      const size_t off =
          ((static_cast<size_t>(page) * p.bs + sl) * p.Hkv + hk) * kHeadDim + 4 * lane;
      const uint2 kraw = __ldg(reinterpret_cast<const uint2*>(p.k + off));
      const uint2 vraw = __ldg(reinterpret_cast<const uint2*>(p.v + off));
      float kf[4], vf[4];
      {
        const __nv_bfloat162 k0 = *reinterpret_cast<const __nv_bfloat162*>(&kraw.x);
        const __nv_bfloat162 k1 = *reinterpret_cast<const __nv_bfloat162*>(&kraw.y);
        const __nv_bfloat162 v0 = *reinterpret_cast<const __nv_bfloat162*>(&vraw.x);
        const __nv_bfloat162 v1 = *reinterpret_cast<const __nv_bfloat162*>(&vraw.y);
        kf[0] = __low2float(k0);
        kf[1] = __high2float(k0);
        kf[2] = __low2float(k1);
        kf[3] = __high2float(k1);
        vf[0] = __low2float(v0);
        vf[1] = __high2float(v0);
        vf[2] = __low2float(v1);
        vf[3] = __high2float(v1);
      }
      #pragma unroll
      for (int j = 0; j < kHeadsPerPass; ++j) {
        float d = qv[j][0] * kf[0] + qv[j][1] * kf[1] + qv[j][2] * kf[2] + qv[j][3] * kf[3];
        #pragma unroll
        for (int off2 = 16; off2 > 0; off2 >>= 1) d += __shfl_xor_sync(kFull, d, off2);
        const float sc = d * p.scale_log2;
        const float mn = fmaxf(m[j], sc);
        const float al = exp2f(m[j] - mn);
        const float pw = exp2f(sc - mn);
        l[j] = l[j] * al + pw;
        #pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = acc[j][i] * al + pw * vf[i];
        m[j] = mn;
      }
    }
    #pragma unroll
    for (int j = 0; j < kHeadsPerPass; ++j) {
      if (lane == 0) {
        sm_m[w][j] = m[j];
        sm_l[w][j] = l[j];
      }
      sm_acc[w][j][lane] = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
    }
    __syncthreads();
    for (int j = w; j < cnt; j += kWarps) {
      float M = -INFINITY;
      #pragma unroll
      for (int i = 0; i < kWarps; ++i) M = fmaxf(M, sm_m[i][j]);
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      if (M != -INFINITY) {
        float L = 0.f;
        #pragma unroll
        for (int i = 0; i < kWarps; ++i) {
          const float f = exp2f(sm_m[i][j] - M);  // an idle warp has m = -inf -> 0
          L += sm_l[i][j] * f;
          const float4 x = sm_acc[i][j][lane];
          o[0] += x.x * f;
          o[1] += x.y * f;
          o[2] += x.z * f;
          o[3] += x.w * f;
        }
        #pragma unroll
        for (int i = 0; i < 4; ++i) o[i] /= L;
      }
      __nv_bfloat16* op =
          p.out + (static_cast<size_t>(b) * p.Hq + hk * G + j0 + j) * kHeadDim + 4 * lane;
      uint2 st;
      __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]);
      __nv_bfloat162 hi = __floats2bfloat162_rn(o[2], o[3]);
      st.x = *reinterpret_cast<unsigned*>(&lo);
      st.y = *reinterpret_cast<unsigned*>(&hi);
      *reinterpret_cast<uint2*>(op) = st;
    }
    __syncthreads();
  }
}

cudaError_t launch_simt(const SimtParams& p, cudaStream_t s) {
  const long long grid = static_cast<long long>(p.B) * p.Hkv;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  gqa_decode_simt_kernel<<<static_cast<unsigned>(grid), kWarps * 32, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace gqa
