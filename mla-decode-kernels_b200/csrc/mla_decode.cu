// MLA absorbed-path paged decode on sm_100a (the reference's roadmap kernel
// K2: latent cache [num_blocks, 64, 576], README.md "Roadmap"; no reference
// code exists, kernels/mla_decode/ is empty).  Operator, as FlashMLA's
// flash_mla_with_kvcache computes it: for request b, query position i, head h,
//   out[b, i, h, :] = softmax_t(scale * q[b, i, h, :] . C_t) @ C_t[0:512]
// over the request's cached latent rows C_t (576 = 512 latent + 64 rope
// dims; one latent "kv head"), t < S_b, or t < S_b - s_q + 1 + i when causal;
// lse[b, h, i] = ln sum_t exp(score_t).
//
// One CTA = (request, group of NH <= 64 query rows, page range).  Tokens are
// the MMA M dimension and query rows the N dimension, so small head counts
// waste no tensor-core work and one page read serves all NH rows:
//   S^T[64 tok, NH]  = C[64 tok, 576] . Q[NH, 576]^T     (M = 64, 36 MMAs)
//   O^T[512, NH]    += C[64 tok, 0:512]^T . P^T[64, NH]  (M = 128, 4 x 4 MMAs)
// with S^T and O^T in tensor memory.
//
// Warps: 0 = TMA producer (one 64-token page per stage: nine 64-column boxes
// of a 128-byte-swizzled tensor map), 1 = MMA issuer + TMEM owner, 2-5 =
// softmax / correction / epilogue (warp w reads TMEM lanes 32 (w % 4) ..).
// Online softmax in the log2 domain with a lazily raised reference max: P is
// computed against the current reference m_ref[h] and O^T / l are only
// rescaled when a tile's score exceeds m_ref by more than 2^8 (the bound on
// exp2 growth kept in fp32 / bf16 range), which after the first tiles is rare.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "gqa_decode.h"
#include "gqa_ptx.cuh"
#include "mla_decode.h"
#include "umma_ptx.cuh"

namespace gqa {
namespace mla {

constexpr int kD = 576;             // latent + rope dims per cached token
constexpr int kDV = 512;            // value dims (the latent part)
constexpr int kPage = 64;           // tokens per cache page (FlashMLA's block size)
constexpr int kCols = kD / 64;      // 64-element (128-byte) column boxes per row: 9
constexpr int kColBytes = kPage * 128;            // one box of a page: 8 KB
constexpr int kStageBytes = kCols * kColBytes;    // one page: 72 KB
constexpr int kStages = 2;
constexpr int kThreads = 192;       // producer, MMA, 4 softmax warps
constexpr float kRescaleLog2 = 8.f; // lazy rescale threshold (log2 units)

__device__ int g_mla_status;

struct Params {
  CUtensorMap tm_q;   // [rows_total, 576] bf16, box {64, NH}, 128B swizzle
  CUtensorMap tm_kv;  // [num_blocks * 64, 576] bf16, box {64, 64}, 128B swizzle
  const int* block_table;
  const int* seq_lens;
  __nv_bfloat16* out;  // [B, s_q, h_q, 512] (num_splits == 1)
  float* lse;          // [B, h_q, s_q]      (num_splits == 1)
  float* part_acc;     // [B * rows, ns, 512] unnormalised (num_splits > 1)
  float* part_m;       // [B * rows, ns] log2-domain reference max
  float* part_l;       // [B * rows, ns]
  int B, s_q, h_q, rows, n_hg, max_blocks, num_blocks, num_splits, causal;
  float scale_log2;    // softmax_scale * log2(e)
  int smem_q, smem_ring, smem_p, smem_small;  // byte offsets in dynamic smem
  uint32_t tmem_cols;
};

__device__ __forceinline__ void raise(int bit) { atomicOr(&g_mla_status, bit); }

// Bounded mbarrier wait with one outcome for the whole warp.
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// P^T buffer: [64 tokens x NH] bf16 rows of R = 2 NH bytes with the matching
// swizzle (SW32 / SW64 / SW128 for NH = 16 / 32 / 64): the 16-byte chunk
// index (address bits 4..) is XOR-ed with the bits above bit 7.
__device__ __forceinline__ uint32_t p_swz(uint32_t off, int NH) {
  const uint32_t mask = NH == 64 ? 7u : (NH == 32 ? 3u : 1u);
  return off ^ (((off >> 7) & mask) << 4);
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Visible tokens of query row `row` (0 .. s_q*h_q-1) of a request with S
// cached tokens.
__device__ __forceinline__ int visible(const Params& p, int S, int row) {
  if (!p.causal) return S;
  const int i = row / p.h_q;
  return max(0, min(S, S - p.s_q + 1 + i));
}

template <int NH>
__global__ void __launch_bounds__(kThreads, 1) mla_decode_kernel(const __grid_constant__ Params p) {
  static_assert(NH == 16 || NH == 32 || NH == 64, "query rows per CTA");
  // P^T buffers: two (softmax of tile t+1 overlaps PV of tile t) where shared
  // memory allows, one at NH = 64
  constexpr int NP = NH == 64 ? 1 : 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment of every swizzle atom
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sQ = s_base + p.smem_q;
  const uint32_t sRing = s_base + p.smem_ring;
  const uint32_t sP = s_base + p.smem_p;
  unsigned char* small = smem + p.smem_small;
  // small region: 14 mbarriers, TMEM base, votes [2][4], red [4][64],
  // m_ref [64], alpha [64], visible tokens per query row [64]
  const uint32_t bars = s_base + p.smem_small;
  const uint32_t bar_q = bars + 0, bar_full = bars + 8, bar_empty = bars + 24,
                 bar_sfull = bars + 40, bar_sfree = bars + 56, bar_pfull = bars + 72,
                 bar_pv = bars + 88, bar_fin = bars + 104;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(small + 112);
  int* vote = reinterpret_cast<int*>(small + 128);                // [2][4]
  float* red = reinterpret_cast<float*>(small + 160);             // [4][64]
  float* mref = reinterpret_cast<float*>(small + 160 + 1024);     // [64]
  float* alpha_s = reinterpret_cast<float*>(small + 160 + 1280);  // [64]
  int* vis_s = reinterpret_cast<int*>(small + 160 + 1536);        // [64]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x;
  const int hg = unit % p.n_hg;
  const int sp = (unit / p.n_hg) % p.num_splits;
  const int b = unit / (p.n_hg * p.num_splits);
  const int row0 = hg * NH;
  // lengths beyond the page table's capacity are cut to it (no read past a row)
  const int S = max(0, min(p.seq_lens[b], p.max_blocks * kPage));
  const int pages = (S + kPage - 1) / kPage;
  const int chunk = (pages + p.num_splits - 1) / p.num_splits;
  const int pg0 = min(pages, sp * chunk), pg1 = min(pages, pg0 + chunk);
  const int ntiles = pg1 - pg0;
  constexpr uint32_t o_col = 0, s_col0 = 4 * NH;  // TMEM columns: O^T blocks, S^T buffers
  constexpr uint32_t R = 2 * NH;                 // P^T row bytes
  constexpr uint32_t kPBytes = kPage * R;        // one P^T buffer

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
      mbar_init(bar_sfull + 8 * s, 1);
      mbar_init(bar_sfree + 8 * s, 4);
      mbar_init(bar_pfull + 8 * s, 4);
      mbar_init(bar_pv + 8 * s, 1);
    }
    mbar_init(bar_fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), p.tmem_cols);
    tmem_relinquish();
  }
  if (threadIdx.x < 64) {
    mref[threadIdx.x] = -INFINITY;
    // rows past the last query row (padding of the final group) see nothing
    const int row = row0 + threadIdx.x;
    vis_s[threadIdx.x] = row < p.rows ? visible(p, S, row) : 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0 && ntiles > 0) {
      tma_prefetch_desc(&p.tm_kv);
      mbar_arrive_expect_tx(bar_q, static_cast<uint32_t>(NH * kD * 2));
      for (int c = 0; c < kCols; ++c)
        tma_load_2d(sQ + c * NH * 128, &p.tm_q, 64 * c, b * p.rows + row0, bar_q);
      const int* bt = p.block_table + static_cast<size_t>(b) * p.max_blocks;
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t & 1;
        if (t >= kStages && !mbar_wait(bar_empty + 8 * s, ((t - kStages) >> 1) & 1)) {
          raise(kStatusWaitTimeout);
          break;
        }
        int page = __ldg(bt + pg0 + t);
        if (page < 0 || page >= p.num_blocks) {
          raise(kStatusBadPage);
          page = 0;
        }
        mbar_arrive_expect_tx(bar_full + 8 * s, kStageBytes);
        for (int c = 0; c < kCols; ++c)
          tma_load_2d(sRing + s * kStageBytes + c * kColBytes, &p.tm_kv, 64 * c, page * kPage,
                      bar_full + 8 * s);
        issued = t + 1;
      }
      // every issued copy has landed before the CTA may exit
      if (!mbar_wait(bar_q, 0)) raise(kStatusWaitTimeout);
      for (int t = max(0, issued - kStages); t < issued; ++t)
        if (!mbar_wait(bar_full + 8 * (t & 1), (t >> 1) & 1)) raise(kStatusWaitTimeout);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    // Polls for the next ready step instead of blocking in a fixed order, so
    // PV of tile t (which frees t's stage for the next load) never waits
    // behind the arrival of page t+1.  Lane 0 decides and issues; the whole
    // warp zeroes the tail rows of a request's last page.
    constexpr uint32_t idesc_qk = umma_idesc_bf16(64, NH, false, false);
    constexpr uint32_t idesc_pv = umma_idesc_bf16(128, NH, true, true);
    constexpr uint32_t p_layout = NH == 64 ? kSwizzle128 : (NH == 32 ? kSwizzle64 : kSwizzle32);
    bool ok = true;
    if (ntiles > 0) ok = wait_warp(bar_q, 0);
    int qk = 0, pv = 0;  // next tile whose S = Q K^T / O^T += V^T P^T is issued
    unsigned long long idle_since = global_timer_ns();
    while (ok && pv < ntiles) {
      int action = 0;  // 1 = PV(pv), 2 = QK(qk)
      if (lane == 0) {
        if (pv < qk && mbar_test_wait(bar_pfull + 8 * (pv & 1), (pv >> 1) & 1)) {
          action = 1;
        } else if (qk < ntiles && qk <= pv + 1 &&
                   mbar_test_wait(bar_full + 8 * (qk & 1), (qk >> 1) & 1) &&
                   (qk < 2 || mbar_test_wait(bar_sfree + 8 * (qk & 1), ((qk - 2) >> 1) & 1))) {
          action = 2;
        }
      }
      action = __shfl_sync(0xffffffffu, action, 0);
      if (action == 0) {
        if (global_timer_ns() - idle_since > kWaitLimitNs) ok = false;
        continue;
      }
      idle_since = global_timer_ns();
      tc_fence_after();
      if (action == 2) {
        const int s = qk & 1, buf = qk & 1;
        // Zero the cache rows past the request's end in its last page (they
        // may hold anything, NaN included): 0 * NaN would poison O^T.
        const int nv = min(kPage, S - (pg0 + qk) * kPage);
        if (nv < kPage) {
          const int zrows = kPage - nv;
          for (int i = lane; i < kCols * zrows * 8; i += 32) {
            const int c = i / (zrows * 8), r = nv + (i / 8) % zrows, k = i % 8;
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(
                             sRing + s * kStageBytes + c * kColBytes + r * 128 + k * 16),
                         "r"(0u)
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        if (lane == 0) {
          const uint32_t kv = sRing + s * kStageBytes;
          #pragma unroll 1
          for (int c = 0; c < kCols; ++c) {
            #pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t a =
                  umma_smem_desc(kv + c * kColBytes + kk * 32, 16, 1024, kSwizzle128);
              const uint64_t bq =
                  umma_smem_desc(sQ + c * NH * 128 + kk * 32, 16, 1024, kSwizzle128);
              umma_bf16_ss(tmem + s_col0 + buf * NH, a, bq, idesc_qk, (c | kk) != 0);
            }
          }
          umma_commit(bar_sfull + 8 * buf);
        }
        __syncwarp();
        ++qk;
      } else {
        if (lane == 0) {
          const uint32_t kv = sRing + (pv & 1) * kStageBytes;
          const uint32_t pb = sP + (pv % NP) * kPBytes;
          #pragma unroll 1
          for (int j = 0; j < 4; ++j) {
            #pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t a = umma_smem_desc(kv + 2 * j * kColBytes + kk * 16 * 128,
                                                kColBytes, 1024, kSwizzle128);
              const uint64_t bp = umma_smem_desc(pb + kk * 16 * R, kPBytes, 8 * R, p_layout);
              umma_bf16_ss(tmem + o_col + j * NH, a, bp, idesc_pv, (pv | kk) != 0);
            }
          }
          umma_commit(bar_pv + 8 * (pv & 1));
          umma_commit(bar_empty + 8 * (pv & 1));
        }
        __syncwarp();
        ++pv;
      }
    }
    if (!ok) raise(kStatusWaitTimeout);
    // every MMA this thread issued has completed before TMEM is released
    if (lane == 0) umma_commit(bar_fin);
    __syncwarp();
    if (!wait_warp(bar_fin, 0)) raise(kStatusWaitTimeout);
  } else {
    // --------------------------- softmax warps 2..5 ----------------------------
    // Every softmax warp runs the same sequence of named barriers whatever
    // happens (a failed wait only clears `ok`), so they can never deadlock.
    const int tq = warp & 3;        // TMEM lane quadrant
    const bool active = lane < 16;  // S^T rows (M = 64 layout): lanes 0-15 of a quadrant
    const int tok_in_tile = 16 * tq + lane;
    const uint32_t lane_base = static_cast<uint32_t>(32 * tq) << 16;
    const int sidx = threadIdx.x - 64;  // 0..127
    float lpart[NH];
    #pragma unroll
    for (int h = 0; h < NH; ++h) lpart[h] = 0.f;
    bool ok = true;
    // Completion of PV(k) is phase k >> 1 of bar_pv[k & 1].
    auto wait_pv = [&](int k) {
      if (k >= 0 && ok && !wait_warp(bar_pv + 8 * (k & 1), (k >> 1) & 1)) ok = false;
    };
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t & 1;
      if (ok && !wait_warp(bar_sfull + 8 * buf, (t >> 1) & 1)) ok = false;
      tc_fence_after();
      float x[NH];
      #pragma unroll
      for (int c16 = 0; c16 < NH / 16; ++c16) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + s_col0 + buf * NH + 16 * c16, r);
        tmem_wait_ld();
        #pragma unroll
        for (int k = 0; k < 16; ++k) x[16 * c16 + k] = __uint_as_float(r[k]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree + 8 * buf);
      const int tok = (pg0 + t) * kPage + tok_in_tile;
      bool need = false;
      #pragma unroll
      for (int h = 0; h < NH; ++h) {
        const bool valid = active && tok < vis_s[h];
        x[h] = valid ? x[h] * p.scale_log2 : -INFINITY;
        need |= x[h] > mref[h] + kRescaleLog2;
      }
      need = __any_sync(0xffffffffu, need);
      if (lane == 0) vote[(t & 1) * 4 + tq] = need ? 1 : 0;
      named_bar_sync(1, 128);
      const int* v = vote + (t & 1) * 4;
      const bool rescale = (v[0] | v[1] | v[2] | v[3]) != 0;
      if (rescale) {
        // tile max per head over the 64 token rows (16 lanes x 4 warps)
        #pragma unroll
        for (int h = 0; h < NH; ++h) {
          float m = x[h];
          #pragma unroll
          for (int off = 8; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
          if (lane == 0) red[tq * 64 + h] = m;
        }
        named_bar_sync(1, 128);
        if (sidx < NH) {
          const int h = sidx;
          const float tmax = fmaxf(fmaxf(red[h], red[64 + h]), fmaxf(red[128 + h], red[192 + h]));
          const float mo = mref[h];
          const float mn = fmaxf(mo, tmax);
          alpha_s[h] = mo == -INFINITY ? 0.f : exp2f(mo - mn);
          mref[h] = mn;
        }
        named_bar_sync(1, 128);
        #pragma unroll
        for (int h = 0; h < NH; ++h) lpart[h] *= alpha_s[h];
        if (t >= 1) {
          // O^T[dv, h] *= alpha[h] on this warp's quadrant (dv rows 32 tq..),
          // once every earlier PV has accumulated into it
          wait_pv(t - 1);
          tc_fence_after();
          #pragma unroll 1
          for (int j = 0; j < 4; ++j) {
            #pragma unroll
            for (int c16 = 0; c16 < NH / 16; ++c16) {
              uint32_t r[16];
              const uint32_t a = tmem + lane_base + o_col + j * NH + 16 * c16;
              tmem_ld16(a, r);
              tmem_wait_ld();
              #pragma unroll
              for (int k = 0; k < 16; ++k)
                r[k] = __float_as_uint(__uint_as_float(r[k]) * alpha_s[16 * c16 + k]);
              tmem_st16(a, r);
            }
          }
          tmem_wait_st();
        }
      }
      // P^T row of this token: p_h = 2^(x_h - m_ref_h), masked rows 0; the
      // buffer is free once the PV that last read it has completed
      wait_pv(t - NP);
      const uint32_t pb = sP + (t % NP) * kPBytes;
      if (active) {
        #pragma unroll
        for (int c8 = 0; c8 < NH / 8; ++c8) {
          float pv[8];
          #pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int h = 8 * c8 + k;
            pv[k] = x[h] == -INFINITY ? 0.f : exp2f(x[h] - mref[h]);
            lpart[h] += pv[k];
          }
          const uint32_t off = p_swz(tok_in_tile * R + 16 * c8, NH);
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(pb + off),
                       "r"(pack2(pv[0], pv[1])), "r"(pack2(pv[2], pv[3])),
                       "r"(pack2(pv[4], pv[5])), "r"(pack2(pv[6], pv[7]))
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_pfull + 8 * (t & 1));
    }
    // ------------------------------ epilogue ---------------------------------
    wait_pv(ntiles - 1);
    tc_fence_after();
    if (!ok) raise(kStatusWaitTimeout);
    // l[h] = sum over the 64 token rows of the per-thread partial sums
    named_bar_sync(1, 128);
    #pragma unroll
    for (int h = 0; h < NH; ++h) {
      float l = active ? lpart[h] : 0.f;
      #pragma unroll
      for (int off = 8; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) red[tq * 64 + h] = l;
    }
    named_bar_sync(1, 128);
    const int L = 32 * tq + lane;  // dv row within each 128-row block of O^T
    const bool final_out = p.num_splits == 1;
    #pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      #pragma unroll
      for (int c16 = 0; c16 < NH / 16; ++c16) {
        uint32_t r[16];
        if (ntiles > 0) {
          tmem_ld16(tmem + lane_base + o_col + j * NH + 16 * c16, r);
          tmem_wait_ld();
        } else {
          #pragma unroll
          for (int k = 0; k < 16; ++k) r[k] = 0u;
        }
        #pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int h = 16 * c16 + k;
          if (row0 + h >= p.rows) continue;  // padding rows of the last group
          const float l = red[h] + red[64 + h] + red[128 + h] + red[192 + h];
          const float o = __uint_as_float(r[k]);
          const size_t grow = static_cast<size_t>(b) * p.rows + row0 + h;
          if (final_out)
            p.out[grow * kDV + 128 * j + L] = __float2bfloat16(l > 0.f ? o / l : 0.f);
          else
            p.part_acc[(grow * p.num_splits + sp) * kDV + 128 * j + L] = l > 0.f ? o : 0.f;
        }
      }
    }
    if (sidx < NH && row0 + sidx < p.rows) {
      const int h = sidx;
      const int row = row0 + h;
      const float l = red[h] + red[64 + h] + red[128 + h] + red[192 + h];
      const float m = l > 0.f ? mref[h] : -INFINITY;
      const size_t grow = static_cast<size_t>(b) * p.rows + row;
      if (final_out) {
        const int i = row / p.h_q, hq = row % p.h_q;
        p.lse[(static_cast<size_t>(b) * p.h_q + hq) * p.s_q + i] =
            l > 0.f ? (m + log2f(l)) * 0.69314718056f : -INFINITY;
      } else {
        p.part_m[grow * p.num_splits + sp] = m;
        p.part_l[grow * p.num_splits + sp] = l;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

// Merge of the num_splits partial states of every (request, query row):
// one warp per row, lane = 16 of the 512 value dims; writes out and lse.
struct CombineParams {
  const float* part_acc;
  const float* part_m;
  const float* part_l;
  __nv_bfloat16* out;
  float* lse;
  int B, s_q, h_q, rows, num_splits;
};

__global__ void __launch_bounds__(128) mla_combine_kernel(const __grid_constant__ CombineParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long grow = static_cast<long long>(blockIdx.x) * 4 + warp;
  if (grow >= static_cast<long long>(p.B) * p.rows) return;
  const int ns = p.num_splits;
  const float* m = p.part_m + grow * ns;
  const float* l = p.part_l + grow * ns;
  float M = -INFINITY;
  for (int s = lane; s < ns; s += 32) M = fmaxf(M, __ldg(m + s));
  #pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float Ls = 0.f;
  float4 a[4];
  #pragma unroll
  for (int k = 0; k < 4; ++k) a[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < ns; ++s) {
    const float ms = __ldg(m + s);
    const float w = ms == -INFINITY ? 0.f : exp2f(ms - M);
    Ls += w * __ldg(l + s);
    const float4* src = reinterpret_cast<const float4*>(p.part_acc + (grow * ns + s) * kDV);
    #pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 v = __ldg(src + lane + 32 * k);
      a[k].x += w * v.x;
      a[k].y += w * v.y;
      a[k].z += w * v.z;
      a[k].w += w * v.w;
    }
  }
  const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
  #pragma unroll
  for (int k = 0; k < 4; ++k) {
    __nv_bfloat16* dst = p.out + grow * kDV + 4 * (lane + 32 * k);
    dst[0] = __float2bfloat16(a[k].x * inv);
    dst[1] = __float2bfloat16(a[k].y * inv);
    dst[2] = __float2bfloat16(a[k].z * inv);
    dst[3] = __float2bfloat16(a[k].w * inv);
  }
  if (lane == 0) {
    const int b = static_cast<int>(grow / p.rows), row = static_cast<int>(grow % p.rows);
    const int i = row / p.h_q, hq = row % p.h_q;
    p.lse[(static_cast<size_t>(b) * p.h_q + hq) * p.s_q + i] =
        Ls > 0.f ? (M + log2f(Ls)) * 0.69314718056f : -INFINITY;
  }
}

}  // namespace mla
}  // namespace gqa

// ================================ host side =================================

namespace {

using gqa::mla::kD;
using gqa::mla::kDV;
using gqa::mla::kPage;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor map over rows of 576 elements (1152 bytes), box 64 x box_rows,
// 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD) * 2};
  cuuint32_t box[2] = {64u, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Query rows per CTA: the smallest of 16 / 32 / 64 holding all rows of a
// request, else 64 (the last group of a request is padded; padded rows are
// computed on whatever the q tile holds there and never stored).
int rows_per_cta(int rows) {
  if (rows <= 0) return 0;
  return rows <= 16 ? 16 : (rows <= 32 ? 32 : 64);
}

struct Layout {
  int NH, n_hg, q, ring, pbuf, small, total;
  uint32_t tmem_cols;
};

Layout layout_for(int rows) {
  Layout L{};
  L.NH = rows_per_cta(rows);
  if (L.NH == 0) return L;
  L.n_hg = (rows + L.NH - 1) / L.NH;
  L.q = 0;
  L.ring = L.q + gqa::mla::kCols * L.NH * 128;
  L.pbuf = L.ring + gqa::mla::kStages * gqa::mla::kStageBytes;
  L.small = L.pbuf + (L.NH == 64 ? 1 : 2) * kPage * 2 * L.NH;  // one / two P^T buffers
  L.total = L.small + 2048 + 1024;  // small region (1952 B used) + alignment slack
  const int cols = 6 * L.NH;
  L.tmem_cols = cols <= 128 ? 128u : (cols <= 256 ? 256u : 512u);
  return L;
}

size_t part_bytes(int B, int rows, int ns) {
  const size_t states = static_cast<size_t>(B) * rows * ns;
  const size_t acc = states * kDV * sizeof(float);
  return ((acc + 255) & ~size_t(255)) + 2 * (((states * sizeof(float)) + 255) & ~size_t(255));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int mla_decode_pick_splits(int B, int s_q, int h_q, int max_pages, int num_sms) {
  const int rows = s_q * h_q;
  const Layout L = layout_for(rows);
  if (L.NH == 0 || B <= 0 || num_sms <= 0) return 1;
  const long long units = static_cast<long long>(B) * L.n_hg;
  // One CTA per SM at a time: the smallest split count whose CTAs fill their
  // last wave to >= 90 % (at least one full wave), keeping >= 4 pages per
  // split; else the best fill among those.
  const long long cap = std::max(1, std::min(64, max_pages / 4));
  long long best = 1;
  double best_fill = 0.0;
  for (long long ns = 1; ns <= cap; ++ns) {
    const long long ctas = units * ns;
    const long long waves = (ctas + num_sms - 1) / num_sms;
    const double fill = static_cast<double>(ctas) / (static_cast<double>(waves) * num_sms);
    if (ctas >= num_sms && fill >= 0.9) return static_cast<int>(ns);
    if (fill > best_fill + 1e-9) {
      best_fill = fill;
      best = ns;
    }
  }
  return static_cast<int>(best);
}

size_t mla_decode_workspace_bytes(int B, int s_q, int h_q, int num_splits) {
  if (B <= 0 || s_q <= 0 || h_q <= 0 || num_splits <= 1) return 0;
  return part_bytes(B, s_q * h_q, num_splits);
}

cudaError_t mla_decode_launch(const gqa_bf16* q, const gqa_bf16* kv_cache, const int* block_table,
                              const int* seq_lens, gqa_bf16* out, float* lse, int B, int s_q,
                              int h_q, int page_size, int max_blocks, int num_blocks,
                              float softmax_scale, int causal, int num_splits, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream) {
  using namespace gqa::mla;
  if (B < 0 || s_q <= 0 || h_q <= 0 || page_size != kPage || max_blocks <= 0 || num_blocks <= 0 ||
      num_splits < 1 || num_splits > 64)
    return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  const int rows = s_q * h_q;
  const Layout L = layout_for(rows);
  if (L.NH == 0) return cudaErrorInvalidValue;
  if (!q || !kv_cache || !block_table || !seq_lens || !out || !lse) return cudaErrorInvalidValue;
  if (!aligned16(q) || !aligned16(kv_cache)) return cudaErrorMisalignedAddress;
  Params p{};
  if (!make_map(&p.tm_q, q, static_cast<uint64_t>(B) * rows, static_cast<uint32_t>(L.NH)) ||
      !make_map(&p.tm_kv, kv_cache, static_cast<uint64_t>(num_blocks) * kPage, kPage))
    return cudaErrorInvalidValue;
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.out = out;
  p.lse = lse;
  p.B = B;
  p.s_q = s_q;
  p.h_q = h_q;
  p.rows = rows;
  p.n_hg = L.n_hg;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.num_splits = num_splits;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.smem_q = L.q;
  p.smem_ring = L.ring;
  p.smem_p = L.pbuf;
  p.smem_small = L.small;
  p.tmem_cols = L.tmem_cols;
  if (num_splits > 1) {
    const size_t need = part_bytes(B, rows, num_splits);
    if (!workspace || workspace_bytes < need || !aligned16(workspace)) return cudaErrorInvalidValue;
    const size_t states = static_cast<size_t>(B) * rows * num_splits;
    unsigned char* w = static_cast<unsigned char*>(workspace);
    const size_t acc = ((states * kDV * sizeof(float)) + 255) & ~size_t(255);
    const size_t ml = ((states * sizeof(float)) + 255) & ~size_t(255);
    p.part_acc = reinterpret_cast<float*>(w);
    p.part_m = reinterpret_cast<float*>(w + acc);
    p.part_l = reinterpret_cast<float*>(w + acc + ml);
  }
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    for (auto fn : {mla_decode_kernel<16>, mla_decode_kernel<32>, mla_decode_kernel<64>}) {
      const cudaError_t e =
          cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
      if (e != cudaSuccess) attr_err = e;
    }
  });
  if (attr_err != cudaSuccess) return attr_err;
  if (L.total > 232448) return cudaErrorInvalidValue;
  const long long grid = static_cast<long long>(B) * L.n_hg * num_splits;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  const unsigned g = static_cast<unsigned>(grid);
  if (L.NH == 64)
    mla_decode_kernel<64><<<g, kThreads, L.total, stream>>>(p);
  else if (L.NH == 32)
    mla_decode_kernel<32><<<g, kThreads, L.total, stream>>>(p);
  else
    mla_decode_kernel<16><<<g, kThreads, L.total, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || num_splits == 1) return e;
  CombineParams c{p.part_acc, p.part_m, p.part_l, out, lse, B, s_q, h_q, rows, num_splits};
  const long long nrows = static_cast<long long>(B) * rows;
  mla_combine_kernel<<<static_cast<unsigned>((nrows + 3) / 4), 128, 0, stream>>>(c);
  return cudaGetLastError();
}

int mla_decode_get_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gqa::mla::g_mla_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(gqa::mla::g_mla_status, &z, sizeof(int));
  }
  return v;
}

}  // extern "C"
