// DSA-style sparse decode (the reference's roadmap kernel K3: "indexer +
// top-k + sparse gather", README.md "Roadmap"; no reference code exists,
// kernels/sparse_decode/ is empty).  Three kernels; the attention over the
// selected tokens is the MLA decode (mla_decode.cu) on the gathered rows.
//
//   indexer   I[b, i, t] = sum_j w[b, i, j] * relu(q_idx[b, i, j, :] . k_idx[t, :])
//             for t < visible(b, i), DeepSeek sparse attention's lightning
//             indexer: 128-dim index keys paged like the latent cache.
//             tcgen05: S^T[128 tokens, s_q * H] = K_tile . Q^T (8 MMAs of
//             M = 128 per two pages), ReLU and the weighted head sum in the
//             TMEM-reading epilogue (one token per thread).
//   top-k     the k largest scores of each (b, i), ties to the lower token
//             index, in ascending token order, -1 padded: a 4-pass radix
//             select (8 bits per pass) and an ordered block compaction.
//   gather    the selected latent rows into contiguous 64-token pages.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "dsa_decode.h"
#include "gqa_ptx.cuh"
#include "umma_ptx.cuh"

namespace gqa {
namespace dsa {

constexpr int kPage = 64;                 // tokens per page
constexpr int kTile = 128;                // tokens per MMA tile (two pages)
constexpr int kBox = kPage * 128;         // one 64-dim box of a page: 8 KB
constexpr int kTileBytes = 2 * 2 * kBox;  // two pages x two 64-dim columns: 32 KB
constexpr int kStages = 4;
constexpr int kThreads = 192;             // producer, MMA, 4 epilogue warps

__device__ int g_dsa_status;

__device__ __forceinline__ void raise(int bit) { atomicOr(&g_dsa_status, bit); }

__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

struct IndexerParams {
  CUtensorMap tm_k;  // [num_blocks * 64, 128] bf16, box {64, 64}, 128B swizzle
  CUtensorMap tm_q;  // [B * s_q * H, 128] bf16, box {64, NQ}, 128B swizzle
  const float* w;    // [B, s_q, H]
  const int* block_table;
  const int* seq_lens;
  float* scores;     // [B, s_q, stride]
  long long stride;
  int B, s_q, H, max_blocks, num_blocks, causal, num_splits;
};

// Smem: Q (two 64-dim columns of NQ rows), 4-stage ring of 128-token tiles
// laid out column-major (column c: page A rows 0-63, page B rows 64-127),
// weights, barriers.
template <int NQ>
struct IdxGeom {
  static constexpr int kQBytes = 2 * NQ * 128;
  static constexpr int kRing = kQBytes;
  static constexpr int kW = kRing + kStages * kTileBytes;
  static constexpr int kSmall = kW + NQ * 4;
  static constexpr int kSmem = kSmall + 256 + 1024;
  static constexpr uint32_t kTmemCols = 2 * NQ;  // S^T double buffer
};

template <int NQ>
__global__ void __launch_bounds__(kThreads, 1)
    dsa_indexer_kernel(const __grid_constant__ IndexerParams p) {
  using G = IdxGeom<NQ>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sQ = s_base, sRing = s_base + G::kRing;
  float* w_s = reinterpret_cast<float*>(smem + G::kW);
  const uint32_t bars = s_base + G::kSmall;
  const uint32_t bar_q = bars, bar_full = bars + 8, bar_empty = bars + 40, bar_sfull = bars + 72,
                 bar_sfree = bars + 88, bar_fin = bars + 104;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kSmall + 112);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / p.num_splits, sp = blockIdx.x % p.num_splits;
  const int S = max(0, min(p.seq_lens[b], p.max_blocks * kPage));
  const int tiles = (S + kTile - 1) / kTile;
  const int chunk = (tiles + p.num_splits - 1) / p.num_splits;
  const int tl0 = min(tiles, sp * chunk), tl1 = min(tiles, tl0 + chunk);
  const int ntiles = tl1 - tl0;
  const int pages = (S + kPage - 1) / kPage;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_sfull + 8 * s, 1);
      mbar_init(bar_sfree + 8 * s, 4);  // one arrival per epilogue warp
    }
    mbar_init(bar_fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), G::kTmemCols);
    tmem_relinquish();
  }
  for (int e = threadIdx.x; e < NQ; e += blockDim.x)
    w_s[e] = e < p.s_q * p.H ? p.w[static_cast<size_t>(b) * p.s_q * p.H + e] : 0.f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0 && ntiles > 0) {
      mbar_arrive_expect_tx(bar_q, static_cast<uint32_t>(G::kQBytes));
      for (int c = 0; c < 2; ++c)
        tma_load_2d(sQ + c * NQ * 128, &p.tm_q, 64 * c, b * p.s_q * p.H, bar_q);
      const int* bt = p.block_table + static_cast<size_t>(b) * p.max_blocks;
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(bar_empty + 8 * s, ((t - kStages) / kStages) & 1)) {
          raise(1);
          break;
        }
        const int pg = 2 * (tl0 + t);
        const int npg = min(2, pages - pg);  // the second page may not exist
        mbar_arrive_expect_tx(bar_full + 8 * s, static_cast<uint32_t>(npg * 2 * kBox));
        for (int h = 0; h < npg; ++h) {
          int page = __ldg(bt + pg + h);
          if (page < 0 || page >= p.num_blocks) {
            raise(2);
            page = 0;
          }
          for (int c = 0; c < 2; ++c)
            tma_load_2d(sRing + s * kTileBytes + c * 2 * kBox + h * kBox, &p.tm_k, 64 * c,
                        page * kPage, bar_full + 8 * s);
        }
        issued = t + 1;
      }
      // every issued copy has landed before the CTA may exit
      if (!mbar_wait(bar_q, 0)) raise(1);
      for (int t = max(0, issued - kStages); t < issued; ++t)
        if (!mbar_wait(bar_full + 8 * (t % kStages), (t / kStages) & 1)) raise(1);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    constexpr uint32_t idesc = umma_idesc_bf16(128, NQ, false, false);
    bool ok = true;
    if (ntiles > 0) ok = wait_warp(bar_q, 0);
    for (int t = 0; t < ntiles && ok; ++t) {
      const int s = t % kStages, buf = t & 1;
      if (!wait_warp(bar_full + 8 * s, (t / kStages) & 1)) { ok = false; break; }
      if (t >= 2 && !wait_warp(bar_sfree + 8 * buf, ((t - 2) >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        // unrolled, descriptors as constant offsets (16-byte units) from two
        // bases: rebuilding them per MMA roughly doubles the issue cost
        const uint64_t a0 = umma_smem_desc(sRing + s * kTileBytes, 16, 1024, kSwizzle128);
        const uint64_t b0 = umma_smem_desc(sQ, 16, 1024, kSwizzle128);
        #pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = i >> 2, kk = i & 3;
          umma_bf16_ss(tmem + buf * NQ, a0 + static_cast<uint64_t>((c * 2 * kBox + kk * 32) >> 4),
                       b0 + static_cast<uint64_t>((c * NQ * 128 + kk * 32) >> 4), idesc, i != 0);
        }
        umma_commit(bar_sfull + 8 * buf);
        umma_commit(bar_empty + 8 * s);
      }
      __syncwarp();
    }
    if (!ok) raise(1);
    // every MMA this thread issued has completed before TMEM is released
    if (lane == 0) umma_commit(bar_fin);
    __syncwarp();
    if (!wait_warp(bar_fin, 0)) raise(1);
  } else {
    // ------------------- epilogue: one token row per thread --------------------
    const int tq = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(32 * tq) << 16;
    const int row = 32 * tq + lane;  // token within the tile
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t & 1;
      if (ok && !wait_warp(bar_sfull + 8 * buf, (t >> 1) & 1)) ok = false;
      tc_fence_after();
      const int tok = (tl0 + t) * kTile + row;
      float acc[2] = {0.f, 0.f};  // per query position (s_q <= 2)
      #pragma unroll
      for (int c16 = 0; c16 < NQ / 16; ++c16) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + buf * NQ + 16 * c16, r);
        tmem_wait_ld();
        #pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int col = 16 * c16 + k;
          const float v = fmaxf(__uint_as_float(r[k]), 0.f);
          if (col < p.H)
            acc[0] += w_s[col] * v;
          else
            acc[1] += w_s[col] * v;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree + 8 * buf);
      for (int i = 0; i < p.s_q; ++i) {
        const int vis = p.causal ? max(0, min(S, S - p.s_q + 1 + i)) : S;
        if (tok < S)
          p.scores[(static_cast<size_t>(b) * p.s_q + i) * p.stride + tok] =
              tok < vis ? acc[i] : -INFINITY;
      }
    }
    if (!ok) raise(1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, G::kTmemCols);
  }
}

// ---- top-k: radix select + ordered compaction --------------------------------

// Order-preserving map of a float to an unsigned key (larger float, larger
// key); -0 and +0 map to the same key, so they tie like equal values.
__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct TopkParams {
  const float* scores;
  long long stride;
  const int* seq_lens;
  int* indices;  // [B, s_q, k]
  int* counts;   // [B, s_q] selected tokens (min(k, visible)), or null
  int B, s_q, k, max_tokens, causal;
};

constexpr int kTopkThreads = 1024;

// Inclusive block scan of one int per thread; also returns the block total.
// Every thread of the block must call it.
__device__ __forceinline__ int block_scan(int v, int* sh, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
  #pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = sh[lane];
    #pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += y;
    }
    sh[lane] = s;
  }
  __syncthreads();
  const int r = x + (warp > 0 ? sh[warp - 1] : 0);
  *total = sh[31];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kTopkThreads) dsa_topk_kernel(const __grid_constant__ TopkParams p) {
  __shared__ int hist[256];
  __shared__ int sh[32];
  __shared__ uint32_t sh_prefix;
  __shared__ int sh_need;
  const int r = blockIdx.x;  // (b, i)
  const int b = r / p.s_q, i = r % p.s_q;
  const int S = max(0, min(p.seq_lens[b], p.max_tokens));
  const int vis = p.causal ? max(0, min(S, S - p.s_q + 1 + i)) : S;
  const float* sc = p.scores + static_cast<size_t>(r) * p.stride;
  int* out = p.indices + static_cast<size_t>(r) * p.k;
  const int k = p.k;
  if (p.counts && threadIdx.x == 0) p.counts[r] = min(k, vis);
  if (vis <= k) {  // every visible token is selected
    for (int e = threadIdx.x; e < k; e += blockDim.x) out[e] = e < vis ? e : -1;
    return;
  }
  // radix select of the k-th largest key, 8 bits per pass from the top
  uint32_t prefix = 0, pmask = 0;
  int need = k;  // keys still to take at or below the current prefix
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int e = threadIdx.x; e < 256; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    for (int t = threadIdx.x; t < vis; t += blockDim.x) {
      const uint32_t key = order_key(sc[t]);
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int above = 0, dig = 255;
      for (; dig > 0; --dig) {
        if (above + hist[dig] >= need) break;
        above += hist[dig];
      }
      sh_prefix = prefix | (static_cast<uint32_t>(dig) << shift);
      sh_need = need - above;
    }
    __syncthreads();
    prefix = sh_prefix;
    need = sh_need;
    pmask |= 255u << shift;
    __syncthreads();
  }
  // prefix = threshold key T: take every key > T and the first `need` keys
  // equal to T (lowest token indices), in token order
  int base_out = 0, eq_seen = 0;
  for (int c0 = 0; c0 < vis; c0 += blockDim.x) {
    const int t = c0 + threadIdx.x;
    const uint32_t key = t < vis ? order_key(sc[t]) : 0u;
    const int eq = t < vis && key == prefix;
    const int gt = t < vis && key > prefix;
    int eq_total;
    const int eq_rank = block_scan(eq, sh, &eq_total) - eq + eq_seen;  // exclusive
    const int sel = gt || (eq && eq_rank < need);
    int sel_total;
    const int pos = block_scan(sel, sh, &sel_total) - sel + base_out;
    if (sel) out[pos] = t;
    base_out += sel_total;
    eq_seen += eq_total;
  }
  for (int e = base_out + threadIdx.x; e < k; e += blockDim.x) out[e] = -1;
}

// ---- gather of the selected latent rows ---------------------------------------

struct GatherParams {
  const uint4* kv;      // [num_blocks, 64, 576] bf16 as 16-byte units (72 per row)
  const int* block_table;
  const int* indices;   // [B, s_q, k]
  uint4* out;           // [B * s_q, kpad, 576]
  int B, s_q, k, kpad, max_blocks, num_blocks;
};

constexpr int kRowUnits = 576 * 2 / 16;  // 72

__global__ void __launch_bounds__(256) dsa_gather_kernel(const __grid_constant__ GatherParams p) {
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long rows = static_cast<long long>(p.B) * p.s_q * p.kpad;
  if (wid >= rows) return;
  const int slot = static_cast<int>(wid % p.kpad);
  const long long r = wid / p.kpad;  // (b, i)
  const int b = static_cast<int>(r / p.s_q);
  const int t = slot < p.k ? __ldg(p.indices + r * p.k + slot) : -1;
  uint4* dst = p.out + wid * kRowUnits;
  if (t < 0 || t >= p.max_blocks * kPage) {
    for (int u = lane; u < kRowUnits; u += 32) dst[u] = make_uint4(0, 0, 0, 0);
    return;
  }
  int page = __ldg(p.block_table + static_cast<size_t>(b) * p.max_blocks + t / kPage);
  if (page < 0 || page >= p.num_blocks) {
    raise(2);
    page = 0;
  }
  const uint4* src = p.kv + (static_cast<size_t>(page) * kPage + t % kPage) * kRowUnits;
  for (int u = lane; u < kRowUnits; u += 32) dst[u] = __ldg(src + u);
}

}  // namespace dsa
}  // namespace gqa

// ================================ host side =================================

namespace {

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

// 2-D bf16 map over rows of 128 elements (256 bytes), box 64 x box_rows,
// 128-byte swizzle.
bool make_map128(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {128u, static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {256u};
  cuuint32_t box[2] = {64u, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

cudaError_t dsa_indexer_launch(const gqa_bf16* q_idx, const float* w_idx, const gqa_bf16* k_idx,
                               const int* block_table, const int* seq_lens, float* scores,
                               long long scores_stride, int B, int s_q, int n_heads,
                               int page_size, int max_blocks, int num_blocks, int causal,
                               cudaStream_t stream) {
  using namespace gqa::dsa;
  const int NQ = s_q * n_heads;
  if (B < 0 || s_q < 1 || s_q > 2 || page_size != kPage || max_blocks <= 0 || num_blocks <= 0 ||
      (NQ != 64 && NQ != 128) || scores_stride < static_cast<long long>(max_blocks) * kPage)
    return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  if (!q_idx || !w_idx || !k_idx || !block_table || !seq_lens || !scores)
    return cudaErrorInvalidValue;
  if (!aligned16(q_idx) || !aligned16(k_idx)) return cudaErrorMisalignedAddress;
  IndexerParams p{};
  if (!make_map128(&p.tm_k, k_idx, static_cast<uint64_t>(num_blocks) * kPage, kPage) ||
      !make_map128(&p.tm_q, q_idx, static_cast<uint64_t>(B) * NQ, static_cast<uint32_t>(NQ)))
    return cudaErrorInvalidValue;
  p.w = w_idx;
  p.block_table = block_table;
  p.seq_lens = seq_lens;
  p.scores = scores;
  p.stride = scores_stride;
  p.B = B;
  p.s_q = s_q;
  p.H = n_heads;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.causal = causal ? 1 : 0;
  // splits of each request's 128-token tiles: enough CTAs to fill the GPU
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int max_tiles = (max_blocks * kPage + kTile - 1) / kTile;
  int ns = (sms + B - 1) / B;
  ns = ns < 1 ? 1 : (ns > max_tiles ? max_tiles : ns);
  p.num_splits = ns;
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    const cudaError_t e1 = cudaFuncSetAttribute(
        dsa_indexer_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, IdxGeom<64>::kSmem);
    const cudaError_t e2 = cudaFuncSetAttribute(
        dsa_indexer_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, IdxGeom<128>::kSmem);
    attr_err = e1 != cudaSuccess ? e1 : e2;
  });
  if (attr_err != cudaSuccess) return attr_err;
  const long long grid = static_cast<long long>(B) * ns;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (NQ == 64)
    dsa_indexer_kernel<64><<<static_cast<unsigned>(grid), kThreads, IdxGeom<64>::kSmem, stream>>>(p);
  else
    dsa_indexer_kernel<128>
        <<<static_cast<unsigned>(grid), kThreads, IdxGeom<128>::kSmem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t dsa_topk_launch(const float* scores, long long scores_stride, const int* seq_lens,
                            int B, int s_q, int k, int max_tokens, int causal, int* indices,
                            int* counts, cudaStream_t stream) {
  using namespace gqa::dsa;
  if (B < 0 || s_q < 1 || k < 1 || max_tokens < 0 || scores_stride < max_tokens)
    return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  if (!scores || !seq_lens || !indices) return cudaErrorInvalidValue;
  TopkParams p{scores, scores_stride, seq_lens, indices, counts, B, s_q, k, max_tokens,
               causal ? 1 : 0};
  dsa_topk_kernel<<<static_cast<unsigned>(B * s_q), kTopkThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t dsa_gather_launch(const gqa_bf16* kv_cache, const int* block_table,
                              const int* indices, int B, int s_q, int k, int max_blocks,
                              int num_blocks, gqa_bf16* gathered, cudaStream_t stream) {
  using namespace gqa::dsa;
  if (B < 0 || s_q < 1 || k < 1 || max_blocks <= 0 || num_blocks <= 0) return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  if (!kv_cache || !block_table || !indices || !gathered) return cudaErrorInvalidValue;
  if (!aligned16(kv_cache) || !aligned16(gathered)) return cudaErrorMisalignedAddress;
  const int kpad = (k + kPage - 1) / kPage * kPage;
  GatherParams p{reinterpret_cast<const uint4*>(kv_cache), block_table, indices,
                 reinterpret_cast<uint4*>(gathered), B, s_q, k, kpad, max_blocks, num_blocks};
  const long long rows = static_cast<long long>(B) * s_q * kpad;
  const long long blocks = (rows * 32 + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  dsa_gather_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

int dsa_decode_get_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gqa::dsa::g_dsa_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(gqa::dsa::g_dsa_status, &z, sizeof(int));
  }
  return v;
}

}  // extern "C"
