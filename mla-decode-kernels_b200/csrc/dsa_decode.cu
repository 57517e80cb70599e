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

#include "device_once.h"
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
  int B, s_q, H, max_blocks, num_blocks, causal;
};

constexpr int kMaxBatch = 4096;  // requests per launch (the host splits larger batches)

// Smem: two Q buffers (two 64-dim columns of NQ rows each: a CTA's range of
// tiles can span requests, and the next request's Q loads while the last
// tiles of the current one are multiplied), a 4-stage ring of 128-token
// tiles laid out column-major (column c: page A rows 0-63, page B rows
// 64-127), the per-request weights, the tile prefix over the batch, barriers.
template <int NQ>
struct IdxGeom {
  static constexpr int kQBytes = 2 * NQ * 128;
  static constexpr int kRing = 2 * kQBytes;
  static constexpr int kW = kRing + kStages * kTileBytes;
  static constexpr int kPrefix = kW + NQ * 4;
  static constexpr int kSmall = (kPrefix + (kMaxBatch + 1) * 4 + 15) / 16 * 16;
  static constexpr int kSmem = kSmall + 256 + 1024;
  static constexpr uint32_t kTmemCols = 2 * NQ;  // S^T double buffer
  static_assert(kSmem <= 232448, "shared memory");
};

// Persistent: one CTA per SM, and CTA c takes tiles [c T / G, (c + 1) T / G)
// of the batch's T 128-token tiles (request by request), so every SM scans
// the same number of index keys whatever the length distribution.
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
  int* tstart = reinterpret_cast<int*>(smem + G::kPrefix);  // [B + 1] first tile of each request
  const uint32_t bars = s_base + G::kSmall;
  const uint32_t bar_q = bars, bar_qfree = bars + 16, bar_full = bars + 32, bar_empty = bars + 64,
                 bar_sfull = bars + 96, bar_sfree = bars + 112, bar_fin = bars + 128;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kSmall + 144);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int max_tokens = p.max_blocks * kPage;
  // tile prefix over the batch (block-wide scan in chunks of blockDim)
  {
    __shared__ int carry_s;
    __shared__ int wsum[kThreads / 32];
    if (threadIdx.x == 0) carry_s = 0;
    __syncthreads();
    for (int base = 0; base < p.B; base += blockDim.x) {
      const int b = base + threadIdx.x;
      const int S = b < p.B ? max(0, min(p.seq_lens[b], max_tokens)) : 0;
      const int n = (S + kTile - 1) / kTile;
      int x = n;
      #pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
      }
      if (lane == 31) wsum[warp] = x;
      __syncthreads();
      int before = carry_s;
      for (int w2 = 0; w2 < warp; ++w2) before += wsum[w2];
      if (b < p.B) tstart[b] = before + x - n;
      __syncthreads();
      if (threadIdx.x == blockDim.x - 1) carry_s = before + x;
      __syncthreads();
    }
    if (threadIdx.x == 0) tstart[p.B] = carry_s;
  }
  if (threadIdx.x == 0) {
    for (int j = 0; j < 2; ++j) {
      mbar_init(bar_q + 8 * j, 1);
      mbar_init(bar_qfree + 8 * j, 1);
      mbar_init(bar_sfull + 8 * j, 1);
      mbar_init(bar_sfree + 8 * j, 4);  // one arrival per epilogue warp
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), G::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const long long T = tstart[p.B];
  const int g0 = static_cast<int>(T * blockIdx.x / gridDim.x);
  const int g1 = static_cast<int>(T * (blockIdx.x + 1) / gridDim.x);
  const int ntiles = g1 - g0;
  // every role walks the same tiles: request b of global tile g
  auto req_of = [&](int g, int b) {
    while (b + 1 < p.B && tstart[b + 1] <= g) ++b;
    return b;
  };
  int b_first = 0;
  if (ntiles > 0) {  // binary search for the request of the first tile
    int lo = 0, hi = p.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tstart[mid] <= g0) lo = mid;
      else hi = mid - 1;
    }
    b_first = lo;
  }

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0 && ntiles > 0) {
      int b = b_first, ord = -1, prev = -1, issued = 0;
      // page ids of the next tile, loaded while the current one is in flight
      // (the request's length and table row only when the request changes)
      int cur_b = -1, pages_b = 0, npg = 0, pid0 = 0, pid1 = 0;
      const int* bt_b = p.block_table;
      auto fetch_ids = [&](int t, int bb) {
        if (bb != cur_b) {
          cur_b = bb;
          const int S = max(0, min(p.seq_lens[bb], max_tokens));
          pages_b = (S + kPage - 1) / kPage;
          bt_b = p.block_table + static_cast<size_t>(bb) * p.max_blocks;
        }
        const int pg = 2 * (g0 + t - tstart[bb]);
        npg = min(2, pages_b - pg);  // the second page may not exist
        pid0 = __ldg(bt_b + pg);
        pid1 = npg > 1 ? __ldg(bt_b + pg + 1) : 0;
      };
      fetch_ids(0, b_first);
      for (int t = 0; t < ntiles; ++t) {
        const int g = g0 + t;
        b = req_of(g, b);
        if (b != prev) {  // Q of request b into buffer ord & 1
          ++ord;
          prev = b;
          const int qb = ord & 1;
          if (ord >= 2 && !mbar_wait(bar_qfree + 8 * qb, ((ord - 2) >> 1) & 1)) {
            raise(1);
            break;
          }
          mbar_arrive_expect_tx(bar_q + 8 * qb, static_cast<uint32_t>(G::kQBytes));
          for (int c = 0; c < 2; ++c)
            tma_load_2d(sQ + qb * G::kQBytes + c * NQ * 128, &p.tm_q, 64 * c, b * p.s_q * p.H,
                        bar_q + 8 * qb);
        }
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(bar_empty + 8 * s, ((t - kStages) / kStages) & 1)) {
          raise(1);
          break;
        }
        const int n = npg;
        mbar_arrive_expect_tx(bar_full + 8 * s, static_cast<uint32_t>(n * 2 * kBox));
        for (int h = 0; h < n; ++h) {
          int page = h ? pid1 : pid0;
          if (page < 0 || page >= p.num_blocks) {
            raise(2);
            page = 0;
          }
          for (int c = 0; c < 2; ++c)
            tma_load_2d(sRing + s * kTileBytes + c * 2 * kBox + h * kBox, &p.tm_k, 64 * c,
                        page * kPage, bar_full + 8 * s);
        }
        issued = t + 1;
        if (t + 1 < ntiles) fetch_ids(t + 1, req_of(g + 1, b));
      }
      // every issued copy has landed before the CTA may exit
      for (int o = max(0, ord - 1); o <= ord; ++o)
        if (!mbar_wait(bar_q + 8 * (o & 1), (o >> 1) & 1)) raise(1);
      for (int t = max(0, issued - kStages); t < issued; ++t)
        if (!mbar_wait(bar_full + 8 * (t % kStages), (t / kStages) & 1)) raise(1);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    constexpr uint32_t idesc = umma_idesc_bf16(128, NQ, false, false);
    bool ok = true;
    int b = b_first, ord = -1, prev = -1;
    for (int t = 0; t < ntiles && ok; ++t) {
      const int g = g0 + t;
      b = req_of(g, b);
      if (b != prev) {
        ++ord;
        prev = b;
        if (!wait_warp(bar_q + 8 * (ord & 1), (ord >> 1) & 1)) { ok = false; break; }
      }
      const int qb = ord & 1;
      const int s = t % kStages, buf = t & 1;
      if (!wait_warp(bar_full + 8 * s, (t / kStages) & 1)) { ok = false; break; }
      if (t >= 2 && !wait_warp(bar_sfree + 8 * buf, ((t - 2) >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      // the request's last tile of this CTA releases its Q buffer
      const bool last_of_req = t + 1 == ntiles || tstart[b + 1] <= g + 1;
      if (lane == 0) {
        // unrolled, descriptors as constant offsets (16-byte units) from two
        // bases: rebuilding them per MMA roughly doubles the issue cost
        const uint64_t a0 = umma_smem_desc(sRing + s * kTileBytes, 16, 1024, kSwizzle128);
        const uint64_t b0 = umma_smem_desc(sQ + qb * G::kQBytes, 16, 1024, kSwizzle128);
        #pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = i >> 2, kk = i & 3;
          umma_bf16_ss(tmem + buf * NQ, a0 + static_cast<uint64_t>((c * 2 * kBox + kk * 32) >> 4),
                       b0 + static_cast<uint64_t>((c * NQ * 128 + kk * 32) >> 4), idesc, i != 0);
        }
        umma_commit(bar_sfull + 8 * buf);
        umma_commit(bar_empty + 8 * s);
        if (last_of_req) umma_commit(bar_qfree + 8 * qb);
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
    const int et = threadIdx.x - 64;  // 0..127
    bool ok = true;
    int b = b_first, prev = -1, S = 0;
    for (int t = 0; t < ntiles; ++t) {
      const int g = g0 + t;
      b = req_of(g, b);
      if (b != prev) {  // the request's head weights
        prev = b;
        S = max(0, min(p.seq_lens[b], max_tokens));
        named_bar_sync(1, 128);
        for (int e = et; e < NQ; e += 128)
          w_s[e] = e < p.s_q * p.H ? p.w[static_cast<size_t>(b) * p.s_q * p.H + e] : 0.f;
        named_bar_sync(1, 128);
      }
      const int buf = t & 1;
      if (ok && !wait_warp(bar_sfull + 8 * buf, (t >> 1) & 1)) ok = false;
      tc_fence_after();
      const int tok = (g - tstart[b]) * kTile + row;
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
  // Optional: the selected tokens' physical cache rows (block id * 64 +
  // slot, -1 padded) into rows [B, s_q, k], resolved through block_table.
  const int* block_table;
  int* rows;
  int max_blocks, num_blocks;
};

// Cache row of token t of request b: block_table[b, t / 64] * 64 + t % 64.
// A block id outside [0, num_blocks) sets status bit 1 and reads block 0.
__device__ __forceinline__ int cache_row(const TopkParams& p, int b, int t) {
  int page = __ldg(p.block_table + static_cast<size_t>(b) * p.max_blocks + (t >> 6));
  if (static_cast<unsigned>(page) >= static_cast<unsigned>(p.num_blocks)) {
    raise(2);
    page = 0;
  }
  return page * kPage + (t & (kPage - 1));
}

constexpr int kTopkThreads = 1024;
constexpr int kTopkSmemKeys = 40 * 1024;  // rows up to this many tokens keep their keys in smem
constexpr int kHistStride = 257;          // per-warp histogram row (padded against bank overlap)

// One CTA per query row.  Keys (order-preserving integers of the scores) are
// visited in chunks of 1024 tokens, token c * 1024 + tid by thread tid, so
// every pass reads them coalesced.  Four 8-bit radix passes find the k-th
// largest key T and how many keys equal to T to take: each warp counts into
// its own histogram, a thread adds runs of equal digits before touching it
// (the leading digits of similar scores coincide), and one warp turns the
// 256 bins into the next digit with a parallel scan.  The selection is then
// written in token order by ballots over the same chunks, with the chunk x
// warp offsets scanned by one warp (two block barriers per 32 chunks).
template <bool kSmemKeys>
__global__ void __launch_bounds__(kTopkThreads) dsa_topk_kernel(const __grid_constant__ TopkParams p) {
  extern __shared__ uint32_t keys[];
  __shared__ int hw[32 * kHistStride];
  __shared__ int offs[32 * 32];  // [chunk][warp] counts, then exclusive offsets
  __shared__ uint32_t sh_prefix;
  __shared__ int sh_need, sh_eq, sh_total;
  const int r = blockIdx.x;  // (b, i)
  const int b = r / p.s_q, i = r % p.s_q;
  const int S = max(0, min(p.seq_lens[b], p.max_tokens));
  const int vis = p.causal ? max(0, min(S, S - p.s_q + 1 + i)) : S;
  const float* sc = p.scores + static_cast<size_t>(r) * p.stride;
  int* out = p.indices + static_cast<size_t>(r) * p.k;
  int* rows_out = p.rows ? p.rows + static_cast<size_t>(r) * p.k : nullptr;
  const int k = p.k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (p.counts && tid == 0) p.counts[r] = min(k, vis);
  if (vis <= k) {  // every visible token is selected
    for (int e = tid; e < k; e += blockDim.x) {
      out[e] = e < vis ? e : -1;
      if (rows_out) rows_out[e] = e < vis ? cache_row(p, b, e) : -1;
    }
    return;
  }
  if (kSmemKeys) {
    // eight loads in flight per thread, then their keys
    int t = tid;
    for (; t + 7 * kTopkThreads < vis; t += 8 * kTopkThreads) {
      float v[8];
      #pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(sc + t + u * kTopkThreads);
      #pragma unroll
      for (int u = 0; u < 8; ++u) keys[t + u * kTopkThreads] = order_key(v[u]);
    }
    for (; t < vis; t += kTopkThreads) keys[t] = order_key(__ldg(sc + t));
  }
  auto key_at = [&](int t) -> uint32_t { return kSmemKeys ? keys[t] : order_key(sc[t]); };
  const int nch = (vis + blockDim.x - 1) / blockDim.x;
  // ---- radix select of the k-th largest key, 8 bits per pass from the top
  uint32_t prefix = 0, pmask = 0;
  int need = k, eq_total = 0;  // keys still to take at or below the current prefix
  int* hist = hw;              // bins after the per-warp reduction (row 0)
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int e = tid; e < 32 * kHistStride; e += blockDim.x) hw[e] = 0;
    __syncthreads();
    int run_d = -1, run_n = 0;
    for (int c = 0; c < nch; ++c) {
      const int t = c * blockDim.x + tid;
      if (t < vis) {
        const uint32_t key = key_at(t);
        if ((key & pmask) == prefix) {
          const int d = static_cast<int>((key >> shift) & 255u);
          if (d != run_d) {
            if (run_n) atomicAdd(&hw[warp * kHistStride + run_d], run_n);
            run_d = d;
            run_n = 0;
          }
          ++run_n;
        }
      }
    }
    if (run_n) atomicAdd(&hw[warp * kHistStride + run_d], run_n);
    __syncthreads();
    int bin_sum = 0;
    if (tid < 256) {
      #pragma unroll 8
      for (int w = 0; w < 32; ++w) bin_sum += hw[w * kHistStride + tid];
    }
    __syncthreads();
    if (tid < 256) hist[tid] = bin_sum;
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255 - 8 l down to 248 - 8 l (descending digits)
      int c8[8], local = 0;
      #pragma unroll
      for (int j = 0; j < 8; ++j) {
        c8[j] = hist[255 - 8 * lane - j];
        local += c8[j];
      }
      int incl = local;
      #pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      const int above = incl - local;  // keys in the bins above this lane's
      if (above < need && need <= incl) {
        int a = above, j = 0;
        for (; j < 7; ++j) {
          if (a + c8[j] >= need) break;
          a += c8[j];
        }
        const int dig = 255 - 8 * lane - j;
        sh_prefix = prefix | (static_cast<uint32_t>(dig) << shift);
        sh_need = need - a;
        sh_eq = c8[j];
      }
    }
    __syncthreads();
    prefix = sh_prefix;
    need = sh_need;
    eq_total = sh_eq;
    pmask |= 255u << shift;
  }
  // ---- ordered compaction: every key > T and the first `need` keys == T
  const uint32_t T = prefix;
  const bool all_ties = need == eq_total;  // block-uniform
  const unsigned lt = (1u << lane) - 1u;
  int sel_base = 0, eq_base = 0;
  // one warp turns the [chunk][warp] counts of up to 32 chunks into exclusive
  // offsets (chunk-major, token order) and the running total
  auto scan_offsets = [&](int nc, int base) {
    __syncthreads();
    if (warp == 0) {
      int v[32], local = 0;
      #pragma unroll
      for (int w = 0; w < 32; ++w) {
        v[w] = lane < nc ? offs[lane * 32 + w] : 0;
        local += v[w];
      }
      int incl = local;
      #pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      int run = base + incl - local;
      if (lane < nc) {
        #pragma unroll
        for (int w = 0; w < 32; ++w) {
          offs[lane * 32 + w] = run;
          run += v[w];
        }
      }
      if (lane == 31) sh_total = base + incl;
    }
    __syncthreads();
  };
  for (int c0 = 0; c0 < nch; c0 += 32) {
    const int nc = min(32, nch - c0);
    uint32_t eq_bits = 0, gt_bits = 0;  // this thread's keys of the super-chunk
    for (int c = 0; c < nc; ++c) {
      const int t = (c0 + c) * blockDim.x + tid;
      const uint32_t key = t < vis ? key_at(t) : 0u;
      if (t < vis && key > T) gt_bits |= 1u << c;
      if (t < vis && key == T) eq_bits |= 1u << c;
    }
    uint32_t sel_bits = gt_bits;
    if (all_ties) {
      sel_bits |= eq_bits;
    } else {
      // ranks of the ties in token order
      for (int c = 0; c < nc; ++c) {
        const unsigned bal = __ballot_sync(0xffffffffu, (eq_bits >> c) & 1u);
        if (lane == 0) offs[c * 32 + warp] = __popc(bal);
      }
      scan_offsets(nc, eq_base);
      for (int c = 0; c < nc; ++c) {
        const unsigned bal = __ballot_sync(0xffffffffu, (eq_bits >> c) & 1u);
        if ((eq_bits >> c) & 1u) {
          const int rank = offs[c * 32 + warp] + __popc(bal & lt);
          if (rank < need) sel_bits |= 1u << c;
        }
      }
      eq_base = sh_total;
      __syncthreads();  // offs is rewritten below
    }
    for (int c = 0; c < nc; ++c) {
      const unsigned bal = __ballot_sync(0xffffffffu, (sel_bits >> c) & 1u);
      if (lane == 0) offs[c * 32 + warp] = __popc(bal);
    }
    scan_offsets(nc, sel_base);
    for (int c = 0; c < nc; ++c) {
      const unsigned bal = __ballot_sync(0xffffffffu, (sel_bits >> c) & 1u);
      if ((sel_bits >> c) & 1u) {
        const int pos = offs[c * 32 + warp] + __popc(bal & lt);
        const int tok = (c0 + c) * blockDim.x + tid;
        out[pos] = tok;
        if (rows_out) rows_out[pos] = cache_row(p, b, tok);
      }
    }
    sel_base = sh_total;
    __syncthreads();  // offs is rewritten by the next super-chunk
  }
  // vis > k: exactly k tokens were selected, so there is no padding
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
  static gqa::DeviceOnce attr_once;
  const cudaError_t attr_err = attr_once.run([] {
    const cudaError_t e1 = cudaFuncSetAttribute(
        dsa_indexer_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, IdxGeom<64>::kSmem);
    const cudaError_t e2 = cudaFuncSetAttribute(
        dsa_indexer_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, IdxGeom<128>::kSmem);
    return e1 != cudaSuccess ? e1 : e2;
  });
  if (attr_err != cudaSuccess) return attr_err;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // batches of at most kMaxBatch requests (the tile prefix lives in smem)
  for (int b0 = 0; b0 < B; b0 += kMaxBatch) {
    const int nb = B - b0 < kMaxBatch ? B - b0 : kMaxBatch;
    IndexerParams p{};
    const gqa_bf16* q0 = q_idx + static_cast<size_t>(b0) * NQ * 128;
    if (!make_map128(&p.tm_k, k_idx, static_cast<uint64_t>(num_blocks) * kPage, kPage) ||
        !make_map128(&p.tm_q, q0, static_cast<uint64_t>(nb) * NQ, static_cast<uint32_t>(NQ)))
      return cudaErrorInvalidValue;
    p.w = w_idx + static_cast<size_t>(b0) * NQ;
    p.block_table = block_table + static_cast<size_t>(b0) * max_blocks;
    p.seq_lens = seq_lens + b0;
    p.scores = scores + static_cast<size_t>(b0) * s_q * scores_stride;
    p.stride = scores_stride;
    p.B = nb;
    p.s_q = s_q;
    p.H = n_heads;
    p.max_blocks = max_blocks;
    p.num_blocks = num_blocks;
    p.causal = causal ? 1 : 0;
    // one CTA per SM; fewer for small batches (at least one tile each)
    const long long max_tiles = static_cast<long long>(nb) * ((max_blocks * kPage + kTile - 1) / kTile);
    const int grid = static_cast<int>(max_tiles < sms ? max_tiles : sms);
    if (NQ == 64)
      dsa_indexer_kernel<64><<<grid, kThreads, IdxGeom<64>::kSmem, stream>>>(p);
    else
      dsa_indexer_kernel<128><<<grid, kThreads, IdxGeom<128>::kSmem, stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // extern "C"

namespace {

cudaError_t topk_impl(const float* scores, long long scores_stride, const int* seq_lens, int B,
                      int s_q, int k, int max_tokens, int causal, int* indices, int* counts,
                      const int* block_table, int max_blocks, int num_blocks, int* rows,
                      cudaStream_t stream) {
  using namespace gqa::dsa;
  if (B < 0 || s_q < 1 || k < 1 || max_tokens < 0 || scores_stride < max_tokens)
    return cudaErrorInvalidValue;
  if (rows && (!block_table || max_blocks <= 0 || num_blocks <= 0 ||
               max_tokens > static_cast<long long>(max_blocks) * kPage))
    return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  if (!scores || !seq_lens || !indices) return cudaErrorInvalidValue;
  TopkParams p{scores, scores_stride, seq_lens, indices, counts, B, s_q, k, max_tokens,
               causal ? 1 : 0, block_table, rows, max_blocks, num_blocks};
  const unsigned grid = static_cast<unsigned>(B * s_q);
  if (max_tokens <= kTopkSmemKeys) {
    const int smem = max(max_tokens, 1) * 4;
    static gqa::DeviceOnce attr_once;
    const cudaError_t attr_err = attr_once.run([] {
      return cudaFuncSetAttribute(dsa_topk_kernel<true>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kTopkSmemKeys * 4);
    });
    if (attr_err != cudaSuccess) return attr_err;
    dsa_topk_kernel<true><<<grid, kTopkThreads, smem, stream>>>(p);
  } else {
    dsa_topk_kernel<false><<<grid, kTopkThreads, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace

extern "C" {

cudaError_t dsa_topk_launch(const float* scores, long long scores_stride, const int* seq_lens,
                            int B, int s_q, int k, int max_tokens, int causal, int* indices,
                            int* counts, cudaStream_t stream) {
  return topk_impl(scores, scores_stride, seq_lens, B, s_q, k, max_tokens, causal, indices,
                   counts, nullptr, 0, 0, nullptr, stream);
}

cudaError_t dsa_topk_rows_launch(const float* scores, long long scores_stride,
                                 const int* seq_lens, int B, int s_q, int k, int max_tokens,
                                 int causal, const int* block_table, int max_blocks,
                                 int num_blocks, int* indices, int* counts, int* rows,
                                 cudaStream_t stream) {
  if (!rows) return cudaErrorInvalidValue;
  return topk_impl(scores, scores_stride, seq_lens, B, s_q, k, max_tokens, causal, indices,
                   counts, block_table, max_blocks, num_blocks, rows, stream);
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
