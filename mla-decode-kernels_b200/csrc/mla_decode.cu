// MLA absorbed-path paged decode on sm_100a (the reference's roadmap kernel
// K2: latent cache [num_blocks, 64, 576], README.md "Roadmap"; no reference
// code exists, kernels/mla_decode/ is empty).  Operator, as FlashMLA's
// flash_mla_with_kvcache computes it: for request b, query position i, head h,
//   out[b, i, h, :] = softmax_t(scale * q[b, i, h, :] . C_t) @ C_t[0:512]
// over the request's cached latent rows C_t (576 = 512 latent + 64 rope
// dims; one latent "kv head"), t < S_b, or t < S_b - s_q + 1 + i when causal;
// lse[b, h, i] = ln sum_t exp(score_t).
//
// Two kernels, both 2-CTA clusters: CTA r of a pair multiplies latent dims
// 256 r .. 256 r + 255 and half of the rope dims (the pair exchanges partial
// scores over distributed shared memory) and owns value dims 256 r ..
// 256 r + 255 of the output.
//   mla_decode_kernel<NH>    groups of NH <= 64 query rows: tokens on the MMA
//                            M dimension, query rows on N (no padding waste at
//                            small head counts), S^T / O^T in tensor memory.
//   mla_decode_rows_kernel   groups of 128 query rows: rows on M, Q and P as
//                            tensor-memory A operands, one softmax thread per
//                            row, sender warps for the exchange; also the
//                            sparse mode (rows of selected tokens).  Dense:
//                            persistent, one pair per two SMs, each pair an
//                            equal share of the batch's 64-token tiles (a
//                            unit cut between pairs leaves one partial state
//                            per pair, merged by mla_rows_combine_kernel).
//                            Sparse: also one whole unit per pair (no
//                            merge) when a measured cost fit predicts that
//                            faster (near-uniform selections, full waves).
// Online softmax in the log2 domain with a lazily raised reference max: P is
// computed against the current reference m_ref and O / l are only rescaled
// when a tile's score exceeds m_ref by more than 2^8 (the bound on exp2
// growth kept in fp32 / bf16 range), which after the first tiles is rare.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "device_once.h"
#include "gqa_decode.h"
#include "gqa_ptx.cuh"
#include "mla_decode.h"
#include "umma_ptx.cuh"

namespace gqa {
namespace mla {

constexpr int kD = 576;             // latent + rope dims per cached token
constexpr int kDV = 512;            // value dims (the latent part)
constexpr int kPage = 64;           // tokens per cache page (FlashMLA's block size)
constexpr int kColBytes = kPage * 128;            // one 64-dim box of a page: 8 KB
constexpr int kThreads = 320;       // producer, MMA, 8 softmax warps (2 per TMEM quadrant)
constexpr float kRescaleLog2 = 8.f; // lazy rescale threshold (log2 units)

__device__ int g_mla_status;

struct Params {
  CUtensorMap tm_q;   // [rows_total, 576] bf16, box {64, NH}, 128B swizzle
  CUtensorMap tm_kv;  // [num_blocks * 64, 576] bf16, box {64, 64}, 128B swizzle
  CUtensorMap tm_q_rope;   // the same rows, box {32, NH}, 64B swizzle (128-row groups)
  CUtensorMap tm_kv_rope;  // the same rows, box {32, 64}, 64B swizzle (128-row groups)
  const int* sparse_idx;     // sparse: [B * s_q, topk] token positions per query position
                             // (or, with sparse_rows, physical cache rows)
  int sparse_rows;           // sparse: sparse_idx holds block id * 64 + slot, no block_table
  const __nv_bfloat16* kv;   // sparse: the cache (rows copied by the producer warp)
  const __nv_bfloat16* q;    // 128-row groups: q rows (loaded straight into tensor memory)
  int* hdr;                  // 128-row groups: [2] total tiles T and working pairs Pe (0: one unit per pair)
  int per_unit;              // 128-row groups: pair c takes unit c whole (no balancing, no partials)
  int4* unit_info;           // 128-row groups: [units] first slot, first pair, pairs
  float* slot_m;             // 128-row groups: [2 P][128] partial max (log2 domain)
  float* slot_l;             // 128-row groups: [2 P][128] partial sums
  float* slot_acc;           // 128-row groups: [2 P][128][512] unnormalised partial O
  int topk;                  // sparse: index row length
  const int* block_table;
  const int* seq_lens;
  __nv_bfloat16* out;  // [B, s_q, h_q, 512] (num_splits == 1)
  float* lse;          // [B, h_q, s_q]      (num_splits == 1)
  float* part_acc;     // [B * rows, ns, 512] unnormalised (num_splits > 1)
  float* part_m;       // [B * rows, ns] log2-domain reference max
  float* part_l;       // [B * rows, ns]
  int B, s_q, h_q, rows, n_hg, max_blocks, num_blocks, num_splits, causal;
  float scale_log2;    // softmax_scale * log2(e)
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

// Compile-time geometry of the 2-CTA heads-on-N kernel for NH <= 64 query
// rows per pair.
template <int NH>
struct Pair {
  static constexpr int kHalf = NH / 4;               // S^T values per softmax thread
  static constexpr int kWarpCols = NH / 2;           // query rows per softmax warp
  static constexpr int kChunk = kWarpCols < 16 ? kWarpCols : 16;  // TMEM columns per load
  static constexpr int kCols = 5;                    // 64-dim boxes a CTA loads per row
  static constexpr int kStageBytes = kCols * kColBytes;  // 40 KB per page
  static constexpr int kStages = NH == 64 ? 3 : 4;
  static constexpr int kNP = 2;                      // P^T buffers
  static constexpr int kAtomN = NH < 64 ? NH : 64;   // heads per P^T swizzle atom
  static constexpr int kRowB = 2 * kAtomN;           // P^T row bytes inside an atom
  static constexpr int kAtoms = NH / kAtomN;
  static constexpr int kAtomBytes = kPage * kRowB;
  static constexpr int kPBytes = kAtoms * kAtomBytes;
  static constexpr uint32_t kPLayout =
      kAtomN == 64 ? kSwizzle128 : (kAtomN == 32 ? kSwizzle64 : kSwizzle32);
  static constexpr uint32_t kPMask = kAtomN == 64 ? 7u : (kAtomN == 32 ? 3u : 1u);
  static constexpr int kXBytes = kPage * NH * 4;     // partial S^T exchanged per tile
  static constexpr int kQBytes = kCols * NH * 128;
  static constexpr int kQ = 0;
  static constexpr int kRing = kQ + kQBytes;
  static constexpr int kP = kRing + kStages * kStageBytes;
  static constexpr int kX = kP + kNP * kPBytes;
  static constexpr int kSmall = kX + kXBytes;
  static constexpr int kSmallBytes = 4096;
  static constexpr int kSmem = kSmall + kSmallBytes + 1024;  // + alignment slack
  static constexpr uint32_t kTmemCols = 4 * NH;      // O^T 2 x NH, S^T 2 x NH
  static_assert(kSmem <= 232448, "shared memory");
};

// One CTA pair (a 2-CTA cluster) = (request, NH <= 64 query rows, page
// range).  CTA r loads, per 64-token page, latent columns 4r..4r+3 and the
// rope column (five 64-dim boxes, 40 KB): it computes the partial
//   S^T_r[64 tok, NH] over its 256 latent dims + half of the 64 rope dims
// (18 MMAs of M = 64, N = NH), exchanges S^T_r with the peer through
// st.async into the peer's shared memory, and from the full S^T = S^T_0 +
// S^T_1 (identical in both CTAs) the softmax, P^T and
//   O^T_r[256 dv, NH] += C[:, 256 r .. 256 r + 255]^T . P^T
// (8 MMAs of M = 128).  26 MMAs per page per CTA instead of 52.
template <int NH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    mla_decode_kernel(const __grid_constant__ Params p) {
  using G = Pair<NH>;
  constexpr int kStages_ = G::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sQ = s_base + G::kQ, sRing = s_base + G::kRing, sP = s_base + G::kP,
                 sX = s_base + G::kX;
  unsigned char* small = smem + G::kSmall;
  const uint32_t bars = s_base + G::kSmall;
  const uint32_t bar_q = bars, bar_full = bars + 8, bar_empty = bars + 40, bar_sfull = bars + 72,
                 bar_sfree = bars + 88, bar_pfull = bars + 104, bar_pv = bars + 120,
                 bar_xfull = bars + 136, bar_xfree = bars + 144, bar_fin = bars + 152;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(small + 160);
  int* vote = reinterpret_cast<int*>(small + 176);                // [2][8]
  float* red = reinterpret_cast<float*>(small + 256);             // [4][128]
  float* mref = reinterpret_cast<float*>(small + 2304);           // [128]
  float* alpha_s = reinterpret_cast<float*>(small + 2816);        // [128]
  int* vis_s = reinterpret_cast<int*>(small + 3328);              // [128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank(), peer = rank ^ 1u;
  const int unit = blockIdx.x >> 1;
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
  constexpr uint32_t o_col = 0, s_col0 = 2 * NH;  // TMEM columns: O^T blocks, S^T buffers

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_sfull + 8 * s, 1);
      mbar_init(bar_sfree + 8 * s, 8);  // one arrival per softmax warp
      mbar_init(bar_pfull + 8 * s, 8);
      mbar_init(bar_pv + 8 * s, 1);
    }
    mbar_init(bar_xfull, 1);  // armed with the byte count by this CTA, bytes from the peer
    mbar_init(bar_xfree, 8);  // the peer's eight softmax warps have read our partial
    mbar_init(bar_fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), G::kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x < 128) {
    mref[threadIdx.x] = -INFINITY;
    // rows past the last query row (padding of the final group) see nothing
    const int row = row0 + threadIdx.x;
    vis_s[threadIdx.x] = threadIdx.x < NH && row < p.rows ? visible(p, S, row) : 0;
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote access
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // dims of the five boxes this CTA loads: latent columns 4r..4r+3, rope
  auto col_of = [&](int c) { return c < 4 ? 4 * static_cast<int>(rank) + c : 8; };

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0 && ntiles > 0) {
      tma_prefetch_desc(&p.tm_kv);
      mbar_arrive_expect_tx(bar_q, static_cast<uint32_t>(G::kQBytes));
      for (int c = 0; c < G::kCols; ++c)
        tma_load_2d(sQ + c * NH * 128, &p.tm_q, 64 * col_of(c), b * p.rows + row0, bar_q);
      const int* bt = p.block_table + static_cast<size_t>(b) * p.max_blocks;
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages_;
        if (t >= kStages_ && !mbar_wait(bar_empty + 8 * s, ((t - kStages_) / kStages_) & 1)) {
          raise(kStatusWaitTimeout);
          break;
        }
        int page = __ldg(bt + pg0 + t);
        if (page < 0 || page >= p.num_blocks) {
          raise(kStatusBadPage);
          page = 0;
        }
        mbar_arrive_expect_tx(bar_full + 8 * s, G::kStageBytes);
        for (int c = 0; c < G::kCols; ++c)
          tma_load_2d(sRing + s * G::kStageBytes + c * kColBytes, &p.tm_kv, 64 * col_of(c),
                      page * kPage, bar_full + 8 * s);
        issued = t + 1;
      }
      // every issued copy has landed before the CTA may exit
      if (!mbar_wait(bar_q, 0)) raise(kStatusWaitTimeout);
      for (int t = max(0, issued - kStages_); t < issued; ++t)
        if (!mbar_wait(bar_full + 8 * (t % kStages_), (t / kStages_) & 1))
          raise(kStatusWaitTimeout);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    // Polls (non-blocking) for the next ready step so that PV of tile t,
    // which frees t's stage for the next load, never waits behind page t+1.
    constexpr uint32_t idesc_qk = umma_idesc_bf16(64, NH, false, false);
    constexpr uint32_t idesc_pv = umma_idesc_bf16(128, NH, true, true);
    bool ok = true;
    if (ntiles > 0) ok = wait_warp(bar_q, 0);
    int qk = 0, pv = 0;
    unsigned long long idle_since = global_timer_ns();
    while (ok && pv < ntiles) {
      int action = 0;  // 1 = PV(pv), 2 = QK(qk)
      if (lane == 0) {
        if (pv < qk && mbar_test_wait(bar_pfull + 8 * (pv & 1), (pv >> 1) & 1)) {
          action = 1;
        } else if (qk < ntiles && qk <= pv + 1 &&
                   mbar_test_wait(bar_full + 8 * (qk % kStages_), (qk / kStages_) & 1) &&
                   (qk < 2 || mbar_test_wait(bar_sfree + 8 * (qk & 1), ((qk - 2) >> 1) & 1))) {
          action = 2;
        }
      }
      action = __shfl_sync(0xffffffffu, action, 0);
      if (action == 0) {
        // back off: this warp shares an issue slot with a softmax warp
        __nanosleep(64);
        if (global_timer_ns() - idle_since > kWaitLimitNs) ok = false;
        continue;
      }
      idle_since = global_timer_ns();
      tc_fence_after();
      if (action == 2) {
        const int s = qk % kStages_, buf = qk & 1;
        const uint32_t kv = sRing + s * G::kStageBytes;
        // Zero the cache rows past the request's end in its last page (they
        // may hold anything, NaN included): 0 * NaN would poison O^T.
        const int nv = min(kPage, S - (pg0 + qk) * kPage);
        if (nv < kPage) {
          const int zrows = kPage - nv;
          for (int i = lane; i < G::kCols * zrows * 8; i += 32) {
            const int c = i / (zrows * 8), r = nv + (i / 8) % zrows, k = i % 8;
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(
                             kv + c * kColBytes + r * 128 + k * 16),
                         "r"(0u)
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        if (lane == 0) {
          // latent columns: all four k-steps; rope column: k-steps 2r, 2r+1.
          // Unrolled, every descriptor a constant offset (16-byte units) from
          // one base: rebuilding descriptors in a loop roughly doubles the
          // issue cost of each MMA.
          const uint64_t a0 = umma_smem_desc(kv, 16, 1024, kSwizzle128);
          const uint64_t b0 = umma_smem_desc(sQ, 16, 1024, kSwizzle128);
          const uint64_t rope = static_cast<uint64_t>(4 * static_cast<int>(rank));  // 64 bytes
          #pragma unroll
          for (int i = 0; i < 18; ++i) {
            const int c = i < 16 ? i >> 2 : 4;
            const int kk = i < 16 ? i & 3 : i - 16;
            const uint64_t a = a0 + static_cast<uint64_t>((c * kColBytes + kk * 32) >> 4) +
                               (i < 16 ? 0ull : rope);
            const uint64_t bq = b0 + static_cast<uint64_t>((c * NH * 128 + kk * 32) >> 4) +
                                (i < 16 ? 0ull : rope);
            umma_bf16_ss(tmem + s_col0 + buf * NH, a, bq, idesc_qk, i != 0);
          }
          umma_commit(bar_sfull + 8 * buf);
        }
        __syncwarp();
        ++qk;
      } else {
        if (lane == 0) {
          const uint32_t kv = sRing + (pv % kStages_) * G::kStageBytes;
          const uint32_t pb = sP + (pv % G::kNP) * G::kPBytes;
          const uint64_t a0 = umma_smem_desc(kv, kColBytes, 1024, kSwizzle128);
          const uint64_t p0 = umma_smem_desc(pb, G::kAtomBytes, 8 * G::kRowB, G::kPLayout);
          #pragma unroll
          for (int j = 0; j < 2; ++j) {
            #pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16_ss(tmem + o_col + j * NH,
                           a0 + static_cast<uint64_t>((2 * j * kColBytes + kk * 16 * 128) >> 4),
                           p0 + static_cast<uint64_t>((kk * 16 * G::kRowB) >> 4), idesc_pv,
                           (pv | kk) != 0);
          }
          umma_commit(bar_pv + 8 * (pv & 1));
          umma_commit(bar_empty + 8 * (pv % kStages_));
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
    // --------------------------- softmax warps 2..9 ----------------------------
    // Warp w reads TMEM lane quadrant w % 4 (tokens 16 q .. 16 q + 15 in the
    // M = 64 layout) and query rows [cg NH/2, (cg + 1) NH/2), cg = (w - 2) / 4;
    // lanes 0-15 / 16-31 take the first / second half of those rows.
    // Every softmax warp runs the same sequence of named barriers whatever
    // happens (a failed wait only clears `ok`), so they can never deadlock.
    const int tq = warp & 3;              // TMEM lane quadrant
    const int cg = (warp - 2) >> 2;       // column group
    const int wi = warp - 2;              // 0..7
    const int t0 = lane & 15, half = lane >> 4;
    const int tok_in_tile = 16 * tq + t0;
    const int hw = cg * G::kWarpCols;     // first query row of this warp
    const int h0 = hw + half * G::kHalf;  // first query row of this thread
    const uint32_t lane_base = static_cast<uint32_t>(32 * tq) << 16;
    const int sidx = threadIdx.x - 64;    // 0..255
    const uint32_t peer_x = mapa_shared(sX, peer);
    const uint32_t peer_xfull = mapa_shared(bar_xfull, peer);
    const uint32_t peer_xfree = mapa_shared(bar_xfree, peer);
    float lpart[G::kHalf];
    #pragma unroll
    for (int k = 0; k < G::kHalf; ++k) lpart[k] = 0.f;
    int vis_min = 0x7fffffff;  // fewest visible tokens over this thread's rows
    #pragma unroll 1
    for (int k = 0; k < G::kHalf; ++k) vis_min = min(vis_min, vis_s[h0 + k]);
    bool ok = true;
    auto wait_pv = [&](int k) {  // completion of PV(k): phase k >> 1 of bar_pv[k & 1]
      if (k >= 0 && ok && !wait_warp(bar_pv + 8 * (k & 1), (k >> 1) & 1)) ok = false;
    };
    auto wait_cluster = [&](uint32_t bar, uint32_t parity) {
      if (!ok) return;
      bool done = mbar_try_wait_cluster(bar, parity);
      if (!done) {
        const unsigned long long t_start = global_timer_ns();
        while (!(done = mbar_try_wait_cluster(bar, parity)))
          if (global_timer_ns() - t_start > kWaitLimitNs) break;
      }
      if (!__all_sync(0xffffffffu, done)) ok = false;
    };
    for (int t = 0; t < ntiles; ++t) {
      const int buf = t & 1;
      if (sidx == 0) mbar_arrive_expect_tx(bar_xfull, G::kXBytes);  // the peer's partial
      if (ok && !wait_warp(bar_sfull + 8 * buf, (t >> 1) & 1)) ok = false;
      tc_fence_after();
      float x[G::kHalf];
      {
        const uint32_t a = tmem + lane_base + s_col0 + buf * NH + hw;
        if constexpr (G::kHalf == 4) {
          uint32_t r[4];
          tmem_ld_16x32bx2_4<4>(a, r);
          tmem_wait_ld();
          #pragma unroll
          for (int k = 0; k < 4; ++k) x[k] = __uint_as_float(r[k]);
        } else if constexpr (G::kHalf == 8) {
          uint32_t r[8];
          tmem_ld_16x32bx2_8<8>(a, r);
          tmem_wait_ld();
          #pragma unroll
          for (int k = 0; k < 8; ++k) x[k] = __uint_as_float(r[k]);
        } else {
          uint32_t r[G::kHalf / 16][16];
          #pragma unroll
          for (int c16 = 0; c16 < G::kHalf / 16; ++c16)
            tmem_ld_16x32bx2_16<G::kHalf>(a + 16 * c16, r[c16]);
          tmem_wait_ld();
          #pragma unroll
          for (int c16 = 0; c16 < G::kHalf / 16; ++c16) {
            #pragma unroll
            for (int k = 0; k < 16; ++k) x[16 * c16 + k] = __uint_as_float(r[c16][k]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree + 8 * buf);
      // exchange: our partial into the peer's buffer (once it has read the
      // previous one), the peer's partial out of ours
      if (t >= 1) wait_cluster(bar_xfree, (t - 1) & 1);
      #pragma unroll
      for (int k4 = 0; k4 < G::kHalf / 4; ++k4)
        st_async_v4(peer_x + (k4 * 256 + sidx) * 16, __float_as_uint(x[4 * k4]),
                    __float_as_uint(x[4 * k4 + 1]), __float_as_uint(x[4 * k4 + 2]),
                    __float_as_uint(x[4 * k4 + 3]), peer_xfull);
      wait_cluster(bar_xfull, t & 1);
      uint32_t dep = 0;
      #pragma unroll
      for (int k4 = 0; k4 < G::kHalf / 4; ++k4) {
        float4 o;
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(o.x), "=f"(o.y), "=f"(o.z), "=f"(o.w)
                     : "r"(sX + (k4 * 256 + sidx) * 16)
                     : "memory");
        // S0 + S1 in both CTAs (addition commutes: identical bits)
        x[4 * k4] += o.x;
        x[4 * k4 + 1] += o.y;
        x[4 * k4 + 2] += o.z;
        x[4 * k4 + 3] += o.w;
        dep ^= __float_as_uint(o.x) ^ __float_as_uint(o.w);
      }
      // every lane's reads of the peer's partial are complete once all lanes
      // have produced dep; then the peer may overwrite the buffer
      dep = __reduce_xor_sync(0xffffffffu, dep);
      if (lane == 0) mbar_arrive_remote_relaxed(peer_xfree, dep);
      const int tok = (pg0 + t) * kPage + tok_in_tile;
      bool need = false;
      if (tok < vis_min) {  // every row of this thread sees the token
        #pragma unroll
        for (int k = 0; k < G::kHalf; ++k) {
          x[k] *= p.scale_log2;
          need |= x[k] > mref[h0 + k] + kRescaleLog2;
        }
      } else {
        #pragma unroll
        for (int k = 0; k < G::kHalf; ++k) {
          const bool valid = tok < vis_s[h0 + k];
          x[k] = valid ? x[k] * p.scale_log2 : -INFINITY;
          need |= x[k] > mref[h0 + k] + kRescaleLog2;
        }
      }
      need = __any_sync(0xffffffffu, need);
      if (lane == 0) vote[(t & 1) * 8 + wi] = need ? 1 : 0;
      named_bar_sync(1, 256);
      const int* v = vote + (t & 1) * 8;
      const bool rescale = (v[0] | v[1] | v[2] | v[3] | v[4] | v[5] | v[6] | v[7]) != 0;
      if (rescale) {
        // tile max per row over the 64 tokens (16 lanes of each half x 4 warps)
        #pragma unroll
        for (int k = 0; k < G::kHalf; ++k) {
          float m = x[k];
          #pragma unroll
          for (int off = 8; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
          if (t0 == 0) red[tq * 128 + h0 + k] = m;
        }
        named_bar_sync(1, 256);
        if (sidx < NH) {
          const int h = sidx;
          const float tmax =
              fmaxf(fmaxf(red[h], red[128 + h]), fmaxf(red[256 + h], red[384 + h]));
          const float mo = mref[h];
          const float mn = fmaxf(mo, tmax);
          alpha_s[h] = mo == -INFINITY ? 0.f : exp2f(mo - mn);
          mref[h] = mn;
        }
        named_bar_sync(1, 256);
        #pragma unroll
        for (int k = 0; k < G::kHalf; ++k) lpart[k] *= alpha_s[h0 + k];
        if (t >= 1) {
          // O^T[dv, h] *= alpha[h] on this warp's quadrant (dv rows 32 tq..),
          // once every earlier PV has accumulated into it
          wait_pv(t - 1);
          tc_fence_after();
          #pragma unroll 1
          for (int j = 0; j < 2; ++j) {
            #pragma unroll 1
            for (int c = 0; c < G::kWarpCols; c += G::kChunk) {
              const uint32_t a = tmem + lane_base + o_col + j * NH + hw + c;
              if constexpr (G::kChunk == 16) {
                uint32_t r[16];
                tmem_ld16(a, r);
                tmem_wait_ld();
                #pragma unroll
                for (int k = 0; k < 16; ++k)
                  r[k] = __float_as_uint(__uint_as_float(r[k]) * alpha_s[hw + c + k]);
                tmem_st16(a, r);
              } else {
                uint32_t r[8];
                tmem_ld8(a, r);
                tmem_wait_ld();
                #pragma unroll
                for (int k = 0; k < 8; ++k)
                  r[k] = __float_as_uint(__uint_as_float(r[k]) * alpha_s[hw + c + k]);
                tmem_st8(a, r);
              }
            }
          }
          tmem_wait_st();
        }
      }
      // P^T of this token for this thread's rows: p = 2^(x - m_ref), masked
      // entries 0; the buffer is free once the PV that last read it is done
      wait_pv(t - G::kNP);
      const uint32_t pb = sP + (t % G::kNP) * G::kPBytes;
      #pragma unroll
      for (int c4 = 0; c4 < G::kHalf / 4; ++c4) {
        float pv[4], mr[4];
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(mr[0]), "=f"(mr[1]), "=f"(mr[2]), "=f"(mr[3])
                     : "r"(smem_u32(mref + h0 + 4 * c4)));
        #pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int kk = 4 * c4 + k;
          // x = -inf (masked) gives 0; m_ref is finite once any score was
          // seen (the first visible tile always rescales)
          pv[k] = x[kk] == -INFINITY ? 0.f : fast_exp2(x[kk] - mr[k]);
          lpart[kk] += pv[k];
        }
        const int hcol = h0 + 4 * c4;  // first query row of these 4 values
        const uint32_t off = static_cast<uint32_t>((hcol / 64) * G::kAtomBytes +
                                                   tok_in_tile * G::kRowB + (hcol % 64) * 2);
        const uint32_t swz = off ^ (((off >> 7) & G::kPMask) << 4);
        asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(pb + swz),
                     "r"(pack2(pv[0], pv[1])), "r"(pack2(pv[2], pv[3]))
                     : "memory");
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_pfull + 8 * (t & 1));
    }
    // the peer has read our last partial before either CTA may exit
    if (ntiles >= 1) wait_cluster(bar_xfree, (ntiles - 1) & 1);
    // ------------------------------ epilogue ---------------------------------
    wait_pv(ntiles - 1);
    tc_fence_after();
    if (!ok) raise(kStatusWaitTimeout);
    // l[h] = sum over the 64 token rows of the per-thread partial sums
    named_bar_sync(1, 256);
    #pragma unroll
    for (int k = 0; k < G::kHalf; ++k) {
      float l = lpart[k];
      #pragma unroll
      for (int off = 8; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (t0 == 0) red[tq * 128 + h0 + k] = l;
    }
    named_bar_sync(1, 256);
    const int L = 32 * tq + lane;  // dv row within each 128-row block of O^T
    const bool final_out = p.num_splits == 1;
    const int dv0 = 256 * static_cast<int>(rank);
    #pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      #pragma unroll 1
      for (int c = 0; c < G::kWarpCols; c += G::kChunk) {
        uint32_t r[G::kChunk];
        if (ntiles > 0) {
          if constexpr (G::kChunk == 16)
            tmem_ld16(tmem + lane_base + o_col + j * NH + hw + c, r);
          else
            tmem_ld8(tmem + lane_base + o_col + j * NH + hw + c, r);
          tmem_wait_ld();
        } else {
          #pragma unroll
          for (int k = 0; k < G::kChunk; ++k) r[k] = 0u;
        }
        #pragma unroll
        for (int k = 0; k < G::kChunk; ++k) {
          const int h = hw + c + k;
          if (row0 + h >= p.rows) continue;  // padding rows of the last group
          const float l = red[h] + red[128 + h] + red[256 + h] + red[384 + h];
          const float o = __uint_as_float(r[k]);
          const size_t grow = static_cast<size_t>(b) * p.rows + row0 + h;
          const int d = dv0 + 128 * j + L;
          if (final_out)
            p.out[grow * kDV + d] = __float2bfloat16(l > 0.f ? o / l : 0.f);
          else
            p.part_acc[(grow * p.num_splits + sp) * kDV + d] = l > 0.f ? o : 0.f;
        }
      }
    }
    if (rank == 0 && sidx < NH && row0 + sidx < p.rows) {
      const int h = sidx;
      const int row = row0 + h;
      const float l = red[h] + red[128 + h] + red[256 + h] + red[384 + h];
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
    tmem_dealloc(tmem, G::kTmemCols);
  }
  cluster_sync();  // no CTA leaves while its peer may still address its shared memory
}

// ---- 128-row groups: query rows on the MMA M dimension ------------------------
//
// For groups of 128 query rows the roles of the operands flip: the rows are
// the M = 128 dimension, so every thread of the four softmax warps owns one
// row of S, P and O (row max, exp2 and the row sum stay in registers), and
// this CTA's half of Q (256 latent + 32 rope dims) lives in tensor memory as
// the A operand of the QK MMAs, as does P for the PV MMAs.  A page stage
// holds only what this CTA multiplies: its four latent boxes and its 32-dim
// half of the rope box (36 KB): a four-stage ring beside two exchange
// buffers (the partial-S exchange over distributed shared memory, ~16 bytes
// per SM cycle each way, is the kernel's throughput limit; double buffering
// overlaps it with a tile of softmax work).
//   S_r[128 rows, 64 tok]  = Q_r[128, 288] . C_r[64 tok, 288]^T   (18 MMAs, N = 64)
//   S = S_0 + S_1 (the partials exchanged over distributed shared memory)
//   O_r[128 rows, 256 dv] += P[128, 64 tok] . C[64 tok, 256 r .. 256 r + 255]
//                                                                (4 MMAs, N = 256)
// Tensor memory: O_r columns 0-255, Q_r 256-399, P 416-447, S 448-511.
// Q_r arrives by TMA in the last two ring stages, is copied into tensor
// memory by the softmax warps, and those stages then take pages.
struct Rows {
  static constexpr int kRopeBytes = kPage * 64;          // 32 rope dims x 64 tokens
  static constexpr int kStageBytes = 4 * kColBytes + kRopeBytes;  // 36 KB
  static constexpr int kStages = 4;
  static constexpr int kXBytes = 128 * kPage * 4;        // the peer's partial S of a tile
  static constexpr int kRing = 0;
  static constexpr int kX = kRing + kStages * kStageBytes;  // two tiles' partials
  static constexpr int kSmall = kX + 2 * kXBytes;
  // small region: barriers and scan scratch [0, 256), row max / sum exchange
  // [3][2][128] floats, the sparse row queue
  static constexpr int kRed = 256, kRowQ = kRed + 3 * 2 * 128 * 4;
  static constexpr int kRowAhead = 4;                  // tiles resolved and prefetched ahead
  static constexpr int kSmem = kSmall + kRowQ + (kRowAhead + 1) * kPage * 4 + 1024;
  static constexpr int kThreads = 448;  // producer, MMA, eight softmax, four sender warps
  static constexpr int kQStage = kStages - 2;            // first unit's Q_r staged in stages 2-3
  static constexpr int kQLatBytes = 128 * 128;           // one 64-dim box of 128 rows
  static constexpr int kQBytes = 4 * kQLatBytes + 128 * 64;  // = 2 stages
  static constexpr uint32_t kOCol = 0, kQCol = 256, kPCol = 416, kSCol = 448;
  static_assert(kQBytes == 2 * kStageBytes, "Q staging spans the last two stages");
  static_assert(kSmem <= 232448, "shared memory");
};

// Tiles (64-token pages, or 64 selected tokens) of work unit u = (request
// b = u / n_hg, 128-row group hg = u % n_hg).
__device__ __forceinline__ const int* unit_len_ptr(const Params& p, int u) {
  const int b = u / p.n_hg, hg = u % p.n_hg;
  return p.sparse_idx ? p.seq_lens + b * p.s_q + (hg * 128) / p.h_q : p.seq_lens + b;
}

__device__ __forceinline__ int unit_clamp(const Params& p, int len) {
  return max(0, min(len, p.sparse_idx ? p.topk : p.max_blocks * kPage));
}

__device__ __forceinline__ int unit_tokens(const Params& p, int u) {
  return unit_clamp(p, *unit_len_ptr(p, u));
}

// A walk over the pair's range of the batch's tiles, unit by unit (every
// role of the CTA walks the same sequence).
struct TileWalk {
  int u, i, n, S, start;  // unit, tile within it, its tiles, its tokens, its first tile
  __device__ void init(const Params& p, int u0, int start0, int g0) {
    u = u0;
    start = start0;
    S = unit_tokens(p, u);
    n = (S + kPage - 1) / kPage;
    i = g0 - start0;
  }
  // to the next tile; past a unit's last tile, the next unit with tiles
  __device__ void next(const Params& p) {
    if (++i < n) return;
    const int U = p.B * p.n_hg;
    start += n;
    i = 0;
    n = 0;
    while (n == 0 && u + 1 < U) {
      ++u;
      S = unit_tokens(p, u);
      n = (S + kPage - 1) / kPage;
    }
  }
};

// Pair of tile g under the proportional split [c T / P, (c + 1) T / P).
__device__ __forceinline__ int pair_of(long long g, long long T, int P) {
  return static_cast<int>(((g + 1) * P - 1) / T);
}

__device__ __forceinline__ int pair_start(int c, long long T, int P) {
  return static_cast<int>(static_cast<long long>(c) * T / P);
}

// Persistent: P = gridDim.x / 2 CTA pairs, pair c takes tiles [c T / Pe,
// (c + 1) T / Pe) of the batch's T tiles (unit by unit, in order; Pe =
// min(P, T) working pairs), so every pair does the same work whatever the
// lengths; a unit split between pairs leaves one partial state per pair,
// merged by mla_rows_combine_kernel.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Rows::kThreads, 1)
    mla_decode_rows_kernel(const __grid_constant__ Params p) {
  using G = Rows;
  constexpr int kSt = G::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sRing = s_base + G::kRing, sX = s_base + G::kX;
  const uint32_t bars = s_base + G::kSmall;
  const uint32_t bar_full = bars, bar_empty = bars + 32, bar_sfull = bars + 64,
                 bar_sfree = bars + 72, bar_pfull = bars + 80, bar_pv = bars + 88,
                 bar_xfull = bars + 96, bar_xfree = bars + 112, bar_qready = bars + 128,
                 bar_fin = bars + 136, bar_q = bars + 144, bar_qfree = bars + 152;
  const uint32_t sQ = sRing + G::kQStage * G::kStageBytes;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kSmall + 160);
  int* wk = reinterpret_cast<int*>(smem + G::kSmall + 168);  // [0] u0 [1] start0
  int* wsum = reinterpret_cast<int*>(smem + G::kSmall + 192);  // [16] warp sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank(), peer = rank ^ 1u;
  const int P = static_cast<int>(gridDim.x >> 1), c = static_cast<int>(blockIdx.x >> 1);
  const int U = p.B * p.n_hg;
  constexpr int kW = G::kThreads / 32;

  // ---- the pair's tile range: T over the batch, then the unit holding g0 ----
  // (block-wide scans over the units in chunks of the block size)
  auto block_excl_scan = [&](int v, int& total) {
    int x = v;
    #pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    int before = 0, all = 0;
    #pragma unroll
    for (int w = 0; w < kW; ++w) {
      const int s = wsum[w];
      before += w < warp ? s : 0;
      all += s;
    }
    __syncthreads();
    total = all;
    return before + x - v;
  };
  long long T = 0;
  for (int base = 0; base < (p.per_unit ? 0 : U); base += blockDim.x) {
    const int u = base + threadIdx.x;
    const int n = u < U ? (unit_tokens(p, u) + kPage - 1) / kPage : 0;
    int tot = 0;
    block_excl_scan(n, tot);
    T += tot;
  }
  // pairs beyond the tile count stay idle, so every working pair owns at
  // least one tile and the pairs of a unit are consecutive working pairs
  const int Pe = static_cast<int>(T < P ? T : P);
  if (blockIdx.x == 0 && threadIdx.x == 0) {  // for the combine pass
    p.hdr[0] = static_cast<int>(T);
    p.hdr[1] = p.per_unit ? 0 : Pe;
  }
  // one unit per pair: unit c whole, its tiles counted from 0
  const int n_own = p.per_unit && c < U ? (unit_tokens(p, c) + kPage - 1) / kPage : 0;
  const int g0 = p.per_unit ? 0 : (c < Pe ? pair_start(c, T, Pe) : 0);
  const int g1 = p.per_unit ? n_own : (c < Pe ? pair_start(c + 1, T, Pe) : 0);
  const int ntiles = g1 - g0;
  if (threadIdx.x == 0) {
    wk[0] = p.per_unit ? c : 0;
    wk[1] = 0;
  }
  __syncthreads();
  if (ntiles > 0 && !p.per_unit) {
    int carry = 0;
    for (int base = 0; base < U; base += blockDim.x) {
      const int u = base + threadIdx.x;
      const int n = u < U ? (unit_tokens(p, u) + kPage - 1) / kPage : 0;
      int tot = 0;
      const int excl = carry + block_excl_scan(n, tot);
      if (n > 0 && excl <= g0 && g0 < excl + n) {
        wk[0] = u;
        wk[1] = excl;
      }
      carry += tot;
      if (carry > g0) break;  // uniform: every thread has the same carry
    }
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSt; ++s) {
      // sparse: one cp.async completion arrival per producer lane
      mbar_init(bar_full + 8 * s, p.sparse_idx ? 32 : 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_sfull, 1);
    mbar_init(bar_sfree, 12);  // one arrival per softmax and sender warp
    mbar_init(bar_pfull, 8);
    mbar_init(bar_pv, 1);
    for (int j = 0; j < 2; ++j) {
      mbar_init(bar_xfull + 8 * j, 1);  // armed with the byte count here, bytes from the peer
      mbar_init(bar_xfree + 8 * j, 8);  // the peer's eight softmax warps have read our partial
    }
    mbar_init(bar_qready, 4);  // a unit's Q_r is in tensor memory (one arrival per sender warp)
    mbar_init(bar_q, 1);       // the first unit's Q_r has landed in the ring
    mbar_init(bar_qfree, 4);   // ... and has been copied out of it
    mbar_init(bar_fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote access
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int rope_x = 512 + 32 * static_cast<int>(rank);  // this CTA's rope dims
  const int u0 = wk[0], start0 = wk[1];
  // the first unit's Q_r by TMA into ring stages kQStage.. (they take pages
  // once the softmax warps have copied it into tensor memory)
  auto stage_q = [&]() {
    const int b = u0 / p.n_hg, row0 = (u0 % p.n_hg) * 128;
    mbar_arrive_expect_tx(bar_q, G::kQBytes);
    for (int cc = 0; cc < 4; ++cc)
      tma_load_2d(sQ + cc * G::kQLatBytes, &p.tm_q, 64 * (4 * static_cast<int>(rank) + cc),
                  b * p.rows + row0, bar_q);
    tma_load_2d(sQ + 4 * G::kQLatBytes, &p.tm_q_rope, rope_x, b * p.rows + row0, bar_q);
  };

  if (warp == 0 && p.sparse_idx) {
    // -------------------- producer warp, gathered cache rows --------------------
    // Tile t holds selected tokens i * 64 .. + 63 of its unit.  Lane L
    // resolves slots 2L and 2L + 1 to cache rows (a shared queue kRowAhead
    // tiles ahead of use, so the token -> page -> row lookups overlap the
    // ring) and copies this CTA's half of both rows (four 128-byte latent box
    // rows, one 64-byte rope row) with 16-byte cp.async into the swizzled
    // stage layout TMA would have written.  TMA gather copies (four rows each)
    // run into the per-SM TMA operation rate at 80 copies per tile; these do
    // not.
    if (ntiles > 0) {
      int* rowq = reinterpret_cast<int*>(smem + G::kSmall + G::kRowQ);
      if (lane == 0) stage_q();
      TileWalk wa;  // kRowAhead tiles ahead
      wa.init(p, u0, start0, g0);
      auto resolve = [&](int t) {
        if (t >= ntiles) return;
        const int b = wa.u / p.n_hg, hg = wa.u % p.n_hg;
        const int qpos = (hg * 128) / p.h_q;
        const int* idx = p.sparse_idx + static_cast<size_t>(b * p.s_q + qpos) * p.topk;
        int* q_t = rowq + (t % (G::kRowAhead + 1)) * kPage;
        #pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int j = wa.i * kPage + 2 * lane + u;
          int row = -1;
          if (j < wa.S) {
            if (p.sparse_rows) {
              // rows resolved by the top-k kernel: one load, no lookup chain
              row = __ldg(idx + j);
              if (row < 0 || static_cast<long long>(row) >= static_cast<long long>(p.num_blocks) * kPage) {
                raise(kStatusBadPage);
                row = 0;
              }
            } else {
              const int* bt = p.block_table + static_cast<size_t>(b) * p.max_blocks;
              const int tok = __ldg(idx + j);
              int page = tok >= 0 && tok < p.max_blocks * kPage ? __ldg(bt + (tok >> 6)) : -1;
              if (page < 0 || page >= p.num_blocks) {
                raise(kStatusBadPage);
                page = 0;
              }
              row = page * kPage + (tok & (kPage - 1));
            }
            // this CTA's half of the row into L2 while the tile waits its turn
            const char* rp =
                reinterpret_cast<const char*>(p.kv) + static_cast<size_t>(row) * (kD * 2);
            #pragma unroll
            for (int l = 0; l < 4; ++l) prefetch_l2(rp + 512 * rank + 128 * l);
            prefetch_l2(rp + 2 * rope_x);
          }
          q_t[2 * lane + u] = row;
        }
        wa.next(p);
      };
      for (int t = 0; t < G::kRowAhead; ++t) resolve(t);
      const char* kvb = reinterpret_cast<const char*>(p.kv);
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kSt;
        resolve(t + G::kRowAhead);
        const int* q_t = rowq + (t % (G::kRowAhead + 1)) * kPage;
        bool ok = true;
        if (lane == 0) {
          if (t >= kSt)
            ok = mbar_wait(bar_empty + 8 * s, ((t - kSt) / kSt) & 1);
          else if (s >= G::kQStage)
            ok = mbar_wait(bar_qfree, 0);  // the first Q_r has left these stages
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) {
          if (lane == 0) raise(kStatusWaitTimeout);
          break;
        }
        __syncwarp();  // the queue entries other lanes wrote are visible
        // slots past the selection take the tile's first row (their scores are
        // masked, so P = 0 there).  Lane L holds rows 2L and 2L + 1; one warp
        // instruction then copies 512 contiguous bytes of one row (the CTA's
        // latent half: lane -> box lane / 8, 16-byte chunk lane % 8), four
        // 128-byte lines instead of one line per lane, with the row index
        // broadcast by shuffle; the 64-byte rope halves go eight rows per
        // instruction.
        const int first = q_t[0];
        const int ra = q_t[2 * lane] < 0 ? first : q_t[2 * lane];
        const int rb = q_t[2 * lane + 1] < 0 ? first : q_t[2 * lane + 1];
        const uint32_t st = sRing + s * G::kStageBytes;
        const uint32_t dl = st + (lane >> 3) * kColBytes;
        const int cl = lane & 7;
        const char* kvl = kvb + 512 * rank + 16 * lane;
        #pragma unroll
        for (int r = 0; r < kPage; ++r) {
          const int row = __shfl_sync(0xffffffffu, (r & 1) ? rb : ra, r >> 1);
          cp_async_16(dl + r * 128 + ((cl ^ (r & 7)) << 4),
                      kvl + static_cast<size_t>(row) * (kD * 2));
        }
        #pragma unroll
        for (int i = 0; i < kPage / 8; ++i) {
          const int r = 8 * i + (lane >> 2), k = lane & 3;
          const int xa = __shfl_sync(0xffffffffu, ra, r >> 1);
          const int xb = __shfl_sync(0xffffffffu, rb, r >> 1);
          const int row = (r & 1) ? xb : xa;
          cp_async_16(st + 4 * kColBytes + r * 64 + ((k ^ ((r >> 1) & 3)) << 4),
                      kvb + static_cast<size_t>(row) * (kD * 2) + 2 * rope_x + 16 * k);
        }
        cp_async_mbar_arrive(bar_full + 8 * s);  // one of the stage's 32 arrivals
        issued = t + 1;
      }
      // every issued copy has landed before the CTA may exit
      if (lane == 0) {
        if (!mbar_wait(bar_q, 0)) raise(kStatusWaitTimeout);
        for (int t = max(0, issued - kSt); t < issued; ++t)
          if (!mbar_wait(bar_full + 8 * (t % kSt), (t / kSt) & 1)) raise(kStatusWaitTimeout);
      }
    }
  } else if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0 && ntiles > 0) {
      tma_prefetch_desc(&p.tm_kv);
      stage_q();
      TileWalk w, wp;  // this tile, and the tile kSt ahead (L2 prefetch)
      w.init(p, u0, start0, g0);
      wp.init(p, u0, start0, g0);
      for (int k = 0; k < kSt && k + 1 < ntiles; ++k) wp.next(p);
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kSt;
        bool ok = true;
        if (t >= kSt)
          ok = mbar_wait(bar_empty + 8 * s, ((t - kSt) / kSt) & 1);
        else if (s >= G::kQStage)
          ok = mbar_wait(bar_qfree, 0);  // the first Q_r has left these stages
        if (!ok) {
          raise(kStatusWaitTimeout);
          break;
        }
        const int* bt = p.block_table + static_cast<size_t>(w.u / p.n_hg) * p.max_blocks;
        int page = __ldg(bt + w.i);
        if (page < 0 || page >= p.num_blocks) {
          raise(kStatusBadPage);
          page = 0;
        }
        const uint32_t st = sRing + s * G::kStageBytes;
        mbar_arrive_expect_tx(bar_full + 8 * s, G::kStageBytes);
        for (int cc = 0; cc < 4; ++cc)
          tma_load_2d(st + cc * kColBytes, &p.tm_kv, 64 * (4 * static_cast<int>(rank) + cc),
                      page * kPage, bar_full + 8 * s);
        tma_load_2d(st + 4 * kColBytes, &p.tm_kv_rope, rope_x, page * kPage, bar_full + 8 * s);
        issued = t + 1;
        // The page kSt tiles ahead into L2: a stage is held from its load
        // until its PV completes, so the ring alone would expose the full
        // DRAM latency once per kSt tiles.
        if (t + kSt < ntiles) {
          const int* btp = p.block_table + static_cast<size_t>(wp.u / p.n_hg) * p.max_blocks;
          const int pf = __ldg(btp + wp.i);
          if (pf >= 0 && pf < p.num_blocks) {
            for (int cc = 0; cc < 4; ++cc)
              tma_prefetch_2d(&p.tm_kv, 64 * (4 * static_cast<int>(rank) + cc), pf * kPage);
            tma_prefetch_2d(&p.tm_kv_rope, rope_x, pf * kPage);
          }
          if (t + kSt + 1 < ntiles) wp.next(p);
        }
        if (t + 1 < ntiles) w.next(p);
      }
      // every issued copy has landed before the CTA may exit
      if (!mbar_wait(bar_q, 0)) raise(kStatusWaitTimeout);
      for (int t = max(0, issued - kSt); t < issued; ++t)
        if (!mbar_wait(bar_full + 8 * (t % kSt), (t / kSt) & 1)) raise(kStatusWaitTimeout);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    constexpr uint32_t idesc_qk = umma_idesc_bf16(128, 64, false, false);
    constexpr uint32_t idesc_pv = umma_idesc_bf16(128, 256, false, true);
    bool ok = true;
    int qk = 0, pv = 0, qseg = 0;
    TileWalk wq, wv;  // the next QK's tile, the next PV's tile
    if (ntiles > 0) {
      wq.init(p, u0, start0, g0);
      wv.init(p, u0, start0, g0);
    }
    unsigned long long idle_since = global_timer_ns();
    while (ok && pv < ntiles) {
      int action = 0;  // 1 = PV(pv), 2 = QK(qk)
      if (lane == 0) {
        // the first QK of a unit waits for its Q_r in tensor memory
        const bool q_first = qk == 0 || wq.i == 0;
        if (pv < qk && mbar_test_wait(bar_pfull, pv & 1)) {
          action = 1;
        } else if (qk < ntiles && mbar_test_wait(bar_full + 8 * (qk % kSt), (qk / kSt) & 1) &&
                   (qk == 0 || mbar_test_wait(bar_sfree, (qk - 1) & 1)) &&
                   (!q_first || mbar_test_wait(bar_qready, qseg & 1))) {
          action = 2;
        }
      }
      action = __shfl_sync(0xffffffffu, action, 0);
      if (action == 0) {
        __nanosleep(64);
        if (global_timer_ns() - idle_since > kWaitLimitNs) ok = false;
        continue;
      }
      idle_since = global_timer_ns();
      tc_fence_after();
      // stages written by cp.async (generic proxy) are read by the tensor core
      if (p.sparse_idx) fence_proxy_async_smem();
      if (action == 2) {
        const uint32_t kv = sRing + (qk % kSt) * G::kStageBytes;
        // zero the cache rows past the unit's end in its last tile (they may
        // hold anything, NaN included): 0 * NaN would poison O
        const int nv = min(kPage, wq.S - wq.i * kPage);
        if (nv < kPage) {
          const int zrows = kPage - nv;
          for (int i = lane; i < 36 * zrows; i += 32) {
            // 16-byte chunks: 8 per row of each latent box, 4 per rope row
            const int r = nv + i / 36, k = i % 36;
            const uint32_t a = k < 32 ? kv + (k >> 3) * kColBytes + r * 128 + (k & 7) * 16
                                      : kv + 4 * kColBytes + r * 64 + (k - 32) * 16;
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        if (lane == 0) {
          // latent dims 256 r .. 256 r + 255 (16 k-steps, 128-byte swizzle),
          // rope dims 512 + 32 r .. (2 k-steps, 64-byte swizzle).  Fully
          // unrolled with every descriptor a constant offset from two bases
          // (the start address field counts 16-byte units): a loop that
          // rebuilds descriptors costs ~90 issue cycles per MMA against ~46.
          const uint64_t b_lat = umma_smem_desc(kv, 16, 1024, kSwizzle128);
          const uint64_t b_rope = umma_smem_desc(kv + 4 * kColBytes, 16, 512, kSwizzle64);
          #pragma unroll
          for (int i = 0; i < 18; ++i) {
            const uint64_t bk =
                i < 16 ? b_lat + static_cast<uint64_t>(((i >> 2) * kColBytes + (i & 3) * 32) >> 4)
                       : b_rope + static_cast<uint64_t>(((i - 16) * 32) >> 4);
            umma_bf16_ts(tmem + G::kSCol, tmem + G::kQCol + 8 * i, bk, idesc_qk, i != 0);
          }
          umma_commit(bar_sfull);
        }
        __syncwarp();
        if (qk == 0 || wq.i == 0) ++qseg;
        ++qk;
        if (qk < ntiles) wq.next(p);
      } else {
        // the first PV of a unit starts O afresh
        const bool first = pv == 0 || wv.i == 0;
        if (lane == 0) {
          const uint32_t kv = sRing + (pv % kSt) * G::kStageBytes;
          const uint64_t bv = umma_smem_desc(kv, kColBytes, 1024, kSwizzle128);
          #pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_ts(tmem + G::kOCol, tmem + G::kPCol + 8 * kk,
                         bv + static_cast<uint64_t>((kk * 16 * 128) >> 4), idesc_pv,
                         (first ? kk : 1) != 0);
          umma_commit(bar_pv);
          umma_commit(bar_empty + 8 * (pv % kSt));
        }
        __syncwarp();
        ++pv;
        if (pv < ntiles) wv.next(p);
      }
    }
    if (!ok) raise(kStatusWaitTimeout);
    // every MMA this thread issued has completed before TMEM is released
    if (lane == 0) umma_commit(bar_fin);
    __syncwarp();
    if (!wait_warp(bar_fin, 0)) raise(kStatusWaitTimeout);
  } else if (warp >= 10) {
    // -------------------- sender warps 10..13: partials out, Q_r in ----------
    // Warp w (TMEM lane quadrant w % 4) reads this CTA's partial scores of
    // its 32 rows, all 64 tokens, and stores them into the peer's exchange
    // buffer: the ~16 bytes per cycle the pair's link moves no longer stall
    // the softmax warps.  The same warps put each unit's Q_r rows of their
    // quadrant into tensor memory: the first unit's from the ring stages
    // TMA filled, every later one straight from global memory (prefetched
    // into L2 four tiles earlier) as soon as the previous unit's last QK is
    // done, while the softmax warps finish that unit.
    const int qs = warp & 3;
    const int hs = 32 * qs + lane;
    const uint32_t lane_base_s = static_cast<uint32_t>(32 * qs) << 16;
    const uint32_t peer_x = mapa_shared(sX, peer);
    const uint32_t peer_xfull = mapa_shared(bar_xfull, peer);
    bool ok = true;
    auto wait_cluster = [&](uint32_t bar, uint32_t parity) {
      if (!ok) return;
      bool done = mbar_try_wait_cluster(bar, parity);
      if (!done) {
        const unsigned long long t_start = global_timer_ns();
        while (!(done = mbar_try_wait_cluster(bar, parity)))
          if (global_timer_ns() - t_start > kWaitLimitNs) break;
      }
      if (!__all_sync(0xffffffffu, done)) ok = false;
    };
    // Q_r of unit uq, row hs, from global memory: nine chunks of 16 columns
    // (two bf16 each; chunks 0-7 this CTA's latent dims, 8 its rope dims),
    // three chunks in flight at a time; padding rows zero
    auto row_ptr = [&](int uq, bool& valid) {
      const int rowq = (uq % p.n_hg) * 128 + hs;
      valid = rowq < p.rows;
      return reinterpret_cast<const uint4*>(
          p.q + (static_cast<size_t>(uq / p.n_hg) * p.rows + (valid ? rowq : 0)) * kD);
    };
    auto col16 = [&](int j) {  // first 16-byte unit of chunk j in the row
      return j < 8 ? (256 * static_cast<int>(rank) + 32 * j) / 8
                   : (512 + 32 * static_cast<int>(rank)) / 8;
    };
    auto load_q = [&](int uq) {
      bool valid;
      const uint4* src = row_ptr(uq, valid);
      #pragma unroll 1
      for (int j0 = 0; j0 < 9; j0 += 3) {
        uint4 v[3][4];
        #pragma unroll
        for (int jj = 0; jj < 3; ++jj)
          #pragma unroll
          for (int k = 0; k < 4; ++k)
            v[jj][k] = valid ? __ldg(src + col16(j0 + jj) + k) : make_uint4(0, 0, 0, 0);
        #pragma unroll
        for (int jj = 0; jj < 3; ++jj) {
          uint32_t r[16];
          #pragma unroll
          for (int k = 0; k < 4; ++k) {
            r[4 * k] = v[jj][k].x;
            r[4 * k + 1] = v[jj][k].y;
            r[4 * k + 2] = v[jj][k].z;
            r[4 * k + 3] = v[jj][k].w;
          }
          tmem_st16(tmem + lane_base_s + G::kQCol + 16 * (j0 + jj), r);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_qready);
    };
    auto prefetch_q = [&](int uq) {
      bool valid;
      const char* src = reinterpret_cast<const char*>(row_ptr(uq, valid));
      if (!valid) return;
      #pragma unroll
      for (int l = 0; l < 4; ++l) prefetch_l2(src + 512 * rank + 128 * l);
      prefetch_l2(src + 2 * rope_x);
    };
    TileWalk ws;  // the tile being sent
    if (ntiles > 0) {
      ws.init(p, u0, start0, g0);
      // the first unit's Q_r from the ring (128-byte swizzled latent boxes,
      // 64-byte swizzled rope box)
      if (ok && !wait_warp(bar_q, 0)) ok = false;
      const bool valid0 = (u0 % p.n_hg) * 128 + hs < p.rows;
      #pragma unroll 1
      for (int j = 0; j < 9; ++j) {
        uint32_t r[16];
        #pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (valid0) {
            const uint32_t a =
                j < 8 ? sQ + (j >> 1) * G::kQLatBytes + hs * 128 +
                            (((4 * (j & 1) + k) ^ (hs & 7)) << 4)
                      : sQ + 4 * G::kQLatBytes + hs * 64 + ((k ^ ((hs >> 1) & 3)) << 4);
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                         : "r"(a));
          }
          r[4 * k] = v.x;
          r[4 * k + 1] = v.y;
          r[4 * k + 2] = v.z;
          r[4 * k + 3] = v.w;
        }
        tmem_st16(tmem + lane_base_s + G::kQCol + 16 * j, r);
      }
      tmem_wait_st();
      fence_proxy_async_smem();  // our reads precede the TMA writes into these stages
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar_qfree);
        mbar_arrive(bar_qready);
      }
    }
    for (int t = 0; t < ntiles; ++t) {
      const int j = t & 1;
      // this tile ends its unit and the range goes on: the next unit
      const bool unit_end = ws.i == ws.n - 1 && t + 1 < ntiles;
      const int left = ws.n - 1 - ws.i;  // tiles of the unit after this one
      if ((left == 4 || (t == 0 && left < 4)) && t + left + 1 < ntiles) {
        TileWalk wn = ws;
        wn.i = wn.n - 1;
        wn.next(p);
        prefetch_q(wn.u);
      }
      if (ok && !wait_warp(bar_sfull, t & 1)) ok = false;
      tc_fence_after();
      uint32_t r[4][16];
      #pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld16(tmem + lane_base_s + G::kSCol + 16 * cc, r[cc]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree);
      // the peer's softmax warps have read what we put in X[j] two tiles ago
      if (t >= 2) wait_cluster(bar_xfree + 8 * j, ((t - 2) >> 1) & 1);
      #pragma unroll
      for (int g = 0; g < 16; ++g)
        st_async_v4(peer_x + j * G::kXBytes + (g * 128 + hs) * 16, r[g >> 2][4 * (g & 3)],
                    r[g >> 2][4 * (g & 3) + 1], r[g >> 2][4 * (g & 3) + 2],
                    r[g >> 2][4 * (g & 3) + 3], peer_xfull + 8 * j);
      if (t + 1 < ntiles) ws.next(p);
      // every QK of the unit has completed (its last partials were read):
      // the next unit's rows may replace Q_r
      if (unit_end) load_q(ws.u);
    }
    // the peer has read our last two partials before either CTA may exit
    for (int t = max(0, ntiles - 2); t < ntiles; ++t)
      wait_cluster(bar_xfree + 8 * (t & 1), (t >> 1) & 1);
    if (!ok) raise(kStatusWaitTimeout);
  } else {
    // ------------------------- softmax warps 2..9 ----------------------------
    // Warp w owns TMEM lane quadrant w % 4 (rows h = 32 (w % 4) + lane) and
    // tokens 32 hf .. 32 hf + 31 of every tile, hf = (w - 2) / 4; the two
    // warps of a quadrant agree on each tile's row max through shared memory.
    // Every softmax warp runs the same barrier sequence whatever happens (a
    // failed wait only clears `ok`).
    const int q4 = warp & 3, hf = (warp - 2) >> 2;
    const int h = 32 * q4 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(32 * q4) << 16;
    const uint32_t peer_xfree = mapa_shared(bar_xfree, peer);
    float* red = reinterpret_cast<float*>(smem + G::kSmall + G::kRed);  // [3][2][128]
    bool ok = true;
    auto wait_pv = [&](int k) {  // completion of PV(k): phase k of bar_pv
      if (k >= 0 && ok && !wait_warp(bar_pv, k & 1)) ok = false;
    };
    auto wait_cluster = [&](uint32_t bar, uint32_t parity) {
      if (!ok) return;
      bool done = mbar_try_wait_cluster(bar, parity);
      if (!done) {
        const unsigned long long t_start = global_timer_ns();
        while (!(done = mbar_try_wait_cluster(bar, parity)))
          if (global_timer_ns() - t_start > kWaitLimitNs) break;
      }
      if (!__all_sync(0xffffffffu, done)) ok = false;
    };
    // this CTA's partial scores of tile t, this warp's rows and tokens
    auto read_s = [&](int t, float (&x)[32]) {
      if (ok && !wait_warp(bar_sfull, t & 1)) ok = false;
      tc_fence_after();
      uint32_t r[2][16];
      tmem_ld16(tmem + lane_base + G::kSCol + 32 * hf, r[0]);
      tmem_ld16(tmem + lane_base + G::kSCol + 32 * hf + 16, r[1]);
      tmem_wait_ld();
      #pragma unroll
      for (int k = 0; k < 16; ++k) {
        x[k] = __uint_as_float(r[0][k]);
        x[16 + k] = __uint_as_float(r[1][k]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree);
    };
    if (ntiles > 0 && warp == 2 && lane == 0) {
      mbar_arrive_expect_tx(bar_xfull, G::kXBytes);
      if (ntiles > 1) mbar_arrive_expect_tx(bar_xfull + 8, G::kXBytes);
    }
    TileWalk w;
    if (ntiles == 0 && p.per_unit) {
      // one unit per pair and no selected token: zero rows, lse = -inf
      const int b = u0 / p.n_hg, row = (u0 % p.n_hg) * 128 + h;
      if (row < p.rows) {
        uint4* dst = reinterpret_cast<uint4*>(
            p.out + (static_cast<size_t>(b) * p.rows + row) * kDV + 256 * rank + 128 * hf);
        #pragma unroll
        for (int e = 0; e < 16; ++e) dst[e] = make_uint4(0, 0, 0, 0);
        if (rank == 0 && hf == 0)
          p.lse[(static_cast<size_t>(b) * p.h_q + row % p.h_q) * p.s_q + row / p.h_q] = -INFINITY;
      }
    }
    if (ntiles > 0) w.init(p, u0, start0, g0);
    int t = 0;
    while (t < ntiles) {
      // ---- a segment: tiles i0 .. i0 + len - 1 of unit w.u ----
      const int u = w.u, b = u / p.n_hg, hg = u % p.n_hg, S = w.S, n_u = w.n;
      const int i0 = w.i, len = min(n_u - i0, ntiles - t);
      const int row0 = hg * 128, row = row0 + h;
      const bool valid = row < p.rows;
      const int vis = valid ? visible(p, S, row) : 0;
      // the unit's first tile is here: its partial-state layout for the
      // combine pass (pairs c .. c + nseg - 1; this pair's slot for it)
      if (i0 == 0 && !p.per_unit && rank == 0 && warp == 2 && lane == 0)
        p.unit_info[u] = make_int4(2 * c + (t == 0 ? 0 : 1), c,
                                   pair_of(static_cast<long long>(w.start) + n_u - 1, T, Pe) - c + 1,
                                   0);
      // the range goes on past this unit (then the segment runs to its end)
      const bool has_next = t + len < ntiles;
      // the unit's online softmax over the segment; iteration k reads its
      // partial of the next tile of the segment first (freeing S for the
      // QK after it), then adds the peer's partial of tile t + k
      float m_ref = -INFINITY, l = 0.f;
      float xn[32];
      read_s(t, xn);
      // the following unit's length, loaded now so that moving on to it
      // costs no memory round trip (nothing is added to the tile loop: its
      // schedule is sensitive to extra work)
      const int len_next = has_next ? __ldg(unit_len_ptr(p, w.u + 1)) : 0;
      for (int k = 0; k < len; ++k) {
        const int tt = t + k, i = i0 + k;
        float x[32];
        #pragma unroll
        for (int e = 0; e < 32; ++e) x[e] = xn[e];
        if (k + 1 < len) read_s(tt + 1, xn);
        const int j = tt & 1;
        wait_cluster(bar_xfull + 8 * j, (tt >> 1) & 1);
        uint32_t dep = 0;
        #pragma unroll
        for (int g = 0; g < 8; ++g) {
          float4 o;
          asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(o.x), "=f"(o.y), "=f"(o.z), "=f"(o.w)
                       : "r"(sX + j * G::kXBytes + ((8 * hf + g) * 128 + h) * 16)
                       : "memory");
          // S_0 + S_1 in both CTAs (addition commutes: identical bits)
          x[4 * g] += o.x;
          x[4 * g + 1] += o.y;
          x[4 * g + 2] += o.z;
          x[4 * g + 3] += o.w;
          dep ^= __float_as_uint(o.x) ^ __float_as_uint(o.w);
        }
        // every lane's reads are complete once all lanes produced dep; then
        // the peer may overwrite the buffer (with tile tt + 2, armed here)
        dep = __reduce_xor_sync(0xffffffffu, dep);
        // (the segment's last buffer is released after the epilogue, which
        // uses it as scratch)
        if (lane == 0 && k + 1 < len) mbar_arrive_remote_relaxed(peer_xfree + 8 * j, dep);
        if (warp == 2 && lane == 0 && tt + 2 < ntiles)
          mbar_arrive_expect_tx(bar_xfull + 8 * j, G::kXBytes);
        // scores in the log2 domain, masked past the row's visible range
        const int nvis = min(32, max(0, vis - i * kPage - 32 * hf));
        float mt = -INFINITY;
        #pragma unroll
        for (int e = 0; e < 32; ++e) {
          x[e] = e < nvis ? x[e] * p.scale_log2 : -INFINITY;
          mt = fmaxf(mt, x[e]);
        }
        // the row max over both halves of the tile
        red[(j * 2 + hf) * 128 + h] = mt;
        named_bar_sync(1 + q4, 64);
        mt = fmaxf(mt, red[(j * 2 + (hf ^ 1)) * 128 + h]);
        const bool need = mt > m_ref + kRescaleLog2;
        if (__any_sync(0xffffffffu, need)) {
          float alpha = 1.f;
          if (need) {
            alpha = m_ref == -INFINITY ? 0.f : exp2f(m_ref - mt);
            m_ref = mt;
            l *= alpha;
          }
          if (k >= 1) {
            // this warp's 128 of the row's O columns *= alpha once every
            // earlier PV has accumulated into them
            wait_pv(tt - 1);
            tc_fence_after();
            #pragma unroll 1
            for (int cc = 0; cc < 8; ++cc) {
              uint32_t r[16];
              const uint32_t a = tmem + lane_base + G::kOCol + 128 * hf + 16 * cc;
              tmem_ld16(a, r);
              tmem_wait_ld();
              #pragma unroll
              for (int e = 0; e < 16; ++e)
                r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
              tmem_st16(a, r);
            }
            tmem_wait_st();
          }
        }
        // P = 2^(x - m_ref) as bf16 pairs; the buffer is free once PV(tt - 1)
        // (of this unit or the previous one) is done
        uint32_t pk[16];
        #pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = x[2 * e] == -INFINITY ? 0.f : fast_exp2(x[2 * e] - m_ref);
          const float p1 = x[2 * e + 1] == -INFINITY ? 0.f : fast_exp2(x[2 * e + 1] - m_ref);
          l += p0 + p1;
          pk[e] = pack2(p0, p1);
        }
        wait_pv(tt - 1);
        tc_fence_after();
        tmem_st16(tmem + lane_base + G::kPCol + 16 * hf, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_pfull);
      }
      // ---- the segment's epilogue (the sender warps have meanwhile put the
      // next unit's Q_r into tensor memory, so its first QK and exchange
      // overlap this) ----
      const int t_last = t + len - 1;
      wait_pv(t_last);
      tc_fence_after();
      red[(2 * 2 + hf) * 128 + h] = l;
      named_bar_sync(1 + q4, 64);
      l += red[(2 * 2 + (hf ^ 1)) * 128 + h];
      const float m = l > 0.f ? m_ref : -INFINITY;
      const int dv0 = 256 * static_cast<int>(rank) + 128 * hf;
      const int qi = row / p.h_q, hq = row % p.h_q;
      // The rows leave through a 4 KB scratch area of this warp in the
      // exchange buffer of the segment's last tile (read above; the peer
      // refills it only after the release below): each lane writes its row's
      // 128 bytes of a pass (16-byte chunks XOR-swizzled by row), then the
      // warp stores four rows of 128 contiguous bytes per instruction
      // instead of 32 rows of 16.
      const uint32_t scr = sX + (t_last & 1) * G::kXBytes + (warp - 2) * 4096;
      auto put = [&](int ch, uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3) {
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(
                         scr + lane * 128 + ((ch ^ (lane & 7)) << 4)),
                     "r"(x0), "r"(x1), "r"(x2), "r"(x3)
                     : "memory");
      };
      uint32_t dep = 0;
      // pass rows out: the eight 16-byte chunks of row rr of the scratch
      auto drain = [&](auto&& store) {
        __syncwarp();
        #pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = 4 * i + (lane >> 3), ch = lane & 7;
          uint4 v;
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                       : "r"(scr + rr * 128 + ((ch ^ (rr & 7)) << 4))
                       : "memory");
          dep ^= v.x;
          store(32 * q4 + rr, ch, v);
        }
        __syncwarp();
      };
      if (i0 == 0 && len == n_u) {
        // the whole unit in this pair: the final rows, 64 value dims a pass
        const float inv = l > 0.f ? 1.f / l : 0.f;
        #pragma unroll 1
        for (int ps = 0; ps < 2; ++ps) {
          #pragma unroll 1
          for (int cc = 0; cc < 4; cc += 2) {
            uint32_t r[2][16];
            tmem_ld16(tmem + lane_base + G::kOCol + 128 * hf + 64 * ps + 16 * cc, r[0]);
            tmem_ld16(tmem + lane_base + G::kOCol + 128 * hf + 64 * ps + 16 * cc + 16, r[1]);
            tmem_wait_ld();
            #pragma unroll
            for (int x = 0; x < 2; ++x) {
              uint32_t wv[8];
              #pragma unroll
              for (int e = 0; e < 8; ++e)
                wv[e] = pack2(__uint_as_float(r[x][2 * e]) * inv,
                              __uint_as_float(r[x][2 * e + 1]) * inv);
              put(2 * (cc + x), wv[0], wv[1], wv[2], wv[3]);
              put(2 * (cc + x) + 1, wv[4], wv[5], wv[6], wv[7]);
            }
          }
          drain([&](int hr, int ch, uint4 v) {
            const int orow = row0 + hr;
            if (orow < p.rows)
              *reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(b) * p.rows + orow) * kDV +
                                        dv0 + 64 * ps + 8 * ch) = v;
          });
        }
        if (rank == 0 && hf == 0 && valid)
          p.lse[(static_cast<size_t>(b) * p.h_q + hq) * p.s_q + qi] =
              l > 0.f ? (m + log2f(l)) * 0.69314718056f : -INFINITY;
      } else {
        // a partial state in this pair's slot (its first or its last unit),
        // 32 value dims a pass
        const int slot = 2 * c + (t == 0 ? 0 : 1);  // c < Pe <= P
        float* acc = p.slot_acc + static_cast<size_t>(slot) * 128 * kDV;
        #pragma unroll 1
        for (int ps = 0; ps < 4; ++ps) {
          uint32_t r[2][16];
          tmem_ld16(tmem + lane_base + G::kOCol + 128 * hf + 32 * ps, r[0]);
          tmem_ld16(tmem + lane_base + G::kOCol + 128 * hf + 32 * ps + 16, r[1]);
          tmem_wait_ld();
          #pragma unroll
          for (int x = 0; x < 2; ++x)
            #pragma unroll
            for (int e = 0; e < 4; ++e)
              put(4 * x + e, r[x][4 * e], r[x][4 * e + 1], r[x][4 * e + 2], r[x][4 * e + 3]);
          drain([&](int hr, int ch, uint4 v) {
            *reinterpret_cast<uint4*>(acc + static_cast<size_t>(hr) * kDV + dv0 + 32 * ps + 4 * ch) = v;
          });
        }
        if (rank == 0 && hf == 0) {  // identical in both CTAs of the pair
          p.slot_m[static_cast<size_t>(slot) * 128 + h] = m;
          p.slot_l[static_cast<size_t>(slot) * 128 + h] = l;
        }
        // mla_rows_combine_kernel merges the unit's partial states
      }
      // the scratch reads are done: the peer may refill the buffer
      dep = __reduce_xor_sync(0xffffffffu, dep);
      if (lane == 0) mbar_arrive_remote_relaxed(peer_xfree + 8 * (t_last & 1), dep);
      tc_fence_before();
      // next segment: the next unit's first tile
      t += len;
      if (has_next) {
        const int n_next = (unit_clamp(p, len_next) + kPage - 1) / kPage;
        if (n_next > 0) {  // the usual case: the next unit has tiles
          w.start += w.n;
          ++w.u;
          w.i = 0;
          w.S = unit_clamp(p, len_next);
          w.n = n_next;
        } else {
          w.i = w.n - 1;
          w.next(p);
        }
      }
    }
    if (!ok) raise(kStatusWaitTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  cluster_sync();  // no CTA leaves while its peer may still address its shared memory
}

// Units of the persistent 128-row kernel that were split between pairs:
// merge their partial states (one per pair) into out and lse; also the
// output of units with no tokens, which no pair visits.  One warp per query
// row (eight rows per block): lane k < nseg loads segment k's max and sum
// (warp-reduced), then every lane merges 16 of the 512 value dims, four
// segments' loads in flight at a time.  The unit's layout (first slot,
// first pair, pairs) was recorded by the pair that ran its first tile:
// segment 0 is in that slot, segment k > 0 in slot 2 (first pair + k),
// where it opens that pair's range.
__global__ void __launch_bounds__(256)
    mla_rows_combine_kernel(const __grid_constant__ Params p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u = blockIdx.x >> 4, h = (blockIdx.x & 15) * 8 + warp;
  const int b = u / p.n_hg, row = (u % p.n_hg) * 128 + h;
  const int4 info = __ldcg(p.unit_info + u);  // in flight with the token count
  const int n_u = (unit_tokens(p, u) + kPage - 1) / kPage;
  if (row >= p.rows) return;
  int s0 = 0, c0 = 0, nseg = 0;
  if (n_u > 0) {
    s0 = info.x;
    c0 = info.y;
    nseg = info.z;
    if (nseg <= 1) return;  // written by its pair
  }
  auto slot = [&](int k) { return static_cast<size_t>(k == 0 ? s0 : 2 * (c0 + k)) * 128 + h; };
  float M = -INFINITY, L = 0.f;
  float4 a[4];
  #pragma unroll
  for (int d = 0; d < 4; ++d) a[d] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k0 = 0; k0 < nseg; k0 += 32) {
    // this group's maxima and sums, one segment per lane
    const int kl = k0 + lane;
    const float ml = kl < nseg ? __ldcg(p.slot_m + slot(kl)) : -INFINITY;
    const float ll = kl < nseg ? __ldcg(p.slot_l + slot(kl)) : 0.f;
    float mg = ml;
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, off));
    const float mn = fmaxf(M, mg);
    // rescale what earlier groups merged (at most one group below 32 pairs)
    const float r = M == -INFINITY ? 0.f : exp2f(M - mn);
    L *= r;
    #pragma unroll
    for (int d = 0; d < 4; ++d) {
      a[d].x *= r;
      a[d].y *= r;
      a[d].z *= r;
      a[d].w *= r;
    }
    M = mn;
    const float wl = ml == -INFINITY ? 0.f : exp2f(ml - M);
    float ls = wl * ll;
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
    L += ls;
    const int ng = min(32, nseg - k0);
    for (int e0 = 0; e0 < ng; e0 += 4) {
      float4 v[4][4];
      float w[4];
      #pragma unroll
      for (int e = 0; e < 4; ++e) {
        w[e] = __shfl_sync(0xffffffffu, wl, (e0 + e) & 31);
        if (e0 + e < ng) {
          const float4* src =
              reinterpret_cast<const float4*>(p.slot_acc + slot(k0 + e0 + e) * kDV) + 4 * lane;
          #pragma unroll
          for (int d = 0; d < 4; ++d) v[e][d] = __ldcg(src + d);
        } else {
          w[e] = 0.f;
          #pragma unroll
          for (int d = 0; d < 4; ++d) v[e][d] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      #pragma unroll
      for (int e = 0; e < 4; ++e) {
        #pragma unroll
        for (int d = 0; d < 4; ++d) {
          a[d].x += w[e] * v[e][d].x;
          a[d].y += w[e] * v[e][d].y;
          a[d].z += w[e] * v[e][d].z;
          a[d].w += w[e] * v[e][d].w;
        }
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  uint4* dst =
      reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(b) * p.rows + row) * kDV + 16 * lane);
  #pragma unroll
  for (int d = 0; d < 2; ++d)
    dst[d] = make_uint4(pack2(a[2 * d].x * inv, a[2 * d].y * inv),
                        pack2(a[2 * d].z * inv, a[2 * d].w * inv),
                        pack2(a[2 * d + 1].x * inv, a[2 * d + 1].y * inv),
                        pack2(a[2 * d + 1].z * inv, a[2 * d + 1].w * inv));
  if (lane == 0)
    p.lse[(static_cast<size_t>(b) * p.h_q + row % p.h_q) * p.s_q + row / p.h_q] =
        L > 0.f ? (M + log2f(L)) * 0.69314718056f : -INFINITY;
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
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint32_t box_rows,
              uint32_t box_cols = 64) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD) * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Query rows per CTA: the smallest of 16 / 32 / 64 holding all rows of a
// request, else 64 (the last group of a request is padded; padded rows are
// computed on whatever the q tile holds there and never stored).
// Query rows per CTA pair: the smallest of 16 / 32 / 64 / 128 holding all
// rows of a request, else 128 (the last group of a request is padded;
// padded rows are computed on whatever the q tile holds there and never
// stored).
int rows_per_pair(int rows) {
  if (rows <= 0) return 0;
  return rows <= 16 ? 16 : (rows <= 32 ? 32 : (rows <= 64 ? 64 : 128));
}

struct Layout {
  int NH, n_hg, smem;
};

Layout layout_for(int rows) {
  Layout L{};
  L.NH = rows_per_pair(rows);
  if (L.NH == 0) return L;
  L.n_hg = (rows + L.NH - 1) / L.NH;
  L.smem = L.NH == 16    ? gqa::mla::Pair<16>::kSmem
           : L.NH == 32  ? gqa::mla::Pair<32>::kSmem
           : L.NH == 64  ? gqa::mla::Pair<64>::kSmem
                         : gqa::mla::Rows::kSmem;  // 128-row groups: the rows kernel
  return L;
}

// 128-row groups run persistent on as many CTA pairs as fit on the device
// at once: at most half the SMs, fewer when the GPCs' SM counts leave some
// SMs without a cluster partner (cached per device).
int rows_pairs() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  v = sms / 2 > 0 ? sms / 2 : 1;
  int n = 0;
  using gqa::mla::Rows;
  using gqa::mla::mla_decode_rows_kernel;
  if (cudaFuncSetAttribute(mla_decode_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           Rows::kSmem) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * v);
    cfg.blockDim = dim3(Rows::kThreads);
    cfg.dynamicSmemBytes = Rows::kSmem;
    if (cudaOccupancyMaxActiveClusters(&n, mla_decode_rows_kernel, &cfg) == cudaSuccess && n > 0 &&
        n < v)
      v = n;
  }
  cudaGetLastError();  // a failed query leaves the SM-count bound
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

// Workspace of the persistent 128-row kernel: the tile count and working
// pairs, per-unit first tile and tile count, partial max and sum [2 P][128],
// partial O [2 P][128][512].
struct RowsWs {
  size_t hdr, info, m, l, acc, total;
};
RowsWs rows_ws(int units, int P) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  RowsWs w{};
  w.hdr = 0;
  w.info = 256;
  w.m = w.info + up(static_cast<size_t>(units) * sizeof(int4));
  w.l = w.m + up(static_cast<size_t>(2) * P * 128 * sizeof(float));
  w.acc = w.l + up(static_cast<size_t>(2) * P * 128 * sizeof(float));
  w.total = w.acc + static_cast<size_t>(2) * P * 128 * kDV * sizeof(float);
  return w;
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
  if (L.NH == 128) return 1;  // persistent, balanced by tiles: no splits
  const long long units = static_cast<long long>(B) * L.n_hg;
  // Cost model over CTA-pair waves (groups of fewer than 128 rows): each
  // split is a pair that pays a fixed start (tensor memory, Q staging, the
  // first pages' latency) worth about five page-times, and splits > 1 add
  // partial states and a combine pass.  Fitted on B200 when every group ran
  // one pair per (unit, split): it picked the fastest of 1-16 splits for
  // ~8K-token requests and 2K-token selections.
  const long long slots = std::max(1, num_sms / 2);
  const long long cap = std::max(1, std::min(64, max_pages / 2));
  const long long pages = std::max(1, max_pages);
  long long best = 1;
  double best_cost = 1e300;
  for (long long ns = 1; ns <= cap; ++ns) {
    const long long waves = (units * ns + slots - 1) / slots;
    const double cost = static_cast<double>(waves) *
                        (static_cast<double>((pages + ns - 1) / ns) + 5.0 + (ns > 1 ? 1.0 : 0.0));
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = ns;
    }
  }
  return static_cast<int>(best);
}

size_t mla_decode_workspace_bytes(int B, int s_q, int h_q, int num_splits) {
  if (B <= 0 || s_q <= 0 || h_q <= 0) return 0;
  const Layout L = layout_for(s_q * h_q);
  if (L.NH == 128) return rows_ws(B * L.n_hg, rows_pairs()).total;  // persistent, any num_splits
  if (num_splits <= 1) return 0;
  return part_bytes(B, s_q * h_q, num_splits);
}

}  // extern "C"

namespace {

// The dense launch and the sparse one (sparse_idx != null: seq_lens holds
// the selected counts per query position, and h_q is a multiple of 128 so
// that every 128-row group belongs to one query position).
cudaError_t mla_launch_impl(const gqa_bf16* q, const gqa_bf16* kv_cache, const int* block_table,
                            const int* seq_lens, const int* sparse_idx, int topk, gqa_bf16* out,
                            float* lse, int B, int s_q, int h_q, int page_size, int max_blocks,
                            int num_blocks, float softmax_scale, int causal, int num_splits,
                            void* workspace, size_t workspace_bytes, cudaStream_t stream,
                            int sparse_rows = 0) {
  using namespace gqa::mla;
  if (B < 0 || s_q <= 0 || h_q <= 0 || page_size != kPage || max_blocks <= 0 || num_blocks <= 0 ||
      num_splits < 1 || num_splits > 64)
    return cudaErrorInvalidValue;
  if (sparse_idx && (h_q % 128 != 0 || topk <= 0 || causal)) return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  const int rows = s_q * h_q;
  const Layout L = layout_for(rows);
  if (L.NH == 0) return cudaErrorInvalidValue;
  if (!q || !kv_cache || (!block_table && !sparse_rows) || !seq_lens || !out || !lse)
    return cudaErrorInvalidValue;
  if (!aligned16(q) || !aligned16(kv_cache)) return cudaErrorMisalignedAddress;
  Params p{};
  p.sparse_idx = sparse_idx;
  p.sparse_rows = sparse_rows;
  p.kv = reinterpret_cast<const __nv_bfloat16*>(kv_cache);
  p.topk = topk;

  if (!make_map(&p.tm_q, q, static_cast<uint64_t>(B) * rows, static_cast<uint32_t>(L.NH)) ||
      !make_map(&p.tm_kv, kv_cache, static_cast<uint64_t>(num_blocks) * kPage, kPage))
    return cudaErrorInvalidValue;
  if (L.NH == 128 &&
      (!make_map(&p.tm_q_rope, q, static_cast<uint64_t>(B) * rows, 128u, 32u) ||
       !make_map(&p.tm_kv_rope, kv_cache, static_cast<uint64_t>(num_blocks) * kPage, kPage, 32u)))
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
  p.num_splits = L.NH == 128 ? 1 : num_splits;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  int P = L.NH == 128 ? rows_pairs() : 0;
  // Sparse selections make near-uniform units of up to ceil(topk / 64)
  // tiles.  Whole units per pair (in waves) skip the partial states and
  // the merge but idle pairs in a short last wave; the balanced split pays
  // a fixed cost per launch (unit boundaries, the merge pass).  Measured on
  // B200 (top-k 2048, 128 heads): about 3.3 us per tile + 6 us per wave of
  // whole units, against 30 us + 3.7 us per tile of the balanced split, so
  // choose whichever the two fits predict faster.  Dense caches always
  // take the balanced split.
  p.per_unit = 0;
  if (L.NH == 128 && sparse_idx) {
    const long long U = static_cast<long long>(B) * L.n_hg, nt = (topk + kPage - 1) / kPage;
    const long long waves = (U + P - 1) / P;
    const double whole = static_cast<double>(waves) * (3.3 * nt + 6.0);
    const double balanced = 30.0 + 3.7 * static_cast<double>(U * nt) / P;
    p.per_unit = whole <= balanced ? 1 : 0;
  }
  if (L.NH == 128) {
    const RowsWs wl = rows_ws(B * L.n_hg, P);
    if (!workspace || workspace_bytes < wl.total || !aligned16(workspace))
      return cudaErrorInvalidValue;
    unsigned char* w = static_cast<unsigned char*>(workspace);
    p.hdr = reinterpret_cast<int*>(w + wl.hdr);
    p.unit_info = reinterpret_cast<int4*>(w + wl.info);
    p.slot_m = reinterpret_cast<float*>(w + wl.m);
    p.slot_l = reinterpret_cast<float*>(w + wl.l);
    p.slot_acc = reinterpret_cast<float*>(w + wl.acc);
  } else if (num_splits > 1) {
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
  static gqa::DeviceOnce attr_once;
  const cudaError_t attr_err = attr_once.run([] {
    const cudaError_t e[4] = {
        cudaFuncSetAttribute(mla_decode_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Pair<16>::kSmem),
        cudaFuncSetAttribute(mla_decode_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Pair<32>::kSmem),
        cudaFuncSetAttribute(mla_decode_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Pair<64>::kSmem),
        cudaFuncSetAttribute(mla_decode_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Rows::kSmem)};
    for (cudaError_t x : e)
      if (x != cudaSuccess) return x;
    return cudaSuccess;
  });
  if (attr_err != cudaSuccess) return attr_err;
  if (L.NH == 128) {
    // persistent pairs over the batch's tiles, then the split units' merge
    const long long pairs = p.per_unit ? static_cast<long long>(B) * L.n_hg : P;
    if (2 * pairs > 0x7fffffffLL) return cudaErrorInvalidValue;
    mla_decode_rows_kernel<<<static_cast<unsigned>(2 * pairs), Rows::kThreads, Rows::kSmem,
                             stream>>>(p);
    const cudaError_t e1 = cudaGetLastError();
    if (e1 != cudaSuccess || p.per_unit) return e1;  // one unit per pair: nothing to merge
    const long long blocks = static_cast<long long>(B) * L.n_hg * 16;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    mla_rows_combine_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
    return cudaGetLastError();
  }
  const long long grid = 2LL * B * L.n_hg * num_splits;  // 2-CTA clusters
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  const unsigned g = static_cast<unsigned>(grid);
  if (L.NH == 64)
    mla_decode_kernel<64><<<g, kThreads, L.smem, stream>>>(p);
  else if (L.NH == 32)
    mla_decode_kernel<32><<<g, kThreads, L.smem, stream>>>(p);
  else
    mla_decode_kernel<16><<<g, kThreads, L.smem, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || num_splits == 1) return e;
  CombineParams c{p.part_acc, p.part_m, p.part_l, out, lse, B, s_q, h_q, rows, num_splits};
  const long long nrows = static_cast<long long>(B) * rows;
  mla_combine_kernel<<<static_cast<unsigned>((nrows + 3) / 4), 128, 0, stream>>>(c);
  return cudaGetLastError();
}

}  // namespace

extern "C" {

cudaError_t mla_decode_launch(const gqa_bf16* q, const gqa_bf16* kv_cache, const int* block_table,
                              const int* seq_lens, gqa_bf16* out, float* lse, int B, int s_q,
                              int h_q, int page_size, int max_blocks, int num_blocks,
                              float softmax_scale, int causal, int num_splits, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream) {
  return mla_launch_impl(q, kv_cache, block_table, seq_lens, nullptr, 0, out, lse, B, s_q, h_q,
                         page_size, max_blocks, num_blocks, softmax_scale, causal, num_splits,
                         workspace, workspace_bytes, stream);
}

cudaError_t mla_decode_sparse_launch(const gqa_bf16* q, const gqa_bf16* kv_cache,
                                     const int* block_table, const int* indices,
                                     const int* counts, int topk, gqa_bf16* out, float* lse, int B,
                                     int s_q, int h_q, int page_size, int max_blocks,
                                     int num_blocks, float softmax_scale, int num_splits,
                                     void* workspace, size_t workspace_bytes,
                                     cudaStream_t stream) {
  if (!indices) return cudaErrorInvalidValue;
  return mla_launch_impl(q, kv_cache, block_table, counts, indices, topk, out, lse, B, s_q, h_q,
                         page_size, max_blocks, num_blocks, softmax_scale, 0, num_splits,
                         workspace, workspace_bytes, stream);
}

cudaError_t mla_decode_sparse_rows_launch(const gqa_bf16* q, const gqa_bf16* kv_cache,
                                          const int* cache_rows, const int* counts, int topk,
                                          gqa_bf16* out, float* lse, int B, int s_q, int h_q,
                                          int page_size, int num_blocks, float softmax_scale,
                                          int num_splits, void* workspace,
                                          size_t workspace_bytes, cudaStream_t stream) {
  if (!cache_rows) return cudaErrorInvalidValue;
  return mla_launch_impl(q, kv_cache, nullptr, counts, cache_rows, topk, out, lse, B, s_q, h_q,
                         page_size, 1, num_blocks, softmax_scale, 0, num_splits, workspace,
                         workspace_bytes, stream, 1);
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
