// Paged-KV GQA decode scan for sm_100a.
//
// Computes, for every request b and q head h (kv head hk = h / (Hq/Hkv),
// kernels/gqa_decode/v0_naive.cu:10, docs/decisions/k1-002):
//     out[b, h, :] = softmax_t(q[b,h,:] . K[t, hk, :] * scale) @ V[t, hk, :]
// over the first seq_lens[b] tokens, gathered through block_table from the
// NHD caches [num_blocks, bs, Hkv, 128] (python/reference.py:7-40).
//
// CTA layout (one persistent CTA per SM):
//   * warp ncw (the producer) walks the CTA's segments and, for every
//     16-token stage, issues 32 cp.async.bulk copies: lanes 0-15 copy the K
//     rows of the stage's tokens (HG heads = HG*256 contiguous bytes of a
//     token), lanes 16-31 the V rows.  Rows land in a ring of `nstages`
//     stages with a 16-byte skew per row so ldmatrix reads are bank-conflict
//     free.  Completion is tracked by mbarrier transaction counts.
//   * warps 0..ncw-1 (consumers) each own one kv head of the row and one
//     tile of up to 8 q heads.  Per stage: S^T[16 tok x 8 heads] = K q^T on
//     tensor cores (m16n8k16 bf16, tokens in M), fp32 online softmax in the
//     log2 domain, P^T transposed in registers (movmatrix) and
//     out^T[128 x 8] += V^T P^T on tensor cores.  One K/V read from HBM
//     serves all G q heads of the kv head.
// The running state (m, l, acc) is fp32 (docs/decisions/k1-003).  Partials
// are merged with M = max m_i, f_i = 2^(m_i - M), out = sum(acc_i f_i) /
// sum(l_i f_i) (kernels/gqa_decode/v2_splitkv.cu:97-107).
#include <math.h>

#include "gqa_internal.h"
#include "gqa_ptx.cuh"

namespace gqa {

__device__ int g_status;

namespace {

constexpr unsigned kFull = 0xffffffffu;
enum SegKind : int { kDirect = 0, kPartial = 1, kZero = 2 };

__device__ __forceinline__ void raise_status(int bits) { atomicOr(&g_status, bits); }

// Tokens of request b that are read: seq_lens[b] clamped to the table's
// capacity, so a bad length can never walk past the request's table row.
__device__ __forceinline__ int eff_len(const int* seq_lens, int b, long long cap) {
  long long s = ld_nc_s32(&seq_lens[b]);
  if (s < 0) s = 0;
  if (s > cap) s = cap;
  return static_cast<int>(s);
}

// Tokens of request b under the launch's page table.  CSR: (pages - 1) *
// bs + tokens of the last page, clamped to the pages present.
__device__ __forceinline__ int req_len(const ScanParams& p, int b, long long cap) {
  if (!p.csr) return eff_len(p.seq_lens, b, cap);
  const int n = ld_nc_s32(&p.kv_indptr[b + 1]) - ld_nc_s32(&p.kv_indptr[b]);
  if (n <= 0) return 0;
  long long s = static_cast<long long>(n - 1) * p.bs + ld_nc_s32(&p.kv_last[b]);
  if (s < 0) s = 0;
  if (s > static_cast<long long>(n) * p.bs) s = static_cast<long long>(n) * p.bs;
  return static_cast<int>(s);
}

// Physical block ids of request b, indexed by logical block.
__device__ __forceinline__ const int* page_row(const ScanParams& p, int b) {
  if (p.csr) return p.kv_indices + ld_nc_s32(&p.kv_indptr[b]);
  return p.block_table + static_cast<size_t>(b) * p.max_blocks;
}

struct Seg {
  int b, hg, row;  // request, kv-head group, row = b * NHG + hg
  int S;           // tokens of the request
  int s0, s1;      // stage range [s0, s1) inside the row
  int kind;        // SegKind
  int slot;        // FIXED: split index; BALANCED: first-slot base (see below)
  int nparts;      // number of segments the row was cut into
  long long cfirst;  // BALANCED: index of the first CTA that holds this row
};

// BALANCED ranges: the T stages of all rows, in row order, are cut into E =
// min(grid, T / 2) ranges with proportional boundaries [c T / E, (c+1) T / E)
// - sizes differ by at most one stage, and every range holds at least two
// stages so that no row is cut into single-stage parts.  CTAs c >= E idle.
__device__ __forceinline__ long long range_parts(long long T, long long grid) {
  return max(1LL, min(grid, T / 2));
}

__device__ __forceinline__ long long range_start(long long c, long long T, long long E) {
  return c >= E ? T : c * T / E;
}

// The range that holds stage g (0 <= g < T): the largest c with
// c T / E <= g, i.e. c T < (g + 1) E.
__device__ __forceinline__ long long range_owner(long long g, long long T, long long E) {
  return ((g + 1) * E - 1) / T;
}

struct SegIter {
  // FIXED
  int task, task_end, task_step;
  // BALANCED
  long long g, g_end, T, E, row0;
  int b, hg, S, L;
};

__device__ __forceinline__ bool iter_next(SegIter& it, const ScanParams& p, long long cap,
                                          Seg& s) {
  if (p.schedule == kFixed) {
    const int ns = p.num_splits;
    while (it.task < it.task_end) {
      const int t = it.task;
      it.task += it.task_step;
      const int row = t / ns;
      const int split = t - row * ns;
      const int b = row / p.NHG;
      const int hg = row - b * p.NHG;
      const int S = req_len(p, b, cap);
      const int L = (S + kStageTokens - 1) / kStageTokens;
      if (L == 0) {
        if (split != 0) continue;
        s = Seg{b, hg, row, 0, 0, 0, kZero, 0, 1, 0};
        return true;
      }
      const int chunk = (L + ns - 1) / ns;
      const int s0 = split * chunk;
      if (s0 >= L) continue;
      const int s1 = min(L, s0 + chunk);
      const int nonempty = (L + chunk - 1) / chunk;
      s = Seg{b, hg, row, S, s0, s1, nonempty == 1 ? kDirect : kPartial, split, nonempty, 0};
      return true;
    }
    return false;
  }
  while (it.g < it.g_end) {
    const long long rs = it.row0 + static_cast<long long>(it.hg) * it.L;
    const long long re = rs + it.L;
    if (it.g >= re) {
      if (++it.hg == p.NHG) {
        it.hg = 0;
        it.row0 += static_cast<long long>(p.NHG) * it.L;
        if (++it.b >= p.B) {
          it.g = it.g_end;
          return false;
        }
        it.S = req_len(p, it.b, cap);
        it.L = (it.S + kStageTokens - 1) / kStageTokens;
      }
      continue;
    }
    const long long e = min(it.g_end, re);
    s.b = it.b;
    s.hg = it.hg;
    s.row = it.b * p.NHG + it.hg;
    s.S = it.S;
    s.s0 = static_cast<int>(it.g - rs);
    s.s1 = static_cast<int>(e - rs);
    s.cfirst = range_owner(rs, it.T, it.E);
    s.nparts = static_cast<int>(range_owner(re - 1, it.T, it.E) - s.cfirst + 1);
    s.kind = s.nparts == 1 ? kDirect : kPartial;
    s.slot = static_cast<int>(blockIdx.x) + s.row;
    it.g = e;
    return true;
  }
  return false;
}

// Block-wide start of the CTA's range in the BALANCED schedule.  Every
// thread takes part; afterwards sh_* hold the range and its first request.
__device__ __forceinline__ void balanced_start(const ScanParams& p, long long cap, long long* sh_warp,
                               long long* sh_info) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthr = blockDim.x, nwarps = nthr >> 5;
  const int chunk = (p.B + nthr - 1) / nthr;
  const int blo = min(p.B, tid * chunk), bhi = min(p.B, blo + chunk);
  long long local = 0;
  for (int b = blo; b < bhi; ++b)
    local += (req_len(p, b, cap) + kStageTokens - 1) / kStageTokens;
  long long x = local;
  #pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const long long y = __shfl_up_sync(kFull, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) sh_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    long long t = lane < nwarps ? sh_warp[lane] : 0;
    #pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(kFull, t, off);
      if (lane >= off) t += y;
    }
    if (lane < nwarps) sh_warp[lane] = t;
  }
  __syncthreads();
  const long long excl = x - local + (warp > 0 ? sh_warp[warp - 1] : 0);
  const long long total = sh_warp[nwarps - 1];
  const long long T = total * p.NHG;
  const long long E = range_parts(T, gridDim.x);
  const long long g0 = range_start(blockIdx.x, T, E);
  const long long g1 = range_start(blockIdx.x + 1LL, T, E);
  if (tid == 0) {
    sh_info[0] = g0;
    sh_info[1] = g1;
    sh_info[2] = E;
    sh_info[3] = 0;  // first request
    sh_info[4] = 0;  // stages before it
    sh_info[5] = T;
  }
  __syncthreads();
  if (g0 < g1 && g0 >= excl * p.NHG && g0 < (excl + local) * p.NHG) {
    long long P = excl;
    for (int b = blo; b < bhi; ++b) {
      const long long L = (req_len(p, b, cap) + kStageTokens - 1) / kStageTokens;
      if (g0 < (P + L) * p.NHG) {
        sh_info[3] = b;
        sh_info[4] = P;
        break;
      }
      P += L;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void store_bf16x4(__nv_bfloat16* dst, float a, float b, float c,
                                             float d) {
  uint2 v;
  v.x = pack_bf16x2(a, b);
  v.y = pack_bf16x2(c, d);
  *reinterpret_cast<uint2*>(dst) = v;
}

// Zero output (or a neutral state: m = -inf, l = 0, acc = 0) for the q heads
// [hbase, hbase+cnt) of request b, which has no tokens.  The reference's
// kernels divide by l = 0 there (docs/decisions/k1-004); python/reference.py
// yields 0.  With kOutExchange nothing is written here: the row is recorded
// with no parts and the merge kernel exchanges its neutral state.
__device__ __forceinline__ void write_empty(const ScanParams& p, int b, int hbase, int cnt,
                                            int lane) {
  const size_t bh0 = static_cast<size_t>(b) * p.Hq + hbase;
  for (int n = 0; n < cnt; ++n) {
    if (p.out_mode == kOutBf16) {
      store_bf16x4(p.out + (bh0 + n) * kHeadDim + 4 * lane, 0.f, 0.f, 0.f, 0.f);
    } else if (p.out_mode == kOutState) {
      if (lane == 0) {
        p.res_m[bh0 + n] = -INFINITY;
        p.res_l[bh0 + n] = 0.f;
      }
      *reinterpret_cast<float4*>(p.res_acc + (bh0 + n) * kHeadDim + 4 * lane) =
          make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

}  // namespace

// kMaxWarps bounds the CTA (consumer warps + the copy warp) so the register
// budget fits it: 9 warps for groups of up to 8 heads per kv head (the common
// shapes, no spills), 17 for the widest groups.
template <int kMaxWarps>
__global__ void __launch_bounds__(kMaxWarps * 32, 1)
    gqa_decode_scan_kernel(const __grid_constant__ ScanParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ long long sh_warp[32];
  __shared__ long long sh_info[8];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long cap = static_cast<long long>(p.max_blocks) * p.bs;
  const uint32_t ring = smem_u32(smem);
  const uint32_t bars = ring + p.nstages * p.stage_bytes;
  // full_k[s] = bars + 8 s, full_v[s] = bars + 8 (ns + s), empty[s] = bars + 8 (2 ns + s)
  const uint32_t ns8 = 8u * p.nstages;

  // The merge kernel queued behind this one (programmatic dependent launch)
  // may start now; it waits for this grid's results itself.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nstages; ++s) {
      mbar_init(bars + 8 * s, 1);
      mbar_init(bars + ns8 + 8 * s, 1);
      mbar_init(bars + 2 * ns8 + 8 * s, p.ncw);
    }
    fence_mbar_init();
  }

  if (p.schedule == kBalanced && p.plan) {
    if (threadIdx.x < 4) {
      const long long* e = p.plan + kPlanHeader + static_cast<size_t>(blockIdx.x) * kPlanEntry;
      sh_info[threadIdx.x < 2 ? threadIdx.x : threadIdx.x + 1] = e[threadIdx.x];
    } else if (threadIdx.x == 4) {
      sh_info[2] = p.plan[1];
    } else if (threadIdx.x == 5) {
      sh_info[5] = p.plan[0];
    }
    __syncthreads();
  } else if (p.schedule == kBalanced) {
    balanced_start(p, cap, sh_warp, sh_info);  // contains __syncthreads
  } else {
    __syncthreads();
  }

  SegIter it;
  if (p.schedule == kFixed) {
    it.task = blockIdx.x;
    it.task_step = gridDim.x;
    it.task_end = p.B * p.NHG * p.num_splits;
  } else {
    it.g = sh_info[0];
    it.g_end = sh_info[1];
    it.E = sh_info[2];
    it.T = sh_info[5];
    it.b = static_cast<int>(sh_info[3]);
    it.row0 = sh_info[4] * p.NHG;
    it.hg = 0;
    it.S = it.g < it.g_end ? req_len(p, it.b, cap) : 0;
    it.L = (it.S + kStageTokens - 1) / kStageTokens;
  }

  if (warp == p.ncw) {
    // ------------------------------ producer ------------------------------
    const int i = lane & 15;
    const bool is_v = lane >= 16;
    const unsigned char* base =
        reinterpret_cast<const unsigned char*>(is_v ? p.v : p.k);
    const uint64_t pol = policy_evict_first();
    const uint32_t tx = static_cast<uint32_t>(kStageTokens * p.row_bytes);
    const uint32_t half = static_cast<uint32_t>(kStageTokens * p.row_stride);
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    Seg s;
    if (p.selftest_no_copies) ok = false;  // self-test: nothing arrives in the ring
    while (ok && iter_next(it, p, cap, s)) {
      if (s.kind == kZero) continue;
      const int* bt_row = page_row(p, s.b);
      const size_t head_off = static_cast<size_t>(s.hg) * p.HG;
      for (int st = s.s0; st < s.s1; ++st) {
        const int tok0 = st * kStageTokens;
        const int nvalid = min(kStageTokens, s.S - tok0);
        // Slots past the end of the request re-read the stage's first token
        // (always valid); its scores are masked, and the copy keeps every
        // shared-memory row finite.
        const int tok = tok0 + (i < nvalid ? i : 0);
        const int lb = tok / p.bs;
        const int sl = tok - lb * p.bs;
        int page = __ldg(bt_row + lb);
        if (p.num_blocks > 0 && static_cast<unsigned>(page) >= static_cast<unsigned>(p.num_blocks)) {
          raise_status(kStatusBadPage);
          page = 0;
        }
        const unsigned char* src =
            base + ((static_cast<size_t>(page) * p.bs + sl) * p.Hkv + head_off) * (kHeadDim * 2);
        // Warp-uniform outcome: every lane polls, all must have seen the phase.
        if (!__all_sync(kFull, mbar_wait(bars + 2 * ns8 + 8 * stage, phase ^ 1, p.wait_ns))) {
          raise_status(kStatusWaitTimeout);
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(bars + 8 * stage, tx);
          mbar_arrive_expect_tx(bars + ns8 + 8 * stage, tx);
        }
        __syncwarp();
        const uint32_t dst = ring + stage * p.stage_bytes + (is_v ? half : 0u) + i * p.row_stride;
        bulk_g2s(dst, src, p.row_bytes, bars + (is_v ? ns8 : 0u) + 8 * stage, pol);
        ++issued;
        if (++stage == p.nstages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // Wait (bounded) for this CTA's copies that may still be in flight - at
    // most the last nstages issued - so none lands in shared memory after the
    // CTA has exited.  Normally the consumers have already waited for them;
    // not when a consumer warp gave up on a wait and skipped its remaining
    // stages, or when this warp abandoned the pipeline.  No further phase of
    // these barriers completes, so each wait sees its own phase.
    const long long inflight = min(issued, static_cast<long long>(p.nstages));
    for (long long j = 1; j <= inflight; ++j) {
      const long long idx = issued - j;
      const int stg = static_cast<int>(idx % p.nstages);
      const uint32_t ph = static_cast<uint32_t>((idx / p.nstages) & 1);
      mbar_wait(bars + 8 * stg, ph);
      mbar_wait(bars + ns8 + 8 * stg, ph);
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int hl = warp / p.NT;
  const int qt = warp - hl * p.NT;
  const int j0 = qt * 8;
  const int cnt = min(8, p.G - j0);
  const int g = lane >> 2, tig = lane & 3;
  // ldmatrix row addresses: K (A operand, tokens x d, row-major) and V
  // (A operand of V^T, read transposed).
  const uint32_t k_off = static_cast<uint32_t>(((lane & 7) + ((lane >> 3) & 1) * 8) * p.row_stride +
                                               hl * 256 + (lane >> 4) * 16);
  const uint32_t v_off = static_cast<uint32_t>(((lane & 7) + (lane >> 4) * 8) * p.row_stride +
                                               hl * 256 + ((lane >> 3) & 1) * 16);
  const uint32_t half = static_cast<uint32_t>(kStageTokens * p.row_stride);

  if (p.schedule == kBalanced) {
    // Requests without tokens occupy no stages; CTA (b mod grid) writes them
    // and records their rows as having no parts.
    for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
      if (req_len(p, b, cap) != 0) continue;
      for (int hg = 0; hg < p.NHG; ++hg) {
        write_empty(p, b, (hg * p.HG + hl) * p.G + j0, cnt, lane);
        if (warp == 0 && lane == 0) p.row_info[b * p.NHG + hg] = make_int2(0, 0);
      }
    }
  }

  int stage = 0;
  uint32_t phase = 0;
  // Set when one of this warp's pipeline waits timed out.  The warp then
  // stops reading the ring but still walks its segments, writing an empty
  // state (m = -inf, l = 0, acc = 0) for each, so the merge kernel finds every
  // part and every row record it expects (and the peers every state) exactly
  // as after a normal launch; only the rows this warp held are wrong (status
  // bit 0 says so).
  bool dead = false;
  bool first_seg = true;
  // No cut row ends in this CTA unless its first segment is a row's last part.
  if (p.schedule == kBalanced && warp == 0 && lane == 0) p.ends[blockIdx.x] = make_int2(-1, 0);
  Seg s;
  while (iter_next(it, p, cap, s)) {
    const int hk = s.hg * p.HG + hl;
    const int hbase = hk * p.G + j0;
    if (first_seg && p.schedule == kBalanced && warp == 0 && lane == 0 && s.kind == kPartial &&
        s.s1 == (s.S + kStageTokens - 1) / kStageTokens)
      p.ends[blockIdx.x] = make_int2(s.row, s.nparts);
    first_seg = false;
    if (s.kind == kZero) {
      write_empty(p, s.b, hbase, cnt, lane);
      continue;
    }
    // The CTA holding a row's first stage records where the row's parts are
    // (BALANCED: slots cfirst + row, ... in consecutive CTAs).
    if (p.schedule == kBalanced && s.s0 == 0 && warp == 0 && lane == 0)
      p.row_info[s.row] = make_int2(static_cast<int>(s.cfirst), s.nparts);
    uint32_t qf[8][2];
    {
      const bool has = g < cnt;
      const __nv_bfloat16* qrow =
          p.q + (static_cast<size_t>(s.b) * p.Hq + hbase + (has ? g : 0)) * kHeadDim + 2 * tig;
      #pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qf[ks][0] = has ? __ldg(reinterpret_cast<const unsigned*>(qrow + ks * 16)) : 0u;
        qf[ks][1] = has ? __ldg(reinterpret_cast<const unsigned*>(qrow + ks * 16 + 8)) : 0u;
      }
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float acc[8][4];
    #pragma unroll
    for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;

    for (int st = s.s0; st < s.s1 && !dead; ++st) {
      const int nvalid = min(kStageTokens, s.S - st * kStageTokens);
      const uint32_t kb = ring + stage * p.stage_bytes;
      if (!__all_sync(kFull, mbar_wait(bars + 8 * stage, phase, p.wait_ns))) {
        dead = true;
        break;
      }
      // S^T = K q^T, two independent accumulation chains over d.
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
      #pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kb + k_off + ks * 32, a0, a1, a2, a3);
        mma_bf16_16816(c0, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
        ldsm_x4(kb + k_off + (ks + 1) * 32, a0, a1, a2, a3);
        mma_bf16_16816(c1, a0, a1, a2, a3, qf[ks + 1][0], qf[ks + 1][1]);
      }
      // Lane holds tokens g (s0, s1) and g + 8 (s2, s3), heads 2 tig (+1).
      float sc0 = (c0[0] + c1[0]) * p.scale_log2;
      float sc1 = (c0[1] + c1[1]) * p.scale_log2;
      float sc2 = (c0[2] + c1[2]) * p.scale_log2;
      float sc3 = (c0[3] + c1[3]) * p.scale_log2;
      if (g >= nvalid) sc0 = sc1 = -INFINITY;
      if (g + 8 >= nvalid) sc2 = sc3 = -INFINITY;
      float mx0 = fmaxf(sc0, sc2), mx1 = fmaxf(sc1, sc3);
      #pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
      const float p0 = exp2f(sc0 - mn0), p1 = exp2f(sc1 - mn1);
      const float p2 = exp2f(sc2 - mn0), p3 = exp2f(sc3 - mn1);
      l0 = l0 * al0 + (p0 + p2);
      l1 = l1 * al1 + (p1 + p3);
      m0 = mn0;
      m1 = mn1;
      #pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        acc[mt][0] *= al0;
        acc[mt][1] *= al1;
        acc[mt][2] *= al0;
        acc[mt][3] *= al1;
      }
      // P^T as the B operand: (tokens 2 tig.., head g) from (token g, heads 2 tig..).
      const uint32_t pb0 = movmatrix_trans(pack_bf16x2(p0, p1));
      const uint32_t pb1 = movmatrix_trans(pack_bf16x2(p2, p3));
      if (!__all_sync(kFull, mbar_wait(bars + ns8 + 8 * stage, phase, p.wait_ns))) {
        dead = true;
        break;
      }
      const uint32_t vb = kb + half;
      #pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(vb + v_off + mt * 32, a0, a1, a2, a3);
        mma_bf16_16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + 2 * ns8 + 8 * stage);
      if (++stage == p.nstages) {
        stage = 0;
        phase ^= 1;
      }
    }

    if (dead) {
      if (lane == 0) raise_status(kStatusWaitTimeout);
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
      #pragma unroll
      for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    }

    // ---- segment epilogue ----
    #pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(kFull, l0, off);
      l1 += __shfl_xor_sync(kFull, l1, off);
    }
    const int n0 = 2 * tig, n1 = 2 * tig + 1;
    if (s.kind == kDirect && p.out_mode == kOutBf16) {
      #pragma unroll
      for (int n = 0; n < 2; ++n) {
        const int head = n ? n1 : n0;
        if (head >= cnt) continue;
        const float l = n ? l1 : l0;
        __nv_bfloat16* o = p.out + (static_cast<size_t>(s.b) * p.Hq + hbase + head) * kHeadDim;
        #pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[mt * 16 + g] = __float2bfloat16(acc[mt][n] / l);
          o[mt * 16 + g + 8] = __float2bfloat16(acc[mt][2 + n] / l);
        }
      }
      continue;
    }
    // Unnormalised state: the CTA's partial slot (also a whole row's state
    // with kOutExchange, which the merge kernel sends to the peers), or
    // (kOutState) the request's final shard state.
    float* dm;
    float* dl;
    float* da;
    size_t idx0, idx1;
    if (s.kind == kDirect && p.out_mode == kOutState) {
      dm = p.res_m;
      dl = p.res_l;
      da = p.res_acc;
      idx0 = static_cast<size_t>(s.b) * p.Hq + hbase + n0;
      idx1 = idx0 + 1;
    } else {
      dm = p.part_m;
      dl = p.part_l;
      da = p.part_acc;
      if (p.schedule == kFixed) {
        idx0 = (static_cast<size_t>(s.b) * p.Hq + hbase + n0) * p.num_splits + s.slot;
        idx1 = idx0 + p.num_splits;
      } else {
        idx0 = static_cast<size_t>(s.slot) * (p.HG * p.G) + hl * p.G + j0 + n0;
        idx1 = idx0 + 1;
      }
    }
    #pragma unroll
    for (int n = 0; n < 2; ++n) {
      const int head = n ? n1 : n0;
      if (head >= cnt) continue;
      const size_t idx = n ? idx1 : idx0;
      if (g == 0) {
        dm[idx] = n ? m1 : m0;
        dl[idx] = n ? l1 : l0;
      }
      float* a = da + idx * kHeadDim;
      #pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        a[mt * 16 + g] = acc[mt][n];
        a[mt * 16 + g + 8] = acc[mt][2 + n];
      }
    }
  }
}

// Merge for the FIXED schedule (reference workspace layout), one warp per
// (b, q head), lane = 4 output dims.  Rows whose work fit in one split were
// finished by the scan and are skipped.  Lanes read the (m, l) of 32 splits
// at once; acc rows are read 4 splits per batch so the loads overlap.
__global__ void __launch_bounds__(128) gqa_decode_fixed_merge_kernel(const MergeParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long bh = static_cast<long long>(blockIdx.x) * 4 + warp;
  if (bh >= static_cast<long long>(p.B) * p.Hq) return;
  const int b = static_cast<int>(bh / p.Hq);
  const long long cap = static_cast<long long>(p.max_blocks) * p.bs;
  const int S = eff_len(p.seq_lens, b, cap);
  const int L = (S + kStageTokens - 1) / kStageTokens;
  if (L == 0) return;
  const int chunk = (L + p.num_splits - 1) / p.num_splits;
  const int n = (L + chunk - 1) / chunk;
  if (n <= 1) return;
  const size_t base = static_cast<size_t>(bh) * p.num_splits;
  float M = -INFINITY;
  for (int c0 = 0; c0 < n; c0 += 32) {
    const int kc = min(c0 + lane, n - 1);  // in range on every lane
    float mk = c0 + lane < n ? __ldcg(p.part_m + base + kc) : -INFINITY;
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) mk = fmaxf(mk, __shfl_xor_sync(kFull, mk, off));
    M = fmaxf(M, mk);
  }
  float Lsum = 0.f;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c0 = 0; c0 < n; c0 += 32) {
    const bool in = c0 + lane < n;
    const int kc = min(c0 + lane, n - 1);
    const float w = in ? exp2f(__ldcg(p.part_m + base + kc) - M) : 0.f;
    float lw = in ? __ldcg(p.part_l + base + kc) * w : 0.f;
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) lw += __shfl_xor_sync(kFull, lw, off);
    Lsum += lw;
    const int nc = min(32, n - c0);
    for (int k0 = 0; k0 < nc; k0 += 4) {
      float4 x[4];
      #pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        x[kk] = k0 + kk < nc
                    ? __ldcg(reinterpret_cast<const float4*>(
                                 p.part_acc + (base + c0 + min(k0 + kk, nc - 1)) * kHeadDim) +
                             lane)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      #pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float f = __shfl_sync(kFull, w, (k0 + kk) & 31);
        a.x += x[kk].x * f;
        a.y += x[kk].y * f;
        a.z += x[kk].z * f;
        a.w += x[kk].w * f;
      }
    }
  }
  store_bf16x4(p.out + static_cast<size_t>(bh) * kHeadDim + 4 * lane, a.x / Lsum, a.y / Lsum,
               a.z / Lsum, a.w / Lsum);
}

// Merge of per-shard states (KV range split across GPUs): state i of row r
// at [i * rows + r].  A shard with no tokens holds m = -inf, l = 0.
__global__ void __launch_bounds__(128) gqa_decode_shard_merge_kernel(const ShardMergeParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r = static_cast<long long>(blockIdx.x) * 4 + warp;
  if (r >= p.rows) return;
  float M = -INFINITY;
  for (int i = 0; i < p.nshards; ++i) M = fmaxf(M, p.m[static_cast<size_t>(i) * p.rows + r]);
  __nv_bfloat16* o = p.out + static_cast<size_t>(r) * kHeadDim + 4 * lane;
  if (M == -INFINITY) {
    store_bf16x4(o, 0.f, 0.f, 0.f, 0.f);
    return;
  }
  float Lsum = 0.f;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 0; i < p.nshards; ++i) {
    const size_t st = static_cast<size_t>(i) * p.rows + r;
    const float f = exp2f(p.m[st] - M);
    Lsum += p.l[st] * f;
    const float4 x = reinterpret_cast<const float4*>(p.acc + st * kHeadDim)[lane];
    a.x += x.x * f;
    a.y += x.y * f;
    a.z += x.z * f;
    a.w += x.w * f;
  }
  store_bf16x4(o, a.x / Lsum, a.y / Lsum, a.z / Lsum, a.w / Lsum);
}

constexpr int kSmallWarps = 9;
constexpr int kLargeWarps = kMaxConsumerWarps + 1;

cudaError_t launch_scan(const ScanParams& p, int grid, int threads, int smem, cudaStream_t s) {
  if (threads <= kSmallWarps * 32)
    gqa_decode_scan_kernel<kSmallWarps><<<grid, threads, smem, s>>>(p);
  else
    gqa_decode_scan_kernel<kLargeWarps><<<grid, threads, smem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_fixed_merge(const MergeParams& p, cudaStream_t s) {
  const long long rows = static_cast<long long>(p.B) * p.Hq;
  const int grid = static_cast<int>((rows + 3) / 4);
  gqa_decode_fixed_merge_kernel<<<grid, 128, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_shard_merge(const ShardMergeParams& p, cudaStream_t s) {
  const int grid = (p.rows + 3) / 4;
  gqa_decode_shard_merge_kernel<<<grid, 128, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t scan_kernel_set_smem(int smem_bytes) {
  cudaError_t e = cudaFuncSetAttribute(gqa_decode_scan_kernel<kSmallWarps>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gqa_decode_scan_kernel<kLargeWarps>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
}

cudaError_t scan_kernel_occupancy(int threads, int smem_bytes, int* blocks_per_sm) {
  if (threads <= kSmallWarps * 32)
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        blocks_per_sm, gqa_decode_scan_kernel<kSmallWarps>, threads, smem_bytes);
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      blocks_per_sm, gqa_decode_scan_kernel<kLargeWarps>, threads, smem_bytes);
}

// Self-test of the bounded wait: one warp waits on an mbarrier phase that
// nothing completes.  The wait must give up after limit_ns and report
// kStatusWaitTimeout through the device status word, exactly as a stuck
// pipeline in the scan kernel would, instead of hanging the GPU.
__global__ void __launch_bounds__(32) gqa_decode_wait_selftest_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) unsigned long long bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (!__all_sync(kFull, mbar_wait(b, 0, limit_ns)) && threadIdx.x == 0)
    raise_status(kStatusWaitTimeout);
}

cudaError_t launch_wait_selftest(unsigned long long limit_ns, cudaStream_t s) {
  gqa_decode_wait_selftest_kernel<<<1, 32, 0, s>>>(limit_ns);
  return cudaGetLastError();
}

// Block-wide inclusive scan of one int64 per thread (blockDim.x <= 1024).
__device__ long long block_inclusive_scan(long long x, long long* sh_warp, long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  #pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const long long y = __shfl_up_sync(kFull, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) sh_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    long long t = lane < nwarps ? sh_warp[lane] : 0;
    #pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(kFull, t, off);
      if (lane >= off) t += y;
    }
    if (lane < nwarps) sh_warp[lane] = t;
  }
  __syncthreads();
  const long long r = x + (warp > 0 ? sh_warp[warp - 1] : 0);
  *total = sh_warp[nwarps - 1];
  __syncthreads();
  return r;
}

// One CTA: stage prefix over the requests, then every CTA's range of the
// BALANCED schedule - the same cut balanced_start computes inside the scan.
__global__ void __launch_bounds__(1024)
    gqa_decode_plan_kernel(const __grid_constant__ ScanParams p, long long* plan, long long* prefix,
                           int grid) {
  __shared__ long long sh_warp[32];
  const long long cap = static_cast<long long>(p.max_blocks) * p.bs;
  long long carry = 0;
  if (threadIdx.x == 0) prefix[0] = 0;
  for (int b0 = 0; b0 < p.B; b0 += blockDim.x) {
    const int b = b0 + threadIdx.x;
    const long long L = b < p.B ? (req_len(p, b, cap) + kStageTokens - 1) / kStageTokens : 0;
    long long total;
    const long long incl = block_inclusive_scan(L, sh_warp, &total);
    if (b < p.B) prefix[b + 1] = carry + incl;
    carry += total;
  }
  __syncthreads();
  const long long T = carry * p.NHG;
  const long long E = range_parts(T, grid);
  if (threadIdx.x == 0) {
    plan[0] = T;
    plan[1] = E;
    plan[2] = grid;
  }
  for (int c = threadIdx.x; c < grid; c += blockDim.x) {
    const long long g0 = range_start(c, T, E);
    const long long g1 = range_start(c + 1LL, T, E);
    int b0 = 0;
    if (g0 < g1) {
      // last request whose stages start at or before g0 (an empty request
      // never qualifies: the next one starts at the same stage)
      int lo = 0, hi = p.B - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] * p.NHG <= g0) lo = mid; else hi = mid - 1;
      }
      b0 = lo;
    }
    long long* e = plan + kPlanHeader + static_cast<size_t>(c) * kPlanEntry;
    e[0] = g0;
    e[1] = g1;
    e[2] = b0;
    e[3] = prefix[b0];
  }
}

// One CTA: block_table [B, max_blocks] + seq_lens -> CSR, with the reference
// helper's arithmetic (bench/baselines/flashinfer_adapter.py:33-51):
// n = ceil(S / page), indptr = prefix of n, indices = the first n ids of each
// row, last_page_len = S - (n - 1) * page.
__global__ void __launch_bounds__(1024) gqa_decode_block_table_to_csr_kernel(
    const int* block_table, const int* seq_lens, int B, int max_blocks, int page, int* indptr,
    int* indices, int* last_page_len) {
  __shared__ long long sh_warp[32];
  long long carry = 0;
  if (threadIdx.x == 0) indptr[0] = 0;
  for (int b0 = 0; b0 < B; b0 += blockDim.x) {
    const int b = b0 + threadIdx.x;
    long long n = 0;
    if (b < B) {
      const long long S = seq_lens[b];
      const long long nb = (S + page - 1) / page;
      last_page_len[b] = static_cast<int>(S - (nb - 1) * page);
      n = nb < 0 ? 0 : (nb > max_blocks ? max_blocks : nb);
    }
    long long total;
    const long long incl = block_inclusive_scan(n, sh_warp, &total);
    if (b < B) indptr[b + 1] = static_cast<int>(carry + incl);
    carry += total;
  }
  __syncthreads();
  for (int b = 0; b < B; ++b) {
    const int start = indptr[b];
    const int n = indptr[b + 1] - start;
    for (int j = threadIdx.x; j < n; j += blockDim.x)
      indices[start + j] = block_table[static_cast<size_t>(b) * max_blocks + j];
  }
}

cudaError_t launch_plan(const ScanParams& p, long long* plan, long long* prefix, int grid,
                        cudaStream_t s) {
  gqa_decode_plan_kernel<<<1, 1024, 0, s>>>(p, plan, prefix, grid);
  return cudaGetLastError();
}

cudaError_t launch_block_table_to_csr(const int* block_table, const int* seq_lens, int B,
                                      int max_blocks, int page_size, int* indptr, int* indices,
                                      int* last_page_len, cudaStream_t s) {
  gqa_decode_block_table_to_csr_kernel<<<1, 1024, 0, s>>>(block_table, seq_lens, B, max_blocks,
                                                          page_size, indptr, indices,
                                                          last_page_len);
  return cudaGetLastError();
}

cudaError_t read_status(int* status, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_status, sizeof(int));
  if (e != cudaSuccess || !clear) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
}

}  // namespace gqa

#include "gqa_merge.cuh"
