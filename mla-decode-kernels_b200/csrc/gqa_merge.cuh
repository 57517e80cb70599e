// Merge of the rows the BALANCED scan cut between CTAs, and the cross-rank
// exchange of the KV-range sharded decode.
//
// The scan writes every cut row's partial softmax states into consecutive
// slots (cfirst + row, cfirst + 1 + row, ... - one per CTA holding a part),
// per CTA the record {row, parts} of the cut row whose last part it holds,
// and per row the record {cfirst, parts}.  This kernel is launched right
// behind it with programmatic dependent launch: the scan lets it start at
// once, so its CTAs take each SM as the scan's CTA there leaves (the two do
// not fit on one SM together) and begin the moment the scan's last CTA has
// written its state (griddepcontrol.wait), instead of the last CTA of a row
// merging the row's parts on one SM after its own stream.
// The work is spread over every SM in items of one L2 round trip each:
//   * a row cut into at most 16 parts: one warp per (row, q head), lane = 4
//     output dims, the parts' (m, l) and acc rows all loaded at once;
//   * a row cut into more parts (one long request over every SM): one CTA
//     per (row, q head, 32-dim chunk), its 8 warps taking an eighth of the
//     parts each (lane = one dim: coalesced 128-byte loads), combined
//     through shared memory.
// Merge identity (kernels/gqa_decode/v2_splitkv.cu:97-107 of the reference),
// in log2 units: M = max m_i, w_i = 2^(m_i - M), out = sum w_i acc_i /
// sum w_i l_i.  Parts are combined in a fixed order, so results are
// deterministic.
//
// KV-range sharding over peer memory (kOutExchange): every row, cut or not,
// is merged here per (row, q head, 32-dim chunk) - the same items on every
// rank - and each item's local state is stored with plain peer stores into
// slot `rank` of every rank's exchange buffer as 64-bit words tagged with
// the decode's epoch, then merged with the other ranks' states once every
// word it needs carries the epoch (bounded wait).  Buffers are
// double-buffered by epoch parity: a rank can only run one decode ahead of a
// peer.
//
// Included once, at the end of gqa_scan.cu, so that it shares that
// translation unit's device status word and helpers (raise_status, kFull).
#pragma once

namespace gqa {

namespace merge_detail {

constexpr int kThreads = 256;           // 8 warps per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 32;              // dims of a chunk item (lane = dim)
constexpr int kChunks = kHeadDim / kChunk;
constexpr int kFewParts = 16;           // up to this many parts: one warp per q head
constexpr int kBatch = 24;              // parts a warp loads per batch (chunk items)

__device__ __forceinline__ float warp_max(float v) {
  #pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, off));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
  #pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
  return v;
}

__device__ __forceinline__ uint2 pack_bf16x4(float a, float b, float c, float d) {
  uint2 v;
  v.x = pack_bf16x2(a, b);
  v.y = pack_bf16x2(c, d);
  return v;
}

// Merge n <= kFewParts parts (slots base, base + 1, ...) of q head j (of QHR
// per row) in one warp, lane = output dims 4 lane .. 4 lane + 3, every load
// in flight at once; writes the bf16 output or the unnormalised state of
// head bh.
__device__ __forceinline__ void merge_head(const CutMergeParams& p, long long base, int n, int j,
                                           size_t bh, int lane) {
  const size_t sl = static_cast<size_t>(base + min(lane, n - 1)) * p.QHR + j;
  const float mk = lane < n ? __ldcg(p.part_m + sl) : -INFINITY;
  const float lk = lane < n ? __ldcg(p.part_l + sl) : 0.f;
  float4 x[kFewParts];
  #pragma unroll
  for (int k = 0; k < kFewParts; ++k) {
    const size_t st = static_cast<size_t>(base + min(k, n - 1)) * p.QHR + j;
    x[k] = k < n ? __ldcg(reinterpret_cast<const float4*>(p.part_acc + st * kHeadDim) + lane)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float M = warp_max(mk);
  const float w = (lane < n && M != -INFINITY) ? exp2f(mk - M) : 0.f;
  const float L = warp_sum(lk * w);
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  #pragma unroll
  for (int k = 0; k < kFewParts; ++k) {
    const float f = __shfl_sync(kFull, w, k);  // 0 for k >= n
    a.x += x[k].x * f;
    a.y += x[k].y * f;
    a.z += x[k].z * f;
    a.w += x[k].w * f;
  }
  if (p.out_mode == kOutState) {
    if (lane == 0) {
      p.res_m[bh] = M;
      p.res_l[bh] = L;
    }
    *reinterpret_cast<float4*>(p.res_acc + bh * kHeadDim + 4 * lane) = a;
  } else {
    *reinterpret_cast<uint2*>(p.out + bh * kHeadDim + 4 * lane) =
        pack_bf16x4(a.x / L, a.y / L, a.z / L, a.w / L);
  }
}

// Shared memory of the CTA-wide chunk merge: each warp's (m, l) and acc.
struct ChunkSmem {
  float m[kWarps], l[kWarps];
  float a[kWarps][kChunk];
};

// Merge n parts of q head j, dims [32 c, 32 c + 32), with the whole CTA:
// warp w takes parts [w n / 8, (w + 1) n / 8), lane = one dim, so each
// part's 32 dims are one coalesced 128-byte load and its (m, l) a broadcast
// load; up to kBatch parts per warp are in flight at once, merged online in
// registers, and the warps' states are combined through shared memory.  The
// result (m, l, acc of lane's dim) is valid in warp 0; n = 0 gives the
// neutral state.  Every thread of the CTA must call it.
__device__ __forceinline__ void merge_chunk(const CutMergeParams& p, long long base, int n, int j,
                                            int c, ChunkSmem& cs, float& Mo, float& Lo,
                                            float& Ao) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k0 = static_cast<int>(static_cast<long long>(warp) * n / kWarps);
  const int k1 = static_cast<int>(static_cast<long long>(warp + 1) * n / kWarps);
  float M = -INFINITY, L = 0.f, A = 0.f;
  for (int b0 = k0; b0 < k1; b0 += kBatch) {
    float m[kBatch], l[kBatch], x[kBatch];
    #pragma unroll
    for (int t = 0; t < kBatch; ++t) {
      const int k = b0 + t;
      const size_t st = static_cast<size_t>(base + min(k, k1 - 1)) * p.QHR + j;  // valid address
      m[t] = k < k1 ? __ldcg(p.part_m + st) : -INFINITY;
      l[t] = k < k1 ? __ldcg(p.part_l + st) : 0.f;
      x[t] = k < k1 ? __ldcg(p.part_acc + st * kHeadDim + kChunk * c + lane) : 0.f;
    }
    float mb = M;
    #pragma unroll
    for (int t = 0; t < kBatch; ++t) mb = fmaxf(mb, m[t]);
    if (mb == -INFINITY) continue;  // warp-uniform: every lane read the same m
    const float sc = M == -INFINITY ? 0.f : exp2f(M - mb);
    L *= sc;
    A *= sc;
    #pragma unroll
    for (int t = 0; t < kBatch; ++t) {
      const float w = m[t] == -INFINITY ? 0.f : exp2f(m[t] - mb);
      L += l[t] * w;
      A += x[t] * w;
    }
    M = mb;
  }
  if (lane == 0) {
    cs.m[warp] = M;
    cs.l[warp] = L;
  }
  cs.a[warp][lane] = A;
  __syncthreads();
  if (warp == 0) {
    float Mc = -INFINITY;
    #pragma unroll
    for (int w = 0; w < kWarps; ++w) Mc = fmaxf(Mc, cs.m[w]);
    float Lc = 0.f, Ac = 0.f;
    #pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = cs.m[w] == -INFINITY ? 0.f : exp2f(cs.m[w] - Mc);
      Lc += cs.l[w] * f;
      Ac += cs.a[w][lane] * f;
    }
    Mo = Mc;
    Lo = Lc;
    Ao = Ac;
  }
  __syncthreads();  // cs is reused by the next item
}

// Exchange buffer: u64 words [2][world][items][kXItem], [2] the epoch
// parity, item = (b * Hq + q head) * kXSlices + chunk; an item's words are
// {m, l, acc[32], -, -}, each the float's bits in the low half and the
// decode's epoch in the high half.
__device__ __forceinline__ unsigned long long* xitem(const CutMergeParams& p, int owner, int src,
                                                     size_t item) {
  return reinterpret_cast<unsigned long long*>(p.xpeer[owner]) +
         (static_cast<size_t>((p.xepoch & 1) * p.xworld + src) * p.xitems + item) * kXItem;
}

__device__ __forceinline__ unsigned long long tag_word(unsigned epoch, float v) {
  return (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
}

// Warp 0: send this rank's state of `item` (lane = one of its 32 dims) to
// every rank, wait for every rank's, merge and write out's 32 dims.  Every
// word carries the epoch, so each lane just polls the words it needs (its
// dim's acc and the (m, l) of every rank) until all carry this decode's
// epoch: no fence and no separate flag, one NVLink latency per exchange.
__device__ __forceinline__ void exchange_chunk(const CutMergeParams& p, float M, float L, float A,
                                               size_t item, size_t bh, int c, int lane) {
  for (int o = 0; o < p.xworld; ++o) {
    unsigned long long* d = xitem(p, o, p.xrank, item);
    st_relaxed_sys_u64(d + 2 + lane, tag_word(p.xepoch, A));
    if (lane < 2) st_relaxed_sys_u64(d + lane, tag_word(p.xepoch, lane == 0 ? M : L));
  }
  // Poll every rank's words at once (all loads of a round in flight), again
  // for the ranks not yet arrived, until all carry this decode's epoch.
  float m[kMaxPeers], l[kMaxPeers], a[kMaxPeers];
  unsigned pending = (1u << p.xworld) - 1u;
  bool ok = true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    unsigned long long wm[kMaxPeers], wl[kMaxPeers], wa[kMaxPeers];
    #pragma unroll
    for (int o = 0; o < kMaxPeers; ++o) {
      if ((pending >> o) & 1u) {
        const unsigned long long* d = xitem(p, p.xrank, o, item);
        wm[o] = ld_relaxed_sys_u64(d);
        wl[o] = ld_relaxed_sys_u64(d + 1);
        wa[o] = ld_relaxed_sys_u64(d + 2 + lane);
      }
    }
    #pragma unroll
    for (int o = 0; o < kMaxPeers; ++o) {
      if (((pending >> o) & 1u) && static_cast<unsigned>(wm[o] >> 32) == p.xepoch &&
          static_cast<unsigned>(wl[o] >> 32) == p.xepoch &&
          static_cast<unsigned>(wa[o] >> 32) == p.xepoch) {
        m[o] = __uint_as_float(static_cast<unsigned>(wm[o]));
        l[o] = __uint_as_float(static_cast<unsigned>(wl[o]));
        a[o] = __uint_as_float(static_cast<unsigned>(wa[o]));
        pending &= ~(1u << o);
      }
    }
    if (pending == 0u) break;
    if (global_timer_ns() - t0 > p.wait_ns) {
      ok = false;
      break;
    }
  }
  #pragma unroll
  for (int o = 0; o < kMaxPeers; ++o) {
    if (o >= p.xworld) {
      m[o] = -INFINITY;
      l[o] = 0.f;
      a[o] = 0.f;
    }
  }
  if (!__all_sync(kFull, ok)) {
    if (lane == 0) raise_status(kStatusPeerTimeout);
    return;
  }
  float Mx = -INFINITY;
  #pragma unroll
  for (int o = 0; o < kMaxPeers; ++o) Mx = fmaxf(Mx, m[o]);
  float Lx = 0.f, Ax = 0.f;
  #pragma unroll
  for (int o = 0; o < kMaxPeers; ++o) {
    const float w = m[o] == -INFINITY ? 0.f : exp2f(m[o] - Mx);
    Lx += l[o] * w;
    Ax += a[o] * w;
  }
  // no tokens on any rank: 0, as python/reference.py gives
  p.out[bh * kHeadDim + kChunk * c + lane] =
      __float2bfloat16(Mx == -INFINITY ? 0.f : Ax / Lx);
}

// kOutExchange: every row, cut or not, is QHR x 4 chunk units, unit u
// handled by CTA u mod ncta (the same units on every rank).
__device__ __forceinline__ void exchange_units(const CutMergeParams& p, int cta, int ncta,
                                               ChunkSmem& cs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long units = static_cast<long long>(p.rows) * p.QHR * kChunks;
  for (long long u = cta; u < units; u += ncta) {
    const long long rh = u / kChunks;  // = b * Hq + q head
    const int c = static_cast<int>(u - rh * kChunks);
    const int r = static_cast<int>(rh / p.QHR);
    const int j = static_cast<int>(rh - static_cast<long long>(r) * p.QHR);
    const int2 ri = p.row_info[r];  // {first CTA, parts}
    float M = 0.f, L = 0.f, A = 0.f;
    merge_chunk(p, static_cast<long long>(ri.x) + r, ri.y, j, c, cs, M, L, A);
    if (warp == 0) exchange_chunk(p, M, L, A, static_cast<size_t>(u),
                                  static_cast<size_t>(rh), c, lane);
  }
}

}  // namespace merge_detail

// Every CTA first compacts, in shared memory, the list of cut rows from the
// scan's per-CTA records (CTA c ends at most one cut row: only its first
// segment can be a row's last part) with each row's number of work units -
// ceil(QHR / 8) units of 8 q heads (one warp each) for rows of at most
// kFewParts parts, else QHR x 4 units of one (q head, 32-dim chunk) merged by
// the whole CTA - and their prefix; then the CTAs stride over the units.
// With kOutExchange every row, cut or not, is QHR x 4 chunk units (the same
// on every rank) read from the per-row records; a CTA handles the same units
// on every rank (the grid is the same), always sending a unit before waiting
// for it.
__global__ void __launch_bounds__(merge_detail::kThreads, 1)
    gqa_decode_cut_merge_kernel(const __grid_constant__ CutMergeParams p) {
  using namespace merge_detail;
  extern __shared__ int sh[];  // [grid] rows | [grid] parts | [grid + 1] unit prefix
  __shared__ ChunkSmem cs;
  __shared__ int sh_warp[kWarps];
  // Everything below reads what the scan wrote.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  if (p.out_mode == kOutExchange) {
    exchange_units(p, blockIdx.x, gridDim.x, cs);
    return;
  }

  int* s_row = sh;
  int* s_n = sh + p.grid;
  int* s_pre = sh + 2 * p.grid;
  const int few_units = (p.QHR + kWarps - 1) / kWarps;
  // chunk of the scan's CTAs per thread, local unit sum, block scan
  const int per = (p.grid + blockDim.x - 1) / blockDim.x;
  const int c0 = min(p.grid, static_cast<int>(threadIdx.x) * per);
  const int c1 = min(p.grid, c0 + per);
  int local = 0;
  for (int c = c0; c < c1; ++c) {
    const int2 e = p.ends[c];  // {row, parts} or {-1, 0}
    const int w = e.x < 0 ? 0 : (e.y <= kFewParts ? few_units : p.QHR * kChunks);
    s_row[c] = e.x;
    s_n[c] = e.y;
    s_pre[c] = w;  // unit count for now
    local += w;
  }
  int x = local;
  #pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(kFull, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) sh_warp[warp] = x;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += sh_warp[w];
  int run = before + x - local;  // exclusive prefix of this thread's chunk
  for (int c = c0; c < c1; ++c) {
    const int w = s_pre[c];
    s_pre[c] = run;
    run += w;
  }
  if (threadIdx.x == blockDim.x - 1) s_pre[p.grid] = run;
  __syncthreads();
  const int total = s_pre[p.grid];
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    // the CTA record holding unit u: largest c with s_pre[c] <= u
    int lo = 0, hi = p.grid - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_pre[mid] <= u) lo = mid; else hi = mid - 1;
    }
    const int r = s_row[lo], n = s_n[lo];
    const long long base = static_cast<long long>(lo) - n + 1 + r;  // slot of the first part
    const int lu = u - s_pre[lo];
    if (n <= kFewParts) {
      const int j = lu * kWarps + warp;
      if (j < p.QHR) merge_head(p, base, n, j, static_cast<size_t>(r) * p.QHR + j, lane);
    } else {
      const int j = lu / kChunks, c = lu - j * kChunks;
      float M = 0.f, L = 0.f, A = 0.f;
      merge_chunk(p, base, n, j, c, cs, M, L, A);
      if (warp == 0) {
        const size_t bh = static_cast<size_t>(r) * p.QHR + j;
        if (p.out_mode == kOutState) {
          if (c == 0 && lane == 0) {
            p.res_m[bh] = M;
            p.res_l[bh] = L;
          }
          p.res_acc[bh * kHeadDim + kChunk * c + lane] = A;
        } else {
          p.out[bh * kHeadDim + kChunk * c + lane] = __float2bfloat16(A / L);
        }
      }
    }
  }
}

// Test emulation of the KV-range sharded decode on one GPU: the exchange
// merge of every rank in one grid, CTA c acting as CTA c mod per_rank of
// rank c / per_rank.  Launched cooperatively, so every CTA is resident and
// each rank's waits for the others' states end.
__global__ void __launch_bounds__(merge_detail::kThreads, 1)
    gqa_decode_exchange_emul_kernel(const __grid_constant__ ExchangeEmulParams e) {
  using namespace merge_detail;
  __shared__ ChunkSmem cs;
  const int r = static_cast<int>(blockIdx.x) / e.per_rank;
  exchange_units(e.rank[r], static_cast<int>(blockIdx.x) - r * e.per_rank, e.per_rank, cs);
}

int exchange_emul_per_rank(int world, int sms) {
  int occ = 0;
  if (world < 1 || cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                       &occ, gqa_decode_exchange_emul_kernel, merge_detail::kThreads, 0) !=
                       cudaSuccess)
    return 0;
  return occ * sms / world;
}

cudaError_t launch_exchange_emulated(const ExchangeEmulParams& e, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(e.world * e.per_rank);
  cfg.blockDim = dim3(merge_detail::kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gqa_decode_exchange_emul_kernel, e);
}

size_t cut_merge_smem_bytes(int grid) { return (3 * static_cast<size_t>(grid) + 1) * sizeof(int); }

// Launched with programmatic stream serialization, so it may start while the
// scan still runs (the scan signals griddepcontrol.launch_dependents at its
// start) and waits for the scan's results inside.
cudaError_t launch_cut_merge(const CutMergeParams& p, int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(merge_detail::kThreads);
  cfg.dynamicSmemBytes = p.out_mode == kOutExchange ? 0 : cut_merge_smem_bytes(p.grid);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gqa_decode_cut_merge_kernel, p);
}

}  // namespace gqa
