// Merge of the rows the BALANCED scan cut between CTAs, and the cross-rank
// exchange of the KV-range sharded decode.
//
// The scan writes every cut row's partial softmax states into consecutive
// slots (cfirst + row, cfirst + 1 + row, ... - one per CTA holding a part),
// per CTA the record {row, parts} of the cut row whose last part it holds,
// and per row the record {cfirst, parts}.  This kernel is launched right
// behind it with programmatic dependent launch: the scan lets it start at
// once, so its CTAs are resident beside the scan's and begin the moment the
// scan's last CTA has written its state (griddepcontrol.wait), instead of the
// last CTA of a row merging the row's parts on one SM after its own stream.
// The work is spread over every SM in items of one L2 round trip each:
//   * a row cut into at most 16 parts: one warp per (row, q head), lane = 4
//     output dims, the parts' (m, l) and acc rows all loaded at once;
//   * a row cut into more parts (one long request over every SM): one warp
//     per (row, q head, 8-dim slice), lane = parts lane, lane + 32, ...,
//     each lane merging its parts online, then one warp reduction.
// Merge identity (kernels/gqa_decode/v2_splitkv.cu:97-107 of the reference),
// in log2 units: M = max m_i, w_i = 2^(m_i - M), out = sum w_i acc_i /
// sum w_i l_i.  Parts are combined in a fixed order, so results are
// deterministic.
//
// KV-range sharding over peer memory (kOutExchange): every row, cut or not,
// is merged here per (row, q head, 8-dim slice) - the same items on every
// rank - and each item's local state is stored with plain peer stores into
// slot `rank` of every rank's exchange buffer, published with a system-scope
// release flag per item, and merged with the other ranks' states once their
// flags arrive (bounded wait).  Buffers are double-buffered by epoch parity:
// a rank can only run one decode ahead of a peer.
//
// Included once, at the end of gqa_scan.cu, so that it shares that
// translation unit's device status word and helpers (raise_status, kFull).
#pragma once

namespace gqa {

namespace merge_detail {

constexpr int kSlices = kHeadDim / 8;   // 8-dim slices of a head
constexpr int kFewParts = 16;           // up to this many parts: one warp per head
constexpr int kPerLane = 5;             // parts a lane loads per batch (many-part rows)

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

// One slice item's merged state, identical on every lane.
struct SliceState {
  float m, l;
  float a[8];
};

// Merge n parts (slots base, base + 1, ...) of q head j (of QHR per row),
// dims [8 s, 8 s + 8), lanes over parts.  n = 0 gives the neutral state.
__device__ __forceinline__ SliceState merge_slice(const CutMergeParams& p, long long base, int n,
                                                  int j, int s, int lane) {
  float Ml = -INFINITY, Ll = 0.f;
  float a[8];
  #pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = 0.f;
  for (int k0 = 0; k0 < n; k0 += 32 * kPerLane) {
    float m[kPerLane], l[kPerLane];
    float4 x0[kPerLane], x1[kPerLane];
    #pragma unroll
    for (int t = 0; t < kPerLane; ++t) {
      const int k = k0 + lane + 32 * t;
      const size_t st = static_cast<size_t>(base + min(k, n - 1)) * p.QHR + j;  // valid address
      const float4* src = reinterpret_cast<const float4*>(p.part_acc + st * kHeadDim + 8 * s);
      m[t] = k < n ? __ldcg(p.part_m + st) : -INFINITY;
      l[t] = k < n ? __ldcg(p.part_l + st) : 0.f;
      x0[t] = k < n ? __ldcg(src) : make_float4(0.f, 0.f, 0.f, 0.f);
      x1[t] = k < n ? __ldcg(src + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mb = Ml;
    #pragma unroll
    for (int t = 0; t < kPerLane; ++t) mb = fmaxf(mb, m[t]);
    if (mb == -INFINITY) continue;  // nothing on this lane yet
    const float sc = Ml == -INFINITY ? 0.f : exp2f(Ml - mb);
    Ll *= sc;
    #pragma unroll
    for (int i = 0; i < 8; ++i) a[i] *= sc;
    #pragma unroll
    for (int t = 0; t < kPerLane; ++t) {
      const float w = m[t] == -INFINITY ? 0.f : exp2f(m[t] - mb);
      Ll += l[t] * w;
      a[0] += x0[t].x * w;
      a[1] += x0[t].y * w;
      a[2] += x0[t].z * w;
      a[3] += x0[t].w * w;
      a[4] += x1[t].x * w;
      a[5] += x1[t].y * w;
      a[6] += x1[t].z * w;
      a[7] += x1[t].w * w;
    }
    Ml = mb;
  }
  SliceState r;
  r.m = warp_max(Ml);
  const float f = (Ml == -INFINITY) ? 0.f : exp2f(Ml - r.m);
  r.l = warp_sum(Ll * f);
  #pragma unroll
  for (int i = 0; i < 8; ++i) r.a[i] = warp_sum(a[i] * f);
  return r;
}

// Merge n <= kFewParts parts of q head j, lane = output dims 4 lane .. 4 lane + 3;
// writes the bf16 output or the unnormalised state of head bh.
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

// Exchange buffer: [flags u32 [2][world][items] | states f32 [2][world][items][kXItem]],
// item = (b * Hq + q head) * kSlices + slice; a state is {m, l, -, -, acc[8]}.
__device__ __forceinline__ unsigned* xflag(const CutMergeParams& p, int owner, int src,
                                           size_t item) {
  return reinterpret_cast<unsigned*>(p.xpeer[owner]) +
         (static_cast<size_t>((p.xepoch & 1) * p.xworld + src) * p.xitems + item);
}

__device__ __forceinline__ float* xstate(const CutMergeParams& p, int owner, int src, size_t item) {
  return reinterpret_cast<float*>(p.xpeer[owner] + p.xflag_bytes) +
         (static_cast<size_t>((p.xepoch & 1) * p.xworld + src) * p.xitems + item) * kXItem;
}

// Send this rank's state of `item` to every rank, wait for every rank's,
// merge and write out's 8 dims.  Lane o handles rank o.
__device__ __forceinline__ void exchange_item(const CutMergeParams& p, const SliceState& st,
                                              size_t item, size_t bh, int s, int lane) {
  if (lane < p.xworld) {
    float* d = xstate(p, lane, p.xrank, item);
    *reinterpret_cast<float4*>(d) = make_float4(st.m, st.l, 0.f, 0.f);
    reinterpret_cast<float4*>(d)[1] = make_float4(st.a[0], st.a[1], st.a[2], st.a[3]);
    reinterpret_cast<float4*>(d)[2] = make_float4(st.a[4], st.a[5], st.a[6], st.a[7]);
  }
  __threadfence_system();
  __syncwarp();
  if (lane < p.xworld) st_release_sys(xflag(p, lane, p.xrank, item), p.xepoch);
  bool ok = true;
  if (lane < p.xworld) {
    const unsigned* f = xflag(p, p.xrank, lane, item);
    ok = ld_acquire_sys(f) == p.xepoch;
    if (!ok) {
      const unsigned long long t0 = global_timer_ns();
      while (!ok && global_timer_ns() - t0 < kWaitLimitNs) ok = ld_acquire_sys(f) == p.xepoch;
    }
  }
  if (!__all_sync(kFull, ok)) {
    if (lane == 0) raise_status(kStatusPeerTimeout);
    return;
  }
  float4 h = make_float4(-INFINITY, 0.f, 0.f, 0.f), a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
  if (lane < p.xworld) {
    const float4* d = reinterpret_cast<const float4*>(xstate(p, p.xrank, lane, item));
    h = __ldcg(d);
    a0 = __ldcg(d + 1);
    a1 = __ldcg(d + 2);
  }
  const float M = warp_max(h.x);
  const float w = (lane < p.xworld && h.x != -INFINITY) ? exp2f(h.x - M) : 0.f;
  const float L = warp_sum(h.y * w);
  float a[8] = {a0.x * w, a0.y * w, a0.z * w, a0.w * w, a1.x * w, a1.y * w, a1.z * w, a1.w * w};
  #pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = warp_sum(a[i]);
  if (lane == 0) {
    __nv_bfloat16* o = p.out + bh * kHeadDim + 8 * s;
    uint4 v;
    if (M == -INFINITY) {  // no tokens on any rank: 0, as python/reference.py gives
      v = make_uint4(0u, 0u, 0u, 0u);
    } else {
      const uint2 lo = pack_bf16x4(a[0] / L, a[1] / L, a[2] / L, a[3] / L);
      const uint2 hi = pack_bf16x4(a[4] / L, a[5] / L, a[6] / L, a[7] / L);
      v = make_uint4(lo.x, lo.y, hi.x, hi.y);
    }
    *reinterpret_cast<uint4*>(o) = v;
  }
}

// Bf16 output or unnormalised state of one slice item.
__device__ __forceinline__ void write_slice(const CutMergeParams& p, const SliceState& st,
                                            size_t bh, int s, int lane) {
  if (lane != 0) return;
  if (p.out_mode == kOutState) {
    if (s == 0) {
      p.res_m[bh] = st.m;
      p.res_l[bh] = st.l;
    }
    float4* d = reinterpret_cast<float4*>(p.res_acc + bh * kHeadDim + 8 * s);
    d[0] = make_float4(st.a[0], st.a[1], st.a[2], st.a[3]);
    d[1] = make_float4(st.a[4], st.a[5], st.a[6], st.a[7]);
  } else {
    const uint2 lo = pack_bf16x4(st.a[0] / st.l, st.a[1] / st.l, st.a[2] / st.l, st.a[3] / st.l);
    const uint2 hi = pack_bf16x4(st.a[4] / st.l, st.a[5] / st.l, st.a[6] / st.l, st.a[7] / st.l);
    *reinterpret_cast<uint4*>(p.out + bh * kHeadDim + 8 * s) = make_uint4(lo.x, lo.y, hi.x, hi.y);
  }
}

}  // namespace merge_detail

// Every CTA first compacts, in shared memory, the list of cut rows from the
// scan's per-CTA records (CTA c ends at most one cut row: only its first
// segment can be a row's last part) with each row's number of work items -
// QHR (one per q head) for rows of at most kFewParts parts, else QHR x
// kSlices - and their prefix; then all warps of the grid stride over the
// items.  With kOutExchange every row, cut or not, is an item set of QHR x
// kSlices (the same on every rank) read from the per-row records; a warp
// handles the same items on every rank (the grid is the same), always
// sending an item before waiting for it.
__global__ void __launch_bounds__(128, 4) gqa_decode_cut_merge_kernel(const __grid_constant__ CutMergeParams p) {
  using namespace merge_detail;
  extern __shared__ int sh[];  // [grid] rows | [grid] parts | [grid + 1] item prefix
  __shared__ int sh_warp[4];
  // Everything below reads what the scan wrote.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long gw = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + warp;

  if (p.out_mode == kOutExchange) {
    const long long heads = static_cast<long long>(p.rows) * p.QHR;
    for (long long f = gw; f < heads * kSlices; f += warps) {
      const int s = static_cast<int>(f / heads);
      const long long rh = f - s * heads;  // = b * Hq + q head
      const int r = static_cast<int>(rh / p.QHR);
      const int j = static_cast<int>(rh - static_cast<long long>(r) * p.QHR);
      const int2 ri = p.row_info[r];  // {first CTA, parts}
      const SliceState st = merge_slice(p, static_cast<long long>(ri.x) + r, ri.y, j, s, lane);
      exchange_item(p, st, static_cast<size_t>(rh) * kSlices + s, static_cast<size_t>(rh), s,
                    lane);
    }
    return;
  }

  int* s_row = sh;
  int* s_n = sh + p.grid;
  int* s_pre = sh + 2 * p.grid;
  // chunk of the scan's CTAs per thread, local item sum, block scan
  const int per = (p.grid + blockDim.x - 1) / blockDim.x;
  const int c0 = min(p.grid, static_cast<int>(threadIdx.x) * per);
  const int c1 = min(p.grid, c0 + per);
  int local = 0;
  for (int c = c0; c < c1; ++c) {
    const int2 e = p.ends[c];  // {row, parts} or {-1, 0}
    const int w = e.x < 0 ? 0 : (e.y <= kFewParts ? p.QHR : p.QHR * kSlices);
    s_row[c] = e.x;
    s_n[c] = e.y;
    s_pre[c] = w;  // item count for now
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
  for (long long f = gw; f < total; f += warps) {
    // the CTA record holding item f: largest c with s_pre[c] <= f
    int lo = 0, hi = p.grid - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_pre[mid] <= f) lo = mid; else hi = mid - 1;
    }
    const int r = s_row[lo], n = s_n[lo];
    const long long base = static_cast<long long>(lo) - n + 1 + r;  // slot of the first part
    const int local_item = static_cast<int>(f - s_pre[lo]);
    if (n <= kFewParts) {
      const int j = local_item;
      merge_head(p, base, n, j, static_cast<size_t>(r) * p.QHR + j, lane);
    } else {
      const int s = local_item / p.QHR;
      const int j = local_item - s * p.QHR;
      const SliceState st = merge_slice(p, base, n, j, s, lane);
      write_slice(p, st, static_cast<size_t>(r) * p.QHR + j, s, lane);
    }
  }
}

size_t cut_merge_smem_bytes(int grid) { return (3 * static_cast<size_t>(grid) + 1) * sizeof(int); }

// Launched with programmatic stream serialization, so it may start while the
// scan still runs (the scan signals griddepcontrol.launch_dependents at its
// start) and waits for the scan's results inside.
cudaError_t launch_cut_merge(const CutMergeParams& p, int grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(128);
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
