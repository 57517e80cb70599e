// C-ABI entry points: argument validation, launch planning and dispatch to
// the kernels.  Declared in include/gqa_decode.h.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "gqa_decode.h"
#include "gqa_internal.h"
#include "gqa_ptx.cuh"

namespace gqa {

int make_shape_plan(int Hq, int Hkv, ShapePlan* sp) {
  if (Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) return -1;
  const int G = Hq / Hkv;
  const int NT = (G + 7) / 8;
  if (NT > kMaxConsumerWarps) return -2;
  int HG = 1;
  for (int d = 1; d <= Hkv && d * NT <= 8; ++d)
    if (Hkv % d == 0) HG = d;
  sp->G = G;
  sp->NT = NT;
  sp->HG = HG;
  sp->NHG = Hkv / HG;
  sp->ncw = HG * NT;
  sp->threads = (sp->ncw + 1) * 32;
  sp->row_bytes = HG * kHeadDim * 2;
  sp->row_stride = sp->row_bytes + 16;
  sp->stage_bytes = 2 * kStageTokens * sp->row_stride;
  sp->nstages = std::max(2, std::min(kMaxStages, kSmemBudget / sp->stage_bytes));
  sp->smem_bytes = sp->nstages * sp->stage_bytes + 3 * 8 * sp->nstages;
  return 0;
}

// BALANCED grid: one CTA per resident slot, capped so the merge kernel's
// per-CTA list of cut rows fits its shared memory.
int balanced_grid(int sms, int occ) { return std::min(sms * occ, kMaxScanGrid); }

// [plan (header + one entry per CTA) | prefix [B + 1] | row records [B*NHG] |
//  CTA records [grid] | m | l | acc].  Nothing needs zeroing: every launch
// writes every record it reads.
BalancedLayout balanced_layout(int B, const ShapePlan& sp, int grid) {
  auto align_up = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t rows = static_cast<size_t>(B) * sp.NHG;
  const size_t qhr = static_cast<size_t>(sp.HG) * sp.G;
  const size_t slots = static_cast<size_t>(grid) + rows;
  BalancedLayout L;
  L.plan = 0;
  L.prefix = L.plan + align_up((kPlanHeader + static_cast<size_t>(grid) * kPlanEntry) *
                               sizeof(long long));
  L.rowinfo = L.prefix + align_up((static_cast<size_t>(B) + 1) * sizeof(long long));
  L.ends = L.rowinfo + align_up(rows * sizeof(int2));
  L.m = L.ends + align_up(static_cast<size_t>(grid) * sizeof(int2));
  L.l = L.m + align_up(slots * qhr * sizeof(float));
  L.acc = L.l + align_up(slots * qhr * sizeof(float));
  L.total = L.acc + align_up(slots * qhr * kHeadDim * sizeof(float));
  return L;
}

}  // namespace gqa

namespace {

using gqa::BalancedLayout;
using gqa::ShapePlan;
using gqa::balanced_grid;
using gqa::balanced_layout;

thread_local cudaError_t t_last_error = cudaSuccess;

constexpr size_t kAlign = 256;
size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Fixed splits through gqa_decode_launch: the reference's [B, Hq, ns](,128)
// partial arrays, acc then m then l.
size_t fixed_ws_bytes(int B, int Hq, int ns) {
  const size_t states = static_cast<size_t>(B) * Hq * ns;
  return align_up(states * gqa::kHeadDim * sizeof(float)) + 2 * align_up(states * sizeof(float));
}

// Per-device facts, cached: SM count and resident CTAs for a (threads, smem).
struct DeviceFacts {
  int sms = 0;
  int smem_attr = 0;
  int occ_threads = 0, occ_smem = 0, occ = 0;
};
constexpr int kMaxDevices = 64;
DeviceFacts g_facts[kMaxDevices];
std::mutex g_facts_mu;

cudaError_t device_facts(const ShapePlan& sp, int* sms, int* occ) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_facts_mu);
  DeviceFacts& f = g_facts[dev];
  if (f.sms == 0) {
    e = cudaDeviceGetAttribute(&f.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  if (f.smem_attr < sp.smem_bytes) {
    e = gqa::scan_kernel_set_smem(sp.smem_bytes);
    if (e != cudaSuccess) return e;
    f.smem_attr = sp.smem_bytes;
  }
  if (f.occ_threads != sp.threads || f.occ_smem != sp.smem_bytes) {
    int o = 0;
    e = gqa::scan_kernel_occupancy(sp.threads, sp.smem_bytes, &o);
    if (e != cudaSuccess) return e;
    if (o < 1) return cudaErrorInvalidConfiguration;
    f.occ_threads = sp.threads;
    f.occ_smem = sp.smem_bytes;
    f.occ = o;
  }
  *sms = f.sms;
  *occ = f.occ;
  return cudaSuccess;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Checks shared by every launcher (python/gqa_decode_ext.cpp:16-62 checks the
// same facts on tensors).
cudaError_t check_common(const void* q, const void* k, const void* v, const int* bt,
                         const int* sl, const void* out, int B, int Hq, int Hkv, int bs,
                         int max_blocks, ShapePlan* sp) {
  if (B < 0 || bs <= 0 || max_blocks <= 0) return cudaErrorInvalidValue;
  if (gqa::make_shape_plan(Hq, Hkv, sp) != 0) return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  if (!q || !k || !v || !bt || !sl || !out) return cudaErrorInvalidValue;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return cudaErrorMisalignedAddress;
  return cudaSuccess;
}

gqa::ScanParams base_params(const gqa_bf16* q, const gqa_bf16* k, const gqa_bf16* v,
                            const int* bt, const int* sl, int B, int Hq, int Hkv, int bs,
                            int max_blocks, int num_blocks, float scale, const ShapePlan& sp) {
  gqa::ScanParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.block_table = bt;
  p.seq_lens = sl;
  // dense page table: the CSR pointers alias it (valid memory, never read)
  p.kv_indptr = sl;
  p.kv_indices = bt;
  p.kv_last = sl;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.bs = bs;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.G = sp.G;
  p.NT = sp.NT;
  p.HG = sp.HG;
  p.NHG = sp.NHG;
  p.ncw = sp.ncw;
  p.row_bytes = sp.row_bytes;
  p.row_stride = sp.row_stride;
  p.stage_bytes = sp.stage_bytes;
  p.nstages = sp.nstages;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.wait_ns = gqa::kWaitLimitNs;
  return p;
}

// FIXED schedule: scan (+ merge when num_splits > 1) into the reference's
// workspace layout.
cudaError_t run_fixed(const gqa_bf16* q, const gqa_bf16* k, const gqa_bf16* v, const int* bt,
                      const int* sl, gqa_bf16* out, int B, int Hq, int Hkv, int bs,
                      int max_blocks, int num_blocks, float scale, int ns, float* ws_acc,
                      float* ws_m, float* ws_l, cudaStream_t stream) {
  ShapePlan sp;
  cudaError_t e = check_common(q, k, v, bt, sl, out, B, Hq, Hkv, bs, max_blocks, &sp);
  if (e != cudaSuccess) return e;
  if (ns < 1 || ns > gqa::kMaxSplits) return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  if (ns > 1 && (!ws_acc || !ws_m || !ws_l || !aligned16(ws_acc))) return cudaErrorInvalidValue;
  int sms = 0, occ = 0;
  e = device_facts(sp, &sms, &occ);
  if (e != cudaSuccess) return e;
  gqa::ScanParams p =
      base_params(q, k, v, bt, sl, B, Hq, Hkv, bs, max_blocks, num_blocks, scale, sp);
  p.out = out;
  p.part_acc = ws_acc;
  p.part_m = ws_m;
  p.part_l = ws_l;
  p.schedule = gqa::kFixed;
  p.num_splits = ns;
  const long long tasks = static_cast<long long>(B) * sp.NHG * ns;
  if (tasks > INT_MAX) return cudaErrorInvalidValue;
  const int grid = static_cast<int>(std::min<long long>(tasks, static_cast<long long>(sms) * occ));
  e = gqa::launch_scan(p, grid, sp.threads, sp.smem_bytes, stream);
  if (e != cudaSuccess || ns == 1) return e;
  gqa::MergeParams mp{};
  mp.part_m = ws_m;
  mp.part_l = ws_l;
  mp.part_acc = ws_acc;
  mp.seq_lens = sl;
  mp.out = out;
  mp.B = B;
  mp.Hq = Hq;
  mp.Hkv = Hkv;
  mp.bs = bs;
  mp.max_blocks = max_blocks;
  mp.num_splits = ns;
  return gqa::launch_fixed_merge(mp, stream);
}

// Page table of a launch, resolved from the C descriptor.
struct Pages {
  const int* bt = nullptr;
  const int* sl = nullptr;
  int max_blocks = 0;
  const int* indptr = nullptr;
  const int* indices = nullptr;
  const int* last = nullptr;
  int bs = 0;
  int num_blocks = 0;
  bool csr = false;
};

cudaError_t resolve_pages(const gqa_decode_pages* d, Pages* pg) {
  if (!d || d->block_size <= 0 || d->num_blocks < 0) return cudaErrorInvalidValue;
  pg->bs = d->block_size;
  pg->num_blocks = d->num_blocks;
  if (d->block_table) {
    if (!d->seq_lens || d->max_blocks <= 0) return cudaErrorInvalidValue;
    pg->bt = d->block_table;
    pg->sl = d->seq_lens;
    pg->max_blocks = d->max_blocks;
    pg->csr = false;
  } else {
    if (!d->kv_indptr || !d->kv_indices || !d->kv_last_page_len) return cudaErrorInvalidValue;
    pg->indptr = d->kv_indptr;
    pg->indices = d->kv_indices;
    pg->last = d->kv_last_page_len;
    pg->max_blocks = 1;  // unused with CSR (lengths come from indptr)
    pg->csr = true;
  }
  // The kernels read only the active table; the other one's pointers still
  // point at valid device memory (the active arrays), never at null.
  if (pg->csr) {
    pg->bt = pg->indices;
    pg->sl = pg->last;
  } else {
    pg->indptr = pg->sl;
    pg->indices = pg->bt;
    pg->last = pg->sl;
  }
  return cudaSuccess;
}

// Peer-exchange arguments of the KV-range sharded decode.
struct Exchange {
  int world = 0, rank = 0;
  unsigned epoch = 0;
  void* const* peers = nullptr;
};

size_t exchange_items(int B, int Hq) {
  return static_cast<size_t>(B) * Hq * gqa::kXSlices;
}

size_t exchange_bytes(int B, int Hq, int world) {
  return 2ull * world * exchange_items(B, Hq) * gqa::kXItem * sizeof(unsigned long long);
}

// Parameters of the scan and the cut-row merge of the BALANCED schedule.
// `p` carries the inputs, the output mode and the schedule; the workspace
// supplies the records and partial slots.
cudaError_t setup_balanced(gqa::ScanParams& p, const BalancedLayout& lay, unsigned char* w,
                           int grid, const Exchange* xchg, gqa::CutMergeParams& mp) {
  mp = gqa::CutMergeParams{};
  if (xchg) {
    if (!p.out || xchg->world < 1 || xchg->world > gqa::kMaxPeers || xchg->rank < 0 ||
        xchg->rank >= xchg->world || xchg->epoch == 0 || !xchg->peers)
      return cudaErrorInvalidValue;
    for (int r = 0; r < xchg->world; ++r) {
      if (!xchg->peers[r] || !aligned16(xchg->peers[r])) return cudaErrorInvalidValue;
      mp.xpeer[r] = static_cast<unsigned char*>(xchg->peers[r]);
    }
    p.out_mode = gqa::kOutExchange;
    mp.xworld = xchg->world;
    mp.xrank = xchg->rank;
    mp.xepoch = xchg->epoch;
    mp.xitems = static_cast<long long>(exchange_items(p.B, p.Hq));
  }
  p.row_info = reinterpret_cast<int2*>(w + lay.rowinfo);
  p.ends = reinterpret_cast<int2*>(w + lay.ends);
  p.part_m = reinterpret_cast<float*>(w + lay.m);
  p.part_l = reinterpret_cast<float*>(w + lay.l);
  p.part_acc = reinterpret_cast<float*>(w + lay.acc);
  p.schedule = gqa::kBalanced;
  p.num_splits = 0;
  mp.row_info = p.row_info;
  mp.ends = p.ends;
  mp.part_m = p.part_m;
  mp.part_l = p.part_l;
  mp.part_acc = p.part_acc;
  mp.out = p.out;
  mp.res_m = p.res_m;
  mp.res_l = p.res_l;
  mp.res_acc = p.res_acc;
  mp.rows = p.B * p.NHG;
  mp.QHR = p.HG * p.G;
  mp.grid = grid;
  mp.out_mode = p.out_mode;
  mp.wait_ns = p.wait_ns;
  return cudaSuccess;
}

// Scan + cut-row merge of the BALANCED schedule; the merge kernel runs one
// CTA per SM.
cudaError_t launch_balanced(gqa::ScanParams& p, const BalancedLayout& lay, unsigned char* w,
                            const ShapePlan& sp, int sms, int grid, cudaStream_t stream,
                            const Exchange* xchg) {
  gqa::CutMergeParams mp;
  cudaError_t e = setup_balanced(p, lay, w, grid, xchg, mp);
  if (e != cudaSuccess) return e;
  e = gqa::launch_scan(p, grid, sp.threads, sp.smem_bytes, stream);
  if (e != cudaSuccess) return e;
  return gqa::launch_cut_merge(mp, sms, stream);
}

// BALANCED schedule: bf16 output, unnormalised states, or peer exchange.
cudaError_t run_balanced(const gqa_bf16* q, const gqa_bf16* k, const gqa_bf16* v, const int* bt,
                         const int* sl, gqa_bf16* out, float* res_m, float* res_l,
                         float* res_acc, int B, int Hq, int Hkv, int bs, int max_blocks,
                         int num_blocks, float scale, void* ws, size_t ws_bytes,
                         cudaStream_t stream, const Exchange* xchg = nullptr,
                         unsigned long long wait_ns = gqa::kWaitLimitNs, int no_copies = 0) {
  ShapePlan sp;
  const void* dst = out ? static_cast<const void*>(out) : static_cast<const void*>(res_acc);
  cudaError_t e = check_common(q, k, v, bt, sl, dst, B, Hq, Hkv, bs, max_blocks, &sp);
  if (e != cudaSuccess) return e;
  if (B == 0) return cudaSuccess;
  if (!out && (!res_m || !res_l)) return cudaErrorInvalidValue;
  int sms = 0, occ = 0;
  e = device_facts(sp, &sms, &occ);
  if (e != cudaSuccess) return e;
  const int grid = balanced_grid(sms, occ);
  const BalancedLayout lay = balanced_layout(B, sp, grid);
  if (!ws || ws_bytes < lay.total || !aligned16(ws)) return cudaErrorInvalidValue;
  gqa::ScanParams p =
      base_params(q, k, v, bt, sl, B, Hq, Hkv, bs, max_blocks, num_blocks, scale, sp);
  p.out = out;
  p.out_mode = out ? gqa::kOutBf16 : gqa::kOutState;
  p.res_m = res_m;
  p.res_l = res_l;
  p.res_acc = res_acc;
  p.wait_ns = wait_ns;
  p.selftest_no_copies = no_copies;
  return launch_balanced(p, lay, static_cast<unsigned char*>(ws), sp, sms, grid, stream, xchg);
}

}  // namespace

namespace gqa {

cudaError_t launch_balanced_noexchange(ScanParams& p, const BalancedLayout& lay,
                                       unsigned char* w, const ShapePlan& sp, int sms, int grid,
                                       cudaStream_t stream) {
  return launch_balanced(p, lay, w, sp, sms, grid, stream, nullptr);
}

// Bodies of the reference-signature launchers.  The C-linkage entry points
// below and the C++-linkage ones in gqa_cxx_abi.cu both call these; each
// records its status for gqa_decode_last_error().
void compat_v0_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                      const __nv_bfloat16* v_cache, const int* block_table, const int* seq_lens,
                      __nv_bfloat16* out, int B, int Hq, int Hkv, int block_size, int max_blocks,
                      float scale, cudaStream_t stream) {
  ShapePlan sp;
  cudaError_t e = check_common(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv,
                               block_size, max_blocks, &sp);
  if (e == cudaSuccess && B > 0) {
    SimtParams p{};
    p.q = q;
    p.k = k_cache;
    p.v = v_cache;
    p.block_table = block_table;
    p.seq_lens = seq_lens;
    p.out = out;
    p.B = B;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.bs = block_size;
    p.max_blocks = max_blocks;
    p.scale_log2 = scale * 1.4426950408889634f;
    e = launch_simt(p, stream);
  }
  t_last_error = e;
}

void compat_v1_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                      const __nv_bfloat16* v_cache, const int* block_table, const int* seq_lens,
                      __nv_bfloat16* out, int B, int Hq, int Hkv, int block_size, int max_blocks,
                      float scale, cudaStream_t stream) {
  t_last_error = run_fixed(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv,
                           block_size, max_blocks, 0, scale, 1, nullptr, nullptr, nullptr, stream);
}

void compat_v2_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                      const __nv_bfloat16* v_cache, const int* block_table, const int* seq_lens,
                      __nv_bfloat16* out, int B, int Hq, int Hkv, int block_size, int max_blocks,
                      float scale, int num_splits, float* ws_acc, float* ws_m, float* ws_l,
                      cudaStream_t stream) {
  t_last_error = run_fixed(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv,
                           block_size, max_blocks, 0, scale, num_splits, ws_acc, ws_m, ws_l,
                           stream);
}

}  // namespace gqa

extern "C" {

void gqa_decode_v0_launch(const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
                          const int* block_table, const int* seq_lens, gqa_bf16* out, int B,
                          int Hq, int Hkv, int block_size, int max_blocks, float scale,
                          cudaStream_t stream) {
  gqa::compat_v0_launch(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv, block_size,
                        max_blocks, scale, stream);
}

void gqa_decode_v1_launch(const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
                          const int* block_table, const int* seq_lens, gqa_bf16* out, int B,
                          int Hq, int Hkv, int block_size, int max_blocks, float scale,
                          cudaStream_t stream) {
  gqa::compat_v1_launch(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv, block_size,
                        max_blocks, scale, stream);
}

void gqa_decode_v2_launch(const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
                          const int* block_table, const int* seq_lens, gqa_bf16* out, int B,
                          int Hq, int Hkv, int block_size, int max_blocks, float scale,
                          int num_splits, float* ws_acc, float* ws_m, float* ws_l,
                          cudaStream_t stream) {
  gqa::compat_v2_launch(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv, block_size,
                        max_blocks, scale, num_splits, ws_acc, ws_m, ws_l, stream);
}

cudaError_t gqa_decode_last_error(void) {
  const cudaError_t e = t_last_error;
  t_last_error = cudaSuccess;
  return e;
}

int gqa_decode_query_plan(int B, int Hq, int Hkv, int num_splits, int num_sms, int ctas_per_sm,
                          gqa_decode_plan_info* plan) {
  ShapePlan sp;
  const int rc = gqa::make_shape_plan(Hq, Hkv, &sp);
  if (rc != 0) return rc;
  if (!plan || B < 0 || num_sms <= 0 || ctas_per_sm <= 0 || num_splits < 0 ||
      num_splits > gqa::kMaxSplits)
    return -1;
  plan->group = sp.G;
  plan->heads_per_row = sp.HG;
  plan->consumer_warps = sp.ncw;
  plan->threads = sp.threads;
  plan->stages = sp.nstages;
  plan->smem_bytes = sp.smem_bytes;
  const long long slots = static_cast<long long>(num_sms) * ctas_per_sm;
  if (num_splits == 0) {
    plan->grid = static_cast<int>(std::min<long long>(slots, gqa::kMaxScanGrid));
    plan->workspace_bytes = balanced_layout(B, sp, plan->grid).total;
  } else {
    const long long tasks = static_cast<long long>(B) * sp.NHG * num_splits;
    plan->grid = static_cast<int>(std::max(1LL, std::min(tasks, slots)));
    plan->workspace_bytes = num_splits > 1 ? fixed_ws_bytes(B, Hq, num_splits) : 0;
  }
  return 0;
}

size_t gqa_decode_workspace_bytes(int B, int Hq, int Hkv, int num_splits) {
  ShapePlan sp;
  if (gqa::make_shape_plan(Hq, Hkv, &sp) != 0 || B <= 0 || num_splits < 0 ||
      num_splits > gqa::kMaxSplits)
    return 0;
  if (num_splits > 0) return num_splits > 1 ? fixed_ws_bytes(B, Hq, num_splits) : 0;
  int sms = 0, occ = 0;
  if (device_facts(sp, &sms, &occ) != cudaSuccess) return 0;
  return balanced_layout(B, sp, balanced_grid(sms, occ)).total;
}

cudaError_t gqa_decode_workspace_init(void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream) {
  if (!workspace || workspace_bytes == 0) return cudaErrorInvalidValue;
  return cudaMemsetAsync(workspace, 0, workspace_bytes, stream);
}

cudaError_t gqa_decode_launch(const gqa_bf16* q, const gqa_bf16* k_cache,
                              const gqa_bf16* v_cache, const int* block_table,
                              const int* seq_lens, gqa_bf16* out, int B, int Hq, int Hkv,
                              int block_size, int max_blocks, int num_blocks, float scale,
                              int num_splits, void* workspace, size_t workspace_bytes,
                              cudaStream_t stream) {
  if (num_blocks < 0 || num_splits < 0 || num_splits > gqa::kMaxSplits)
    return cudaErrorInvalidValue;
  if (num_splits == 0)
    return run_balanced(q, k_cache, v_cache, block_table, seq_lens, out, nullptr, nullptr,
                        nullptr, B, Hq, Hkv, block_size, max_blocks, num_blocks, scale, workspace,
                        workspace_bytes, stream);
  float* acc = nullptr;
  float* m = nullptr;
  float* l = nullptr;
  if (num_splits > 1) {
    const size_t need = fixed_ws_bytes(B, Hq, num_splits);
    if (!workspace || workspace_bytes < need || !aligned16(workspace)) return cudaErrorInvalidValue;
    const size_t states = static_cast<size_t>(B) * Hq * num_splits;
    unsigned char* w = static_cast<unsigned char*>(workspace);
    acc = reinterpret_cast<float*>(w);
    m = reinterpret_cast<float*>(w + align_up(states * gqa::kHeadDim * sizeof(float)));
    l = reinterpret_cast<float*>(w + align_up(states * gqa::kHeadDim * sizeof(float)) +
                                 align_up(states * sizeof(float)));
  }
  return run_fixed(q, k_cache, v_cache, block_table, seq_lens, out, B, Hq, Hkv, block_size,
                   max_blocks, num_blocks, scale, num_splits, acc, m, l, stream);
}

cudaError_t gqa_decode_partial_launch(const gqa_bf16* q, const gqa_bf16* k_cache,
                                      const gqa_bf16* v_cache, const int* block_table,
                                      const int* seq_lens, float* state_m, float* state_l,
                                      float* state_acc, int B, int Hq, int Hkv, int block_size,
                                      int max_blocks, int num_blocks, float scale,
                                      void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream) {
  if (num_blocks < 0 || !state_acc) return cudaErrorInvalidValue;
  return run_balanced(q, k_cache, v_cache, block_table, seq_lens, nullptr, state_m, state_l,
                      state_acc, B, Hq, Hkv, block_size, max_blocks, num_blocks, scale,
                      workspace, workspace_bytes, stream);
}

cudaError_t gqa_decode_block_table_to_csr(const int* block_table, const int* seq_lens, int B,
                                          int max_blocks, int page_size, int* kv_indptr,
                                          int* kv_indices, int* kv_last_page_len,
                                          cudaStream_t stream) {
  if (B < 0 || max_blocks <= 0 || page_size <= 0) return cudaErrorInvalidValue;
  if (B == 0) return kv_indptr ? cudaMemsetAsync(kv_indptr, 0, sizeof(int), stream)
                               : cudaErrorInvalidValue;
  if (!block_table || !seq_lens || !kv_indptr || !kv_indices || !kv_last_page_len)
    return cudaErrorInvalidValue;
  return gqa::launch_block_table_to_csr(block_table, seq_lens, B, max_blocks, page_size, kv_indptr,
                                        kv_indices, kv_last_page_len, stream);
}

cudaError_t gqa_decode_plan(const gqa_decode_pages* pages, int B, int Hq, int Hkv,
                            void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  ShapePlan sp;
  Pages pg;
  cudaError_t e = resolve_pages(pages, &pg);
  if (e != cudaSuccess) return e;
  if (B <= 0 || gqa::make_shape_plan(Hq, Hkv, &sp) != 0) return cudaErrorInvalidValue;
  int sms = 0, occ = 0;
  e = device_facts(sp, &sms, &occ);
  if (e != cudaSuccess) return e;
  const int grid = balanced_grid(sms, occ);
  const BalancedLayout lay = balanced_layout(B, sp, grid);
  if (!workspace || workspace_bytes < lay.total || !aligned16(workspace))
    return cudaErrorInvalidValue;
  unsigned char* w = static_cast<unsigned char*>(workspace);
  gqa::ScanParams p{};
  p.block_table = pg.bt;
  p.seq_lens = pg.sl;
  p.kv_indptr = pg.indptr;
  p.kv_indices = pg.indices;
  p.kv_last = pg.last;
  p.csr = pg.csr ? 1 : 0;
  p.B = B;
  p.bs = pg.bs;
  p.max_blocks = pg.max_blocks;
  p.NHG = sp.NHG;
  return gqa::launch_plan(p, reinterpret_cast<long long*>(w + lay.plan),
                          reinterpret_cast<long long*>(w + lay.prefix), grid, stream);
}

cudaError_t gqa_decode_run(const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
                           const gqa_decode_pages* pages, gqa_bf16* out, int B, int Hq, int Hkv,
                           float scale, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream) {
  ShapePlan sp;
  Pages pg;
  cudaError_t e = resolve_pages(pages, &pg);
  if (e != cudaSuccess) return e;
  e = check_common(q, k_cache, v_cache, pg.csr ? pg.indices : pg.bt,
                   pg.csr ? pg.indptr : pg.sl, out, B, Hq, Hkv, pg.bs, pg.max_blocks, &sp);
  if (e != cudaSuccess) return e;
  if (B == 0) return cudaSuccess;
  int sms = 0, occ = 0;
  e = device_facts(sp, &sms, &occ);
  if (e != cudaSuccess) return e;
  const int grid = balanced_grid(sms, occ);
  const BalancedLayout lay = balanced_layout(B, sp, grid);
  if (!workspace || workspace_bytes < lay.total || !aligned16(workspace))
    return cudaErrorInvalidValue;
  unsigned char* w = static_cast<unsigned char*>(workspace);
  gqa::ScanParams p = base_params(q, k_cache, v_cache, pg.bt, pg.sl, B, Hq, Hkv, pg.bs,
                                  pg.max_blocks, pg.num_blocks, scale, sp);
  p.kv_indptr = pg.indptr;
  p.kv_indices = pg.indices;
  p.kv_last = pg.last;
  p.csr = pg.csr ? 1 : 0;
  p.plan = reinterpret_cast<const long long*>(w + lay.plan);
  p.out = out;
  p.out_mode = gqa::kOutBf16;
  return launch_balanced(p, lay, w, sp, sms, grid, stream, nullptr);
}

size_t gqa_decode_kvshard_buffer_bytes(int B, int Hq, int Hkv, int world) {
  ShapePlan sp;
  if (gqa::make_shape_plan(Hq, Hkv, &sp) != 0 || B <= 0 || world < 1 ||
      world > gqa::kMaxPeers)
    return 0;
  return exchange_bytes(B, Hq, world);
}

cudaError_t gqa_decode_kvshard_launch(const gqa_bf16* q, const gqa_bf16* k_cache,
                                      const gqa_bf16* v_cache, const int* block_table,
                                      const int* seq_lens, gqa_bf16* out, int B, int Hq, int Hkv,
                                      int block_size, int max_blocks, int num_blocks,
                                      float scale, int rank, int world,
                                      void* const* peer_buffers, unsigned epoch,
                                      void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream) {
  if (num_blocks < 0 || !out) return cudaErrorInvalidValue;
  Exchange x;
  x.world = world;
  x.rank = rank;
  x.epoch = epoch;
  x.peers = peer_buffers;
  return run_balanced(q, k_cache, v_cache, block_table, seq_lens, out, nullptr, nullptr, nullptr,
                      B, Hq, Hkv, block_size, max_blocks, num_blocks, scale, workspace,
                      workspace_bytes, stream, &x);
}

cudaError_t gqa_decode_merge_states(const float* state_m, const float* state_l,
                                    const float* state_acc, int nshards, int rows, gqa_bf16* out,
                                    cudaStream_t stream) {
  if (nshards <= 0 || rows < 0) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  if (!state_m || !state_l || !state_acc || !out || !aligned16(state_acc) || !aligned16(out))
    return cudaErrorInvalidValue;
  gqa::ShardMergeParams p{};
  p.m = state_m;
  p.l = state_l;
  p.acc = state_acc;
  p.out = out;
  p.nshards = nshards;
  p.rows = rows;
  return gqa::launch_shard_merge(p, stream);
}

int gqa_decode_pick_splits(int B, int Hq, int Hkv, int seq_len, int num_sms) {
  ShapePlan sp;
  if (gqa::make_shape_plan(Hq, Hkv, &sp) != 0 || B <= 0 || seq_len <= 0 || num_sms <= 0) return 1;
  // Cost model in stage units: every task pays a fixed start-up of ~4
  // stages (pipeline fill), tasks run in waves of num_sms, and a split
  // request pays one merge pass (~2 stages).
  const long long rows = static_cast<long long>(B) * sp.NHG;
  const long long L = (seq_len + gqa::kStageTokens - 1) / gqa::kStageTokens;
  int best = 1;
  double best_cost = 1e300;
  for (int ns = 1; ns <= gqa::kMaxSplits && ns <= L; ++ns) {
    const long long chunk = (L + ns - 1) / ns;
    const long long nonempty = (L + chunk - 1) / chunk;
    if (nonempty != ns) continue;  // same cut as a smaller count
    const long long tasks = rows * ns;
    const long long waves = (tasks + num_sms - 1) / num_sms;
    const double cost = static_cast<double>(waves) * (chunk + 4) + (ns > 1 ? 2.0 : 0.0);
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = ns;
    }
  }
  return best;
}

cudaError_t gqa_decode_get_status(int* status, int clear) {
  if (!status) return cudaErrorInvalidValue;
  return gqa::read_status(status, clear);
}

cudaError_t gqa_decode_selftest_wait_timeout(int limit_us, cudaStream_t stream) {
  if (limit_us <= 0 || limit_us > 2000000) return cudaErrorInvalidValue;
  return gqa::launch_wait_selftest(static_cast<unsigned long long>(limit_us) * 1000ull, stream);
}

cudaError_t gqa_decode_selftest_decode_timeout(const gqa_bf16* q, const gqa_bf16* k_cache,
                                               const gqa_bf16* v_cache, const int* block_table,
                                               const int* seq_lens, gqa_bf16* out, int B, int Hq,
                                               int Hkv, int block_size, int max_blocks,
                                               float scale, int wait_limit_us, void* workspace,
                                               size_t workspace_bytes, cudaStream_t stream) {
  if (wait_limit_us <= 0 || wait_limit_us > 1000000) return cudaErrorInvalidValue;
  return run_balanced(q, k_cache, v_cache, block_table, seq_lens, out, nullptr, nullptr, nullptr,
                      B, Hq, Hkv, block_size, max_blocks, 0, scale, workspace, workspace_bytes,
                      stream, nullptr, static_cast<unsigned long long>(wait_limit_us) * 1000ull,
                      1);
}

cudaError_t gqa_decode_selftest_exchange_timeout(const gqa_bf16* q, const gqa_bf16* k_cache,
                                                 const gqa_bf16* v_cache, const int* block_table,
                                                 const int* seq_lens, gqa_bf16* out, int B,
                                                 int Hq, int Hkv, int block_size, int max_blocks,
                                                 float scale, int wait_limit_us,
                                                 void* exchange_buffers, size_t exchange_bytes,
                                                 void* workspace, size_t workspace_bytes,
                                                 cudaStream_t stream) {
  if (wait_limit_us <= 0 || wait_limit_us > 1000000 || !exchange_buffers) return cudaErrorInvalidValue;
  const size_t one = gqa_decode_kvshard_buffer_bytes(B, Hq, Hkv, 2);
  if (one == 0 || exchange_bytes < 2 * one || !aligned16(exchange_buffers))
    return cudaErrorInvalidValue;
  // rank 0 of a world of two whose rank 1 never runs: its words never reach
  // rank 0's buffer (cleared here, so no word carries the epoch)
  cudaError_t e = cudaMemsetAsync(exchange_buffers, 0, 2 * one, stream);
  if (e != cudaSuccess) return e;
  void* peers[2] = {exchange_buffers, static_cast<unsigned char*>(exchange_buffers) + one};
  Exchange x;
  x.world = 2;
  x.rank = 0;
  x.epoch = 1;
  x.peers = peers;
  return run_balanced(q, k_cache, v_cache, block_table, seq_lens, out, nullptr, nullptr, nullptr,
                      B, Hq, Hkv, block_size, max_blocks, 0, scale, workspace, workspace_bytes,
                      stream, &x, static_cast<unsigned long long>(wait_limit_us) * 1000ull);
}

cudaError_t gqa_decode_selftest_kvshard_emulated(
    const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
    const int* const* block_tables, const int* const* seq_lens, gqa_bf16* const* outs, int world,
    int B, int Hq, int Hkv, int block_size, int max_blocks, int num_blocks, float scale,
    void* exchange_buffers, size_t exchange_bytes_total, void* workspaces,
    size_t workspace_bytes_total, cudaStream_t stream) {
  if (world < 2 || world > gqa::kMaxPeers || !block_tables || !seq_lens || !outs ||
      !exchange_buffers || !workspaces || num_blocks < 0 || !aligned16(exchange_buffers) ||
      !aligned16(workspaces))
    return cudaErrorInvalidValue;
  ShapePlan sp;
  cudaError_t e = check_common(q, k_cache, v_cache, block_tables[0], seq_lens[0], outs[0], B, Hq,
                               Hkv, block_size, max_blocks, &sp);
  if (e != cudaSuccess) return e;
  if (B == 0) return cudaErrorInvalidValue;
  int sms = 0, occ = 0;
  e = device_facts(sp, &sms, &occ);
  if (e != cudaSuccess) return e;
  const int grid = balanced_grid(sms, occ);
  const BalancedLayout lay = balanced_layout(B, sp, grid);
  const size_t ws_one = (lay.total + 255) / 256 * 256;
  const size_t x_one = exchange_bytes(B, Hq, world);
  if (workspace_bytes_total < ws_one * world || exchange_bytes_total < x_one * world)
    return cudaErrorInvalidValue;
  gqa::ExchangeEmulParams ep{};
  ep.world = world;
  ep.per_rank = gqa::exchange_emul_per_rank(world, sms);
  if (ep.per_rank < 1) return cudaErrorInvalidConfiguration;
  void* peers[gqa::kMaxPeers];
  for (int r = 0; r < world; ++r)
    peers[r] = static_cast<unsigned char*>(exchange_buffers) + r * x_one;
  e = cudaMemsetAsync(exchange_buffers, 0, x_one * world, stream);  // no word has the epoch
  if (e != cudaSuccess) return e;
  for (int r = 0; r < world; ++r) {
    e = check_common(q, k_cache, v_cache, block_tables[r], seq_lens[r], outs[r], B, Hq, Hkv,
                     block_size, max_blocks, &sp);
    if (e != cudaSuccess) return e;
    gqa::ScanParams p = base_params(q, k_cache, v_cache, block_tables[r], seq_lens[r], B, Hq, Hkv,
                                    block_size, max_blocks, num_blocks, scale, sp);
    p.out = outs[r];
    Exchange x;
    x.world = world;
    x.rank = r;
    x.epoch = 1;
    x.peers = peers;
    e = setup_balanced(p, lay, static_cast<unsigned char*>(workspaces) + r * ws_one, grid, &x,
                       ep.rank[r]);
    if (e != cudaSuccess) return e;
    e = gqa::launch_scan(p, grid, sp.threads, sp.smem_bytes, stream);
    if (e != cudaSuccess) return e;
  }
  return gqa::launch_exchange_emulated(ep, stream);
}

size_t gqa_decode_selftest_kvshard_emulated_bytes(int B, int Hq, int Hkv, int world,
                                                  size_t* exchange_bytes_total) {
  ShapePlan sp;
  if (gqa::make_shape_plan(Hq, Hkv, &sp) != 0 || B <= 0 || world < 2 || world > gqa::kMaxPeers)
    return 0;
  int sms = 0, occ = 0;
  if (device_facts(sp, &sms, &occ) != cudaSuccess) return 0;
  const BalancedLayout lay = balanced_layout(B, sp, balanced_grid(sms, occ));
  if (exchange_bytes_total) *exchange_bytes_total = exchange_bytes(B, Hq, world) * world;
  return (lay.total + 255) / 256 * 256 * world;
}

const char* gqa_decode_version(void) { return "gqa_decode_b200 0.1.0 (sm_100a)"; }

}  // extern "C"
