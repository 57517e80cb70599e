// Internal types shared by the decode kernels and the C-ABI entry points.
//
// Work model.  A "row" is one request b and one group of HG consecutive kv
// heads (hg).  A row's tokens [0, S_b) are cut into "stages" of 16 tokens,
// the unit of one pipeline slot and one tensor-core M tile.  The scan kernel
// walks a sequence of "segments" (a row and a stage range) in one of two
// schedules:
//   * FIXED     - the reference's split-KV decomposition: every row is cut
//                 into num_splits equal stage chunks (tasks), tasks are dealt
//                 to CTAs round-robin (python/gqa_decode_ext.cpp:97-123,
//                 kernels/gqa_decode/v2_splitkv.cu:30-32 split on tokens;
//                 here the cut is on 16-token stages).
//   * BALANCED  - the flattened sequence of all rows' stages is divided into
//                 gridDim.x equal contiguous ranges, one per resident CTA, so
//                 every SM streams the same number of KV bytes whatever the
//                 batch's length distribution.
// A segment that covers its whole row writes the normalised bf16 output; a
// segment that covers part of a row writes an unnormalised fp32 partial
// (m, l, acc) that a merge combines with the online-softmax identity
// (kernels/gqa_decode/v2_splitkv.cu:97-107).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime_api.h>

namespace gqa {

constexpr int kHeadDim = 128;        // d, fixed by the reference API
constexpr int kStageTokens = 16;     // tokens per pipeline stage / MMA M tile
constexpr int kMaxConsumerWarps = 16;
constexpr int kMaxSplits = 512;      // python/gqa_decode_ext.cpp:102-103
constexpr int kSmemBudget = 200 * 1024;  // dynamic smem per CTA for the stage ring
constexpr int kMaxStages = 8;

enum Schedule : int { kFixed = 0, kBalanced = 1 };

// Where a finished (request, q head) goes.
enum OutMode : int {
  kOutBf16 = 0,      // normalised bf16 `out`
  kOutState = 1,     // unnormalised (m, l, acc) in res_* (KV shard, NCCL exchange)
  kOutExchange = 2,  // state pushed to every rank's exchange buffer, merged in-kernel
};

// KV-range sharding over peer memory: every rank owns one exchange buffer of
// u64 words [2][world][items][kXItem], mapped into every other rank; [2] is
// the epoch parity, an item is one 32-dim chunk of one (request, q head):
// items = B * Hq * 4, each {m, l, acc[32], 2 pad} with the epoch in every
// word's upper half.
constexpr int kMaxPeers = 8;
constexpr int kXItem = 36;       // u64 words per item state
constexpr int kXSlices = 4;      // items per (request, q head)
constexpr int kMaxScanGrid = 2048;  // BALANCED grid cap (the merge kernel's per-CTA list)

// Shape-only launch plan (no device state): how heads map to warps and how
// large the stage ring is.
struct ShapePlan {
  int G;          // q heads per kv head (Hq / Hkv)
  int NT;         // 8-head MMA column tiles per kv head = ceil(G / 8)
  int HG;         // kv heads per row (per CTA)
  int NHG;        // rows per request = Hkv / HG
  int ncw;        // consumer warps = HG * NT
  int threads;    // (ncw + 1) * 32, one producer warp
  int row_bytes;  // bytes of one token's HG kv heads = HG * 256
  int row_stride; // smem stride of one token row = row_bytes + 16 (bank skew)
  int stage_bytes;// K and V rows of one 16-token stage
  int nstages;    // depth of the ring
  int smem_bytes; // dynamic shared memory per CTA
};

// Returns 0 on success, or a negative code for unsupported shapes.
int make_shape_plan(int Hq, int Hkv, ShapePlan* plan);

// Byte offsets of the BALANCED schedule's workspace regions (gqa_api.cu).
struct BalancedLayout {
  size_t plan, prefix, rowinfo, ends, m, l, acc, total;
};
int balanced_grid(int sms, int occ);
BalancedLayout balanced_layout(int B, const ShapePlan& sp, int grid);

struct ScanParams {
  const __nv_bfloat16* q;        // [B, Hq, 128]
  const __nv_bfloat16* k;        // [num_blocks, bs, Hkv, 128]
  const __nv_bfloat16* v;        // [num_blocks, bs, Hkv, 128]
  const int* block_table;        // [B, max_blocks] (dense page table)
  const int* seq_lens;           // [B]
  // CSR page table (csr != 0): pages of request b are
  // kv_indices[kv_indptr[b] .. kv_indptr[b+1]), its last page holding
  // kv_last[b] tokens.
  const int* kv_indptr;
  const int* kv_indices;
  const int* kv_last;
  int csr;
  // Precomputed BALANCED schedule (gqa_decode_plan), or null to compute the
  // CTA's range in the kernel: [T, E (ranges with work), grid, ...(8)] then per CTA
  // {g0, g1, b0, P0}.
  const long long* plan;
  __nv_bfloat16* out;            // [B, Hq, 128]; unused with kOutState
  // Split partials.  FIXED: reference layout [B, Hq, num_splits](,128).
  // BALANCED: slot layout [slot, HG*G](,128), slot = cta + row.
  float* part_m;
  float* part_l;
  float* part_acc;
  // BALANCED: per row {first CTA holding a part, parts} and per CTA {row,
  // parts} of the cut row whose last part it holds ({-1, 0}: none), written
  // by every launch for the merge kernel.
  int2* row_info;                // [B * NHG]
  int2* ends;                    // [grid]
  // kOutState: the final per-(b, q-head) state is written unnormalised
  // here instead of bf16 `out` (KV-range sharding across GPUs).
  float* res_m;                  // [B, Hq]
  float* res_l;                  // [B, Hq]
  float* res_acc;                // [B, Hq, 128]
  int B, Hq, Hkv, bs, max_blocks;
  int num_blocks;                // > 0: check block ids; 0: trust them
  int G, NT, HG, NHG, ncw;
  int row_bytes, row_stride, stage_bytes, nstages;
  int schedule;                  // Schedule
  int num_splits;                // FIXED
  int out_mode;                  // OutMode
  float scale_log2;              // softmax scale * log2(e)
  // Limit of every pipeline wait, in ns of %globaltimer (kWaitLimitNs; the
  // wait-timeout self-test passes a tiny one).  The producer's final drain of
  // its own copies always uses kWaitLimitNs.
  unsigned long long wait_ns;
  // Failure-detection self-test only: the copy warp issues no copy, so every
  // consumer wait runs out (after wait_ns) as it would on a stuck pipeline.
  int selftest_no_copies;
};

// Merge of the BALANCED scan's cut rows (and, with kOutExchange, the
// cross-rank exchange of every row), gqa_merge.cu.
struct CutMergeParams {
  const int2* row_info;          // [rows] {first CTA, parts}
  const int2* ends;              // [grid] {row, parts} / {-1, 0}
  const float* part_m;           // [slot, QHR]
  const float* part_l;
  const float* part_acc;         // [slot, QHR, 128]
  __nv_bfloat16* out;            // [B, Hq, 128]
  float* res_m;                  // kOutState: [B, Hq]
  float* res_l;
  float* res_acc;                // kOutState: [B, Hq, 128]
  int rows, QHR;                 // rows = B * NHG, QHR = q heads per row
  int grid;                      // the scan's grid
  int out_mode;                  // OutMode
  // kOutExchange
  int xworld, xrank;
  unsigned xepoch;               // != 0, identical on every rank for one decode
  long long xitems;              // B * Hq * kXSlices items per (parity, source rank)
  unsigned char* xpeer[kMaxPeers];  // exchange buffer of every rank ([xrank] = own)
  unsigned long long wait_ns;    // limit of the wait for the peers' states (kWaitLimitNs)
};

// Every rank's exchange merge in one cooperative launch on one GPU (test
// emulation of the KV-range sharded decode): CTA c plays rank c / per_rank.
struct ExchangeEmulParams {
  CutMergeParams rank[kMaxPeers];
  int world, per_rank;
};

struct MergeParams {
  const float* part_m;
  const float* part_l;
  const float* part_acc;
  const int* seq_lens;
  __nv_bfloat16* out;
  int B, Hq, Hkv, bs, max_blocks, num_splits;
};

struct SimtParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const int* block_table;
  const int* seq_lens;
  __nv_bfloat16* out;
  int B, Hq, Hkv, bs, max_blocks;
  float scale_log2;
};

struct ShardMergeParams {
  const float* m;    // [nshards, rows]
  const float* l;    // [nshards, rows]
  const float* acc;  // [nshards, rows, 128]
  __nv_bfloat16* out;// [rows, 128]
  int nshards;
  int rows;          // B * Hq
};

// Kernel launchers (gqa_scan.cu / gqa_simt.cu).  They launch and return the
// launch status; validation happens in the C-ABI layer.
cudaError_t launch_scan(const ScanParams& p, int grid, int threads, int smem, cudaStream_t s);
// The cut-row merge, launched with programmatic dependent launch right after
// the scan on the same stream; `grid` = CTAs of the merge kernel.
cudaError_t launch_cut_merge(const CutMergeParams& p, int grid, cudaStream_t s);
// Cooperative launch of the emulated exchange merge (world * per_rank CTAs,
// all resident at once); per_rank from exchange_emul_per_rank.
cudaError_t launch_exchange_emulated(const ExchangeEmulParams& e, cudaStream_t s);
int exchange_emul_per_rank(int world, int sms);
// Scan + cut-row merge of the BALANCED schedule with bf16 output or states,
// the records and partial slots placed in `w` by `lay` (gqa_api.cu).
cudaError_t launch_balanced_noexchange(ScanParams& p, const BalancedLayout& lay,
                                       unsigned char* w, const ShapePlan& sp, int sms, int grid,
                                       cudaStream_t stream);
cudaError_t launch_fixed_merge(const MergeParams& p, cudaStream_t s);
cudaError_t launch_simt(const SimtParams& p, cudaStream_t s);
cudaError_t launch_shard_merge(const ShardMergeParams& p, cudaStream_t s);
cudaError_t scan_kernel_set_smem(int smem_bytes);
cudaError_t scan_kernel_occupancy(int threads, int smem_bytes, int* blocks_per_sm);
cudaError_t read_status(int* status, int clear);
cudaError_t launch_wait_selftest(unsigned long long limit_ns, cudaStream_t s);
// BALANCED plan for `grid` CTAs into plan (header + entries) using prefix
// ([B + 1] int64 scratch); p supplies the page table and shape.
cudaError_t launch_plan(const ScanParams& p, long long* plan, long long* prefix, int grid,
                        cudaStream_t s);
// block_table / seq_lens -> CSR (reference bench/baselines/flashinfer_adapter.py:33-51).
cudaError_t launch_block_table_to_csr(const int* block_table, const int* seq_lens, int B,
                                      int max_blocks, int page_size, int* indptr, int* indices,
                                      int* last_page_len, cudaStream_t s);
// Bodies of the three reference-signature launchers (gqa_api.cu), shared by
// their C-linkage and C++-linkage exports; each records its status for
// gqa_decode_last_error().
void compat_v0_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                      const __nv_bfloat16* v_cache, const int* block_table, const int* seq_lens,
                      __nv_bfloat16* out, int B, int Hq, int Hkv, int block_size, int max_blocks,
                      float scale, cudaStream_t stream);
void compat_v1_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                      const __nv_bfloat16* v_cache, const int* block_table, const int* seq_lens,
                      __nv_bfloat16* out, int B, int Hq, int Hkv, int block_size, int max_blocks,
                      float scale, cudaStream_t stream);
void compat_v2_launch(const __nv_bfloat16* q, const __nv_bfloat16* k_cache,
                      const __nv_bfloat16* v_cache, const int* block_table, const int* seq_lens,
                      __nv_bfloat16* out, int B, int Hq, int Hkv, int block_size, int max_blocks,
                      float scale, int num_splits, float* ws_acc, float* ws_m, float* ws_l,
                      cudaStream_t stream);
constexpr int kPlanHeader = 8;   // int64 header words of a plan
constexpr int kPlanEntry = 4;    // int64 words per CTA entry

}  // namespace gqa
