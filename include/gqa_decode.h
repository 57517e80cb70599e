/*
 * gqa_decode.h - C ABI of the B200 (sm_100a) paged-KV GQA decode engine.
 *
 * Operator (python/reference.py:21-40 of the reference):
 *   out[b, h, :] = softmax_t(q[b, h, :] . K[t, hk, :] * scale) @ V[t, hk, :]
 *   for t < seq_lens[b], hk = h / (Hq / Hkv), with token t of request b
 *   stored in physical block block_table[b, t / block_size], slot
 *   t % block_size.
 *
 * Layouts (all row-major, contiguous, device memory):
 *   q            bf16  [B, Hq, 128]
 *   k_cache      bf16  [num_blocks, block_size, Hkv, 128]   (NHD pages)
 *   v_cache      bf16  [num_blocks, block_size, Hkv, 128]
 *   block_table  int32 [B, max_blocks]
 *   seq_lens     int32 [B]
 *   out          bf16  [B, Hq, 128]
 * q, k_cache, v_cache, out and any workspace must be 16-byte aligned.
 *
 * Every launcher is asynchronous on `stream`, allocates nothing and does not
 * synchronise.  The first three keep the reference's signatures exactly; they
 * return void as the reference does, and report argument errors through
 * gqa_decode_last_error().  This header declares them with C linkage; the
 * library also exports them with the C++ linkage of the reference header
 * (include/gqa_decode.h:6-23 there, no extern "C"), so an object compiled
 * against the reference header - e.g. the reference's own
 * python/gqa_decode_ext.cpp - links against this library unchanged.  The
 * remaining entry points are additions and return cudaError_t.
 */
#ifndef GQA_DECODE_B200_H_
#define GQA_DECODE_B200_H_

#include <stddef.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
#include <cuda_bf16.h>
typedef __nv_bfloat16 gqa_bf16;
extern "C" {
#else
#include <stdint.h>
typedef uint16_t gqa_bf16; /* raw bf16 bits */
#endif

/* Replaces gqa_decode_v0_launch (reference include/gqa_decode.h:6-10,
 * kernels/gqa_decode/v0_naive.cu:27-36).  Here: the CUDA-core grouped scan,
 * one CTA per (request, kv head), no tensor cores and no TMA - the ablation
 * rung. */
void gqa_decode_v0_launch(const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
                          const int* block_table, const int* seq_lens, gqa_bf16* out, int B,
                          int Hq, int Hkv, int block_size, int max_blocks, float scale,
                          cudaStream_t stream);

/* Replaces gqa_decode_v1_launch (reference include/gqa_decode.h:12-16,
 * kernels/gqa_decode/v1_vectorized.cu:73-82).  Here: the unsplit scan - the
 * pipelined TMA + tensor-core kernel with one segment per request. */
void gqa_decode_v1_launch(const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
                          const int* block_table, const int* seq_lens, gqa_bf16* out, int B,
                          int Hq, int Hkv, int block_size, int max_blocks, float scale,
                          cudaStream_t stream);

/* Replaces gqa_decode_v2_launch (reference include/gqa_decode.h:18-23,
 * kernels/gqa_decode/v2_splitkv.cu:110-125).  Split-KV: each request's
 * tokens are cut into num_splits chunks (1..512), partial states go to the
 * caller's fp32 workspace ws_acc [B, Hq, num_splits, 128], ws_m and
 * ws_l [B, Hq, num_splits] (same sizes as the reference), then a merge
 * kernel on the same stream writes out.  num_splits == 1 runs exactly the
 * arithmetic of gqa_decode_v1_launch (bitwise-equal output) and needs no
 * workspace. */
void gqa_decode_v2_launch(const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
                          const int* block_table, const int* seq_lens, gqa_bf16* out, int B,
                          int Hq, int Hkv, int block_size, int max_blocks, float scale,
                          int num_splits, float* ws_acc, float* ws_m, float* ws_l,
                          cudaStream_t stream);

/* Status of the calling thread's last v0/v1/v2 launch; reading it resets it
 * to cudaSuccess.  The reference's launchers have no error channel
 * (include/gqa_decode.h:6-23); the reference extension validated in
 * python/gqa_decode_ext.cpp:16-62 instead. */
cudaError_t gqa_decode_last_error(void);

/* Shape plan of the pipelined kernel (no device access). */
typedef struct gqa_decode_plan_info {
  int group;             /* q heads per kv head, Hq / Hkv */
  int heads_per_row;     /* kv heads one CTA streams per token row */
  int consumer_warps;    /* tensor-core warps per CTA */
  int threads;           /* CTA size, consumer warps + one copy warp */
  int stages;            /* depth of the shared-memory ring (16 tokens each) */
  int smem_bytes;        /* dynamic shared memory per CTA */
  int grid;              /* CTAs launched */
  size_t workspace_bytes;/* bytes gqa_decode_launch needs for these dims */
} gqa_decode_plan_info;

/* Plan for the given dims on a GPU with num_sms SMs running ctas_per_sm CTAs
 * of this kernel each.  num_splits: 0 = balanced schedule, 1..512 = fixed
 * splits.  Returns 0, or -1 for invalid dims / -2 for Hq / Hkv > 128.
 * No reference counterpart (the reference sizes its grid in each launcher). */
int gqa_decode_query_plan(int B, int Hq, int Hkv, int num_splits, int num_sms, int ctas_per_sm,
                          gqa_decode_plan_info* plan);

/* Workspace bytes gqa_decode_launch / gqa_decode_partial_launch need on the
 * current device; 0 when none is needed.  No reference counterpart (the
 * reference extension allocates per call, python/gqa_decode_ext.cpp:106-109). */
size_t gqa_decode_workspace_bytes(int B, int Hq, int Hkv, int num_splits);

/* Zero a workspace.  Optional: every launch writes each workspace record it
 * reads (the balanced schedule's per-row and per-CTA records and partial
 * states), so a workspace needs no initialisation; kept for callers that
 * clear workspaces as a habit. */
cudaError_t gqa_decode_workspace_init(void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream);

/* Decode with the split count chosen by the library (num_splits == 0) or
 * given (1..512, same semantics as gqa_decode_v2_launch).  num_splits == 0
 * selects the balanced schedule: one persistent CTA per SM, each streaming
 * an equal share of all requests' KV, then the rows cut between CTAs
 * merged by a second kernel (below).  num_blocks > 0 makes the kernel check every block id against
 * [0, num_blocks) (a bad id sets status bit 1, value 2, and reads block 0
 * instead).
 * The balanced schedule is two kernels on `stream`: the scan (one
 * persistent CTA per SM; rows held whole by a CTA are written out there) and
 * a small merge of the rows cut between CTAs, launched with programmatic
 * dependent launch so that its CTAs take the SMs as the scan's CTAs leave
 * and merge every cut row across all SMs as soon as the scan has ended.
 * Workspace: gqa_decode_workspace_bytes (no initialisation needed).
 * Concurrent launches must not share one workspace.  Additive to the
 * reference API (its extension exposes num_splits only on v2,
 * python/gqa_decode_ext.cpp:97-123). */
cudaError_t gqa_decode_launch(const gqa_bf16* q, const gqa_bf16* k_cache,
                              const gqa_bf16* v_cache, const int* block_table,
                              const int* seq_lens, gqa_bf16* out, int B, int Hq, int Hkv,
                              int block_size, int max_blocks, int num_blocks, float scale,
                              int num_splits, void* workspace, size_t workspace_bytes,
                              cudaStream_t stream);

/* Like gqa_decode_launch with num_splits == 0, but writes each (request, q
 * head)'s unnormalised softmax state instead of out: state_m, state_l
 * [B, Hq] (running max of score*scale*log2(e), and the sum of
 * 2^(score*scale*log2(e) - m)) and state_acc [B, Hq, 128].  A request with
 * no tokens gets m = -inf, l = 0, acc = 0.  Used to shard one request's KV
 * range across GPUs; combine with gqa_decode_merge_states.  No reference
 * counterpart (the reference keeps states internal,
 * kernels/gqa_decode/v2_splitkv.cu:83-89). */
cudaError_t gqa_decode_partial_launch(const gqa_bf16* q, const gqa_bf16* k_cache,
                                      const gqa_bf16* v_cache, const int* block_table,
                                      const int* seq_lens, float* state_m, float* state_l,
                                      float* state_acc, int B, int Hq, int Hkv, int block_size,
                                      int max_blocks, int num_blocks, float scale,
                                      void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream);

/* Page table of a batch: dense (the reference's block_table [B, max_blocks]
 * + seq_lens [B]) when block_table is non-NULL, else CSR (the FlashInfer
 * paged layout the reference's baseline adapter converts to,
 * bench/baselines/flashinfer_adapter.py:33-51): the pages of request b are
 * kv_indices[kv_indptr[b] .. kv_indptr[b + 1]) and its last page holds
 * kv_last_page_len[b] tokens.  num_blocks > 0 range-checks block ids. */
typedef struct gqa_decode_pages {
  const int* block_table;       /* dense [B, max_blocks], or NULL for CSR */
  const int* seq_lens;          /* dense [B] */
  int max_blocks;               /* dense: columns of block_table */
  const int* kv_indptr;         /* CSR [B + 1] */
  const int* kv_indices;        /* CSR [kv_indptr[B]] */
  const int* kv_last_page_len;  /* CSR [B] */
  int block_size;               /* tokens per page */
  int num_blocks;               /* > 0: check block ids against [0, num_blocks) */
} gqa_decode_pages;

/* Convert a dense page table to CSR on the GPU (one small kernel), with the
 * reference helper's arithmetic (bench/baselines/flashinfer_adapter.py:33-51):
 * n_b = ceil(seq_lens[b] / page_size), kv_indptr = [0, prefix sums of n_b],
 * kv_indices = the first n_b ids of every row, kv_last_page_len =
 * seq_lens - (n_b - 1) * page_size.  kv_indices needs room for
 * B * max_blocks ids. */
cudaError_t gqa_decode_block_table_to_csr(const int* block_table, const int* seq_lens, int B,
                                          int max_blocks, int page_size, int* kv_indptr,
                                          int* kv_indices, int* kv_last_page_len,
                                          cudaStream_t stream);

/* Plan half of the plan/run split (the reference's FlashInfer baseline
 * times only run(), docs/decisions/k1-007): computes on the GPU, into the
 * workspace (gqa_decode_workspace_bytes(B, Hq, Hkv, 0)), every
 * CTA's share of the balanced schedule for this batch's lengths.  No host
 * synchronisation.  The plan stays valid for any number of runs - e.g. all
 * layers of a decode step - while the lengths, B, Hq and Hkv stay the same. */
cudaError_t gqa_decode_plan(const gqa_decode_pages* pages, int B, int Hq, int Hkv,
                            void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Run half: the balanced decode of gqa_decode_launch (num_splits = 0) reading
 * its schedule from the workspace's plan instead of computing it, with a
 * dense or CSR page table.  Launch-only on the host, so it can be captured in
 * a CUDA graph. */
cudaError_t gqa_decode_run(const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
                           const gqa_decode_pages* pages, gqa_bf16* out, int B, int Hq, int Hkv,
                           float scale, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream);

/* Bytes of one rank's exchange buffer for gqa_decode_kvshard_launch with
 * world ranks (1..8); 0 for invalid dims. */
size_t gqa_decode_kvshard_buffer_bytes(int B, int Hq, int Hkv, int world);

/* KV-range sharded decode with the cross-rank merge fused into the decode's
 * own merge kernel (no collective library).  Every rank holds the same q,
 * block_table rows for its own contiguous page range of each request, and
 * seq_lens = its tokens per request.  peer_buffers[r] is rank r's exchange
 * buffer (gqa_decode_kvshard_buffer_bytes, zeroed once before the first
 * call, 16-byte aligned) as mapped into this process (CUDA IPC;
 * peer_buffers[rank] is this rank's own buffer).  After the scan, the merge
 * kernel merges this rank's state of every (request, q head, 32-dim chunk),
 * stores it into every rank's buffer with plain peer stores as 64-bit words
 * tagged with the epoch (no fence, no separate flag), waits (bounded, 4 s;
 * on timeout status bit 2, value 4, and that chunk of out is left unwritten)
 * until every rank's words of the chunk carry the epoch, and merges them
 * into out, identical on all ranks.
 * epoch: non-zero, the same on every rank for one decode, +1 per decode
 * (states are double-buffered by its parity).  Each rank must run on its own
 * GPU, and all ranks' GPUs must have the same number of SMs (their merge
 * kernels wait for one another, item by item).  The reference has no
 * multi-GPU path; the merge is its split identity
 * (kernels/gqa_decode/v2_splitkv.cu:97-107). */
cudaError_t gqa_decode_kvshard_launch(const gqa_bf16* q, const gqa_bf16* k_cache,
                                      const gqa_bf16* v_cache, const int* block_table,
                                      const int* seq_lens, gqa_bf16* out, int B, int Hq, int Hkv,
                                      int block_size, int max_blocks, int num_blocks,
                                      float scale, int rank, int world,
                                      void* const* peer_buffers, unsigned epoch,
                                      void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream);

/* Merge nshards states per row (state i of row r at index i * rows + r, acc
 * at (i * rows + r) * 128) into bf16 out [rows, 128] with the online-softmax
 * identity of kernels/gqa_decode/v2_splitkv.cu:97-107 (reference); rows whose
 * shards are all empty get 0. */
cudaError_t gqa_decode_merge_states(const float* state_m, const float* state_l,
                                    const float* state_acc, int nshards, int rows, gqa_bf16* out,
                                    cudaStream_t stream);

/* Size of the device scratch array behind gqa_decode_launch_noalloc. */
#define GQA_DECODE_NOALLOC_SCRATCH_BYTES (16u << 20)

/* gqa_decode_launch (num_splits == 0, balanced schedule) for callers that
 * cannot allocate device memory - e.g. an engine that gives all of HBM to
 * its own KV-cache pool and forbids later allocations, or a plain C / cgo /
 * JNI binding with no device allocator to hand over a workspace.  No
 * counterpart in the reference (its extension allocates a workspace on every
 * call, python/gqa_decode_ext.cpp:106-109).
 * - The scratch (the schedule, row records and split states) is a file-scope
 *   GQA_DECODE_NOALLOC_SCRATCH_BYTES (16 MiB) device array that every GPU
 *   loading this library holds until the process exits.  This call allocates
 *   nothing: no cudaMalloc, no cudaFree.
 * - Shapes whose scratch need exceeds it are rejected with
 *   cudaErrorInvalidValue before anything is launched.  The need is about
 *   (grid / rows_per_request + B) * Hq * 520 bytes (grid = one CTA per SM,
 *   rows_per_request = Hkv / heads_per_row of gqa_decode_plan_info), the
 *   gqa_decode_workspace_bytes figure: on a 148-SM B200 with Hkv = 8, up to
 *   ~860 requests at Hq = 32 or ~350 at Hq = 64.
 * - The first call on a device looks up the array's device address
 *   (cudaGetSymbolAddress) with that device current; make that first call
 *   before any stream capture.  A first call whose lookup fails returns that
 *   error and keeps nothing, so a later call tries the lookup again.
 * - All calls on a device share the array and it keeps the previous call's
 *   contents; each call writes every record it reads, so nothing needs
 *   clearing.  Calls that overlap on the GPU (other streams, other threads)
 *   race on the array and must be serialised by the caller. */
cudaError_t gqa_decode_launch_noalloc(const gqa_bf16* q, const gqa_bf16* k_cache,
                                      const gqa_bf16* v_cache, const int* block_table,
                                      const int* seq_lens, gqa_bf16* out, int B, int Hq,
                                      int Hkv, int block_size, int max_blocks, int num_blocks,
                                      float scale, cudaStream_t stream);

/* Fixed split count for the v2 schedule at a nominal seq_len: the count
 * (1..512) that minimises the estimated makespan over num_sms SMs.  The
 * reference picks it by offline sweep (bench/run_matrix.py:84-88). */
int gqa_decode_pick_splits(int B, int Hq, int Hkv, int seq_len, int num_sms);

/* Device status word of the current device: bit 0 = a pipeline wait timed
 * out, bit 1 = a block id was out of range, bit 2 = a peer rank's state
 * never arrived (gqa_decode_kvshard_launch).  clear != 0 resets it.
 * Synchronous. */
cudaError_t gqa_decode_get_status(int* status, int clear);

/* Failure-detection self-test: launches one warp that waits on a pipeline
 * barrier nothing will complete, with a limit of limit_us microseconds
 * (1..2,000,000).  The wait gives up and sets status bit 0 exactly as a
 * stuck pipeline in the decode kernels would; read it with
 * gqa_decode_get_status.  No reference counterpart (the reference has no
 * bounded waits). */
cudaError_t gqa_decode_selftest_wait_timeout(int limit_us, cudaStream_t stream);

/* Failure-detection self-test of a whole decode: gqa_decode_launch
 * (num_splits == 0) in which the copy warp issues no copy, so every pipeline
 * wait of the tensor-core warps runs out, each after wait_limit_us
 * (1..1,000,000) instead of 4 s - a stuck pipeline without any fault.  Status
 * bit 0 is then set and out holds no result (NaN / garbage rows), but the
 * launch ends normally and the warps that gave up still wrote empty states
 * and row records for their segments, so the next gqa_decode_launch on the
 * same workspace is correct.  No reference counterpart. */
cudaError_t gqa_decode_selftest_decode_timeout(const gqa_bf16* q, const gqa_bf16* k_cache,
                                               const gqa_bf16* v_cache, const int* block_table,
                                               const int* seq_lens, gqa_bf16* out, int B, int Hq,
                                               int Hkv, int block_size, int max_blocks,
                                               float scale, int wait_limit_us, void* workspace,
                                               size_t workspace_bytes, cudaStream_t stream);

/* Failure-detection self-test of the cross-rank exchange: the decode of
 * gqa_decode_kvshard_launch as rank 0 of a world of two whose rank 1 never
 * runs, on one GPU.  exchange_buffers holds both ranks' buffers
 * (2 * gqa_decode_kvshard_buffer_bytes(B, Hq, Hkv, 2) bytes, 16-byte
 * aligned; cleared here on `stream`).  Rank 0 sends its states into both
 * and waits for rank 1's, which never arrive: every wait gives up after
 * wait_limit_us (1..1,000,000) instead of 4 s, status bit 2 (value 4) is
 * set, out holds no result, and the launch ends normally - what a rank sees
 * when a peer died between decodes.  No reference counterpart. */
cudaError_t gqa_decode_selftest_exchange_timeout(const gqa_bf16* q, const gqa_bf16* k_cache,
                                                 const gqa_bf16* v_cache, const int* block_table,
                                                 const int* seq_lens, gqa_bf16* out, int B,
                                                 int Hq, int Hkv, int block_size, int max_blocks,
                                                 float scale, int wait_limit_us,
                                                 void* exchange_buffers, size_t exchange_bytes,
                                                 void* workspace, size_t workspace_bytes,
                                                 cudaStream_t stream);

/* Test emulation of the KV-range sharded decode (gqa_decode_kvshard_launch)
 * on ONE GPU: `world` (2..8) ranks, rank r decoding the pages of
 * block_tables[r] / seq_lens[r] (device arrays, as each rank would pass
 * them; q and the caches are shared) into outs[r].  Every rank's scan runs,
 * then one cooperative launch runs every rank's exchange merge at once, so
 * the ranks' waits for each other always end; the peer buffers are slices
 * of exchange_buffers and the ranks' workspaces slices of workspaces
 * (sizes from gqa_decode_selftest_kvshard_emulated_bytes).  Every outs[r]
 * must come out equal to the single-GPU decode of the whole request, and
 * identical across r.  No reference counterpart. */
cudaError_t gqa_decode_selftest_kvshard_emulated(
    const gqa_bf16* q, const gqa_bf16* k_cache, const gqa_bf16* v_cache,
    const int* const* block_tables, const int* const* seq_lens, gqa_bf16* const* outs, int world,
    int B, int Hq, int Hkv, int block_size, int max_blocks, int num_blocks, float scale,
    void* exchange_buffers, size_t exchange_bytes_total, void* workspaces,
    size_t workspace_bytes_total, cudaStream_t stream);

/* Workspace bytes (all ranks) of gqa_decode_selftest_kvshard_emulated on the
 * current device, and in *exchange_bytes_total the exchange buffers' bytes;
 * 0 for an invalid shape. */
size_t gqa_decode_selftest_kvshard_emulated_bytes(int B, int Hq, int Hkv, int world,
                                                  size_t* exchange_bytes_total);

/* Library version string. */
const char* gqa_decode_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* GQA_DECODE_B200_H_ */
