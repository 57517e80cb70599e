/*
 * MLA absorbed-path paged decode (latent cache) on B200, C ABI.
 *
 * The reference's roadmap kernel K2 (README.md "Roadmap": latent cache
 * [num_blocks, 64, 576], baseline FlashMLA) has no code in the reference —
 * kernels/mla_decode/ is empty — so there is no reference interface to
 * replace.  The operator and argument meanings follow FlashMLA's
 * flash_mla_with_kvcache, the baseline the reference names:
 *   q          [B, s_q, h_q, 576] bf16 (absorbed nope part 512 + rope 64)
 *   kv_cache   [num_blocks, 64, 1, 576] bf16 (one latent kv head; V = dims 0..511)
 *   block_table[B, max_blocks] int32, seq_lens [B] int32
 *   out        [B, s_q, h_q, 512] bf16
 *   lse        [B, h_q, s_q] fp32 natural-log softmax normaliser
 *              (-inf for a query row that sees no token; out is 0 there)
 * causal != 0 with s_q > 1: query position i sees tokens t < S - s_q + 1 + i.
 * All pointers are device pointers; every entry point is asynchronous on
 * `stream` and allocates nothing.
 */
#ifndef MLA_DECODE_B200_H
#define MLA_DECODE_B200_H

#include <stddef.h>
#include <cuda_runtime.h>

#include "gqa_decode.h" /* gqa_bf16 */

#ifdef __cplusplus
extern "C" {
#endif

/* Split count for B requests of up to max_pages 64-token pages on num_sms
 * SMs: the count (1..64, at least two pages per split) minimising a wave
 * cost model of the 2-CTA work units (pages per split plus a fixed start
 * per unit); larger for few, long requests.  Always 1 when s_q * h_q is a
 * multiple of 128: those query groups run a persistent kernel that spreads
 * the batch's pages evenly over the SMs by itself. */
int mla_decode_pick_splits(int B, int s_q, int h_q, int max_pages, int num_sms);

/* Workspace bytes.  s_q * h_q a multiple of 128: the persistent kernel's
 * partial states (two per CTA pair) and per-unit layout, whatever
 * num_splits is (about 39 MB on 148 SMs).  Otherwise the unnormalised
 * partial states of num_splits > 1, and 0 for num_splits == 1. */
size_t mla_decode_workspace_bytes(int B, int s_q, int h_q, int num_splits);

/* Decode.  Requirements: page_size == 64; 1 <= num_splits <= 64; q and
 * kv_cache 16-byte aligned; a 16-byte aligned workspace of at least
 * mla_decode_workspace_bytes() whenever that is non-zero (calls sharing a
 * workspace must not overlap on the GPU).  Block ids outside
 * [0, num_blocks) set bit 1 of mla_decode_get_status and read block 0. */
cudaError_t mla_decode_launch(const gqa_bf16* q, const gqa_bf16* kv_cache, const int* block_table,
                              const int* seq_lens, gqa_bf16* out, float* lse, int B, int s_q,
                              int h_q, int page_size, int max_blocks, int num_blocks,
                              float softmax_scale, int causal, int num_splits, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream);

/* Sparse decode over selected tokens (the attention step of a DSA-style
 * sparse decode, include/dsa_decode.h): query position i of request b
 * attends to the cache rows of tokens indices[(b * s_q + i) * topk + 0 ..
 * counts[b * s_q + i] - 1] (positions in the request's block_table), read
 * directly from the paged cache.  Requires h_q a multiple of 128 (every
 * 128-row group is one query position); otherwise as mla_decode_launch
 * without causal masking (the selection applies it). */
cudaError_t mla_decode_sparse_launch(const gqa_bf16* q, const gqa_bf16* kv_cache,
                                     const int* block_table, const int* indices,
                                     const int* counts, int topk, gqa_bf16* out, float* lse, int B,
                                     int s_q, int h_q, int page_size, int max_blocks,
                                     int num_blocks, float softmax_scale, int num_splits,
                                     void* workspace, size_t workspace_bytes,
                                     cudaStream_t stream);

/* mla_decode_sparse_launch reading each selected token's physical cache row
 * (block id * 64 + slot, as dsa_topk_rows_launch writes them; -1 padded)
 * instead of its token position and the block table: rows [B * s_q, topk],
 * counts [B * s_q].  Rows outside [0, num_blocks * 64) set status bit 1 and
 * read row 0. */
cudaError_t mla_decode_sparse_rows_launch(const gqa_bf16* q, const gqa_bf16* kv_cache,
                                          const int* cache_rows, const int* counts, int topk,
                                          gqa_bf16* out, float* lse, int B, int s_q, int h_q,
                                          int page_size, int num_blocks, float softmax_scale,
                                          int num_splits, void* workspace,
                                          size_t workspace_bytes, cudaStream_t stream);

/* Device status word of the MLA kernels (bit 0: a bounded wait gave up,
 * bit 1: block id out of range); reset clears it.  Synchronises the device. */
int mla_decode_get_status(int reset);

#ifdef __cplusplus
}
#endif

#endif /* MLA_DECODE_B200_H */
