/*
 * DSA-style sparse decode (indexer + top-k + sparse gather) on B200, C ABI.
 *
 * The reference's roadmap kernel K3 (README.md "Roadmap": "DSA-style sparse
 * decode: indexer + top-k + sparse gather") has no code in the reference —
 * kernels/sparse_decode/ is empty — so there is no reference interface to
 * replace.  The operator is DeepSeek sparse attention's decode step:
 *   scores   I[b, i, t] = sum_j w_idx[b, i, j] * relu(q_idx[b, i, j, :] . k_idx[t, :])
 *            over the tokens query (b, i) can see (t < S_b, or
 *            t < S_b - s_q + 1 + i when causal); q_idx [B, s_q, H, 128] bf16,
 *            w_idx [B, s_q, H] fp32, k_idx [num_blocks, 64, 128] bf16 paged by
 *            the same block_table as the latent cache;
 *   top-k    the k highest-scoring tokens per (b, i), ties to the lower token
 *            index, ascending token order, -1 padded;
 *   gather   their latent rows (kv_cache [num_blocks, 64, 1, 576] bf16) into
 *            contiguous 64-token pages, then MLA decode (include/mla_decode.h)
 *            over them.
 * All pointers are device pointers; entry points are asynchronous on
 * `stream` and allocate nothing.
 */
#ifndef DSA_DECODE_B200_H
#define DSA_DECODE_B200_H

#include <stddef.h>
#include <cuda_runtime.h>

#include "gqa_decode.h" /* gqa_bf16 */

#ifdef __cplusplus
extern "C" {
#endif

/* Indexer scores into scores[(b * s_q + i) * scores_stride + t] for t < S_b
 * (-inf past the visible range).  Requires page_size == 64, s_q in {1, 2},
 * s_q * n_heads in {64, 128}, scores_stride >= max_blocks * 64. */
cudaError_t dsa_indexer_launch(const gqa_bf16* q_idx, const float* w_idx, const gqa_bf16* k_idx,
                               const int* block_table, const int* seq_lens, float* scores,
                               long long scores_stride, int B, int s_q, int n_heads,
                               int page_size, int max_blocks, int num_blocks, int causal,
                               cudaStream_t stream);

/* Top-k token indices per (b, i) into indices[(b * s_q + i) * k + 0..k-1],
 * ascending, -1 padded; counts[b * s_q + i] = min(k, visible) when counts is
 * not null.  max_tokens caps S_b (the page table's capacity). */
cudaError_t dsa_topk_launch(const float* scores, long long scores_stride, const int* seq_lens,
                            int B, int s_q, int k, int max_tokens, int causal, int* indices,
                            int* counts, cudaStream_t stream);

/* dsa_topk_launch plus, for every selected token, its physical row in the
 * paged caches, rows[(b * s_q + i) * k + j] = block_table[b, t / 64] * 64 +
 * t % 64 for token t (-1 padded), so the sparse MLA decode can fetch the row
 * with one load instead of the token -> block -> row chain
 * (mla_decode_sparse_rows_launch).  max_tokens <= max_blocks * 64; a block id
 * outside [0, num_blocks) sets status bit 1 and reads block 0.  No reference
 * counterpart (roadmap kernel K3). */
cudaError_t dsa_topk_rows_launch(const float* scores, long long scores_stride,
                                 const int* seq_lens, int B, int s_q, int k, int max_tokens,
                                 int causal, const int* block_table, int max_blocks,
                                 int num_blocks, int* indices, int* counts, int* rows,
                                 cudaStream_t stream);

/* Latent rows of the selected tokens into gathered[((b * s_q + i) * kpad + slot) * 576],
 * kpad = k rounded up to 64; -1 slots are zero rows. */
cudaError_t dsa_gather_launch(const gqa_bf16* kv_cache, const int* block_table,
                              const int* indices, int B, int s_q, int k, int max_blocks,
                              int num_blocks, gqa_bf16* gathered, cudaStream_t stream);

/* Device status word (bit 0: a bounded wait gave up, bit 1: block id out of
 * range); reset clears it.  Synchronises the device. */
int dsa_decode_get_status(int reset);

#ifdef __cplusplus
}
#endif

#endif /* DSA_DECODE_B200_H */
