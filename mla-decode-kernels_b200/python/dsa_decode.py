"""DSA-style sparse decode on B200: indexer -> top-k -> MLA decode over the
selected cache rows (fetched by the MLA kernel itself for h_q a multiple of
128, gathered into contiguous pages first otherwise).

The reference lists this as roadmap kernel K3 ("DSA-style sparse decode:
indexer + top-k + sparse gather", README.md "Roadmap") and ships no code for
it (kernels/sparse_decode/ is empty).  The operator is DeepSeek sparse
attention's decode step on the MLA latent cache:

    scores  = dsa_indexer(q_idx, w_idx, k_idx, block_table, cache_seqlens, causal)
    idx, n  = dsa_topk(scores, cache_seqlens, topk, causal)
    out, lse = sparse_mla_decode(q, k_cache, block_table, idx, n, softmax_scale)

or all three in one call, sparse_decode(...).  Shapes: q [B, s_q, h_q, 576]
bf16, k_cache [num_blocks, 64, 1, 576] bf16, q_idx [B, s_q, H, 128] bf16,
w_idx [B, s_q, H] fp32, k_idx [num_blocks, 64, 128] bf16 (paged by the same
block_table), idx [B, s_q, topk] int32 token positions (ascending, -1 padded)
-> out [B, s_q, h_q, 512] bf16, lse [B, h_q, s_q] fp32.  Every step is a
CUDA kernel of libgqa_decode_b200.so; there is no fallback.
"""

import threading

import torch

import mla_decode
from binding import _ext

PAGE = 64

_tbl_lock = threading.Lock()
_tbl_cache = {}


def _identity_table(rows, pages_per_row, device):
    """block_table [rows, pages_per_row] = arange: row r's gathered tokens sit
    in pages r * pages_per_row ..  Cached per shape and device."""
    device = torch.device(device)
    key = (rows, pages_per_row, device.type, device.index)
    with _tbl_lock:
        t = _tbl_cache.get(key)
        if t is None:
            t = torch.arange(rows * pages_per_row, dtype=torch.int32,
                             device=device).view(rows, pages_per_row)
            _tbl_cache[key] = t
        return t


def dsa_indexer(q_idx, w_idx, k_idx, block_table, cache_seqlens, causal=False):
    """Lightning-indexer scores [B, s_q, max_blocks * 64] fp32: column t of
    row (b, i) is sum_j w[b, i, j] * relu(q_idx[b, i, j] . k_idx[t]) for the
    tokens (b, i) sees, -inf for the causally hidden ones; columns at or past
    cache_seqlens[b] are not written."""
    return _ext.dsa_indexer(q_idx, w_idx, k_idx, block_table, cache_seqlens, bool(causal))


def dsa_topk(scores, cache_seqlens, topk, causal=False):
    """(indices [B, s_q, topk] int32, counts [B, s_q] int32): the topk
    highest-scoring visible tokens of each (b, i), ties to the lower token
    position, in ascending order, -1 padded; counts = min(topk, visible)."""
    return _ext.dsa_topk(scores, cache_seqlens, int(topk), bool(causal))


def dsa_topk_rows(scores, cache_seqlens, topk, block_table, num_blocks, causal=False):
    """dsa_topk plus each selected token's physical row in the paged caches,
    block_table[b, t // 64] * 64 + t % 64 (-1 padded): (indices, counts,
    rows [B, s_q, topk] int32).  The sparse MLA decode then fetches every
    selected row with one load instead of the token -> block -> row chain."""
    return _ext.dsa_topk_rows(scores, cache_seqlens, int(topk), bool(causal), block_table,
                              int(num_blocks))


def dsa_gather(k_cache, block_table, indices):
    """Latent rows of the selected tokens as pages [B * s_q * kpad / 64, 64, 1,
    576] (kpad = topk rounded up to 64; -1 slots are zero rows)."""
    return _ext.dsa_gather(k_cache, block_table, indices)


def sparse_mla_decode(q, k_cache, block_table, indices, counts, softmax_scale=None,
                      num_splits=0, fused=None):
    """Attention of each (b, i) over its selected tokens only (the selection
    already applies any causal mask).  With h_q a multiple of 128 (fused,
    the default there) the MLA kernel fetches the selected cache rows itself
    (TMA gather, four rows per copy); otherwise the rows are gathered into
    contiguous pages and decoded as B * s_q one-query requests of
    counts[b, i] tokens."""
    B, s_q, h_q = q.shape[0], q.shape[1], q.shape[2]
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    k = indices.shape[-1]
    kpad = (k + PAGE - 1) // PAGE * PAGE
    rows = B * s_q
    if fused is None:
        fused = h_q % 128 == 0
    if fused:
        if num_splits == 0:
            num_splits = int(_ext.mla_pick_splits(rows, 1, h_q, kpad // PAGE,
                                                  mla_decode._num_sms(q.device)))
        nbytes = int(_ext.mla_workspace_bytes(B, s_q, h_q, num_splits))
        ws = (mla_decode.workspace(q.device, nbytes) if nbytes
              else torch.empty(0, dtype=torch.uint8, device=q.device))
        return _ext.mla_decode_sparse(q, k_cache, block_table, indices, counts,
                                      float(softmax_scale), int(num_splits), ws)
    pages = dsa_gather(k_cache, block_table, indices)
    table = _identity_table(rows, kpad // PAGE, q.device)
    out, lse = mla_decode.mla_decode(q.reshape(rows, 1, h_q, q.shape[3]), pages, table,
                                     counts.reshape(rows), softmax_scale, causal=False,
                                     num_splits=num_splits)
    return (out.view(B, s_q, h_q, out.shape[-1]),
            lse.view(B, s_q, h_q).permute(0, 2, 1).contiguous())


def sparse_mla_decode_rows(q, k_cache, rows, counts, softmax_scale=None, num_splits=0):
    """sparse_mla_decode (fused, h_q a multiple of 128) over the physical
    cache rows dsa_topk_rows resolved: identical output, one dependent load
    fewer per selected row in the kernel's copy warp."""
    B, s_q, h_q = q.shape[0], q.shape[1], q.shape[2]
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    kpad = (rows.shape[-1] + PAGE - 1) // PAGE * PAGE
    if num_splits == 0:
        num_splits = int(_ext.mla_pick_splits(B * s_q, 1, h_q, kpad // PAGE,
                                              mla_decode._num_sms(q.device)))
    nbytes = int(_ext.mla_workspace_bytes(B, s_q, h_q, num_splits))
    ws = (mla_decode.workspace(q.device, nbytes) if nbytes
          else torch.empty(0, dtype=torch.uint8, device=q.device))
    return _ext.mla_decode_sparse_rows(q, k_cache, rows, counts, float(softmax_scale),
                                       int(num_splits), ws)


def sparse_decode(q, k_cache, q_idx, w_idx, k_idx, block_table, cache_seqlens, topk,
                  softmax_scale=None, causal=False, num_splits=0):
    """The whole sparse decode step: (out, lse, indices).  With h_q a
    multiple of 128 the top-k kernel also resolves the selected tokens'
    cache rows and the MLA kernel reads those."""
    scores = dsa_indexer(q_idx, w_idx, k_idx, block_table, cache_seqlens, causal)
    if q.shape[2] % 128 == 0:
        indices, counts, rows = dsa_topk_rows(scores, cache_seqlens, topk, block_table,
                                              k_cache.shape[0], causal)
        out, lse = sparse_mla_decode_rows(q, k_cache, rows, counts, softmax_scale, num_splits)
        return out, lse, indices
    indices, counts = dsa_topk(scores, cache_seqlens, topk, causal)
    out, lse = sparse_mla_decode(q, k_cache, block_table, indices, counts, softmax_scale,
                                 num_splits)
    return out, lse, indices


get_status = _ext.dsa_get_status
