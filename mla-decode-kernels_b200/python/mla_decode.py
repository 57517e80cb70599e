"""MLA absorbed-path paged decode (latent cache) on B200: FlashMLA-shaped API.

The reference names FlashMLA as the baseline of its K2 roadmap kernel
(README.md "Roadmap"; docs/k1/notes_w1.md:97-121 quotes its interface and
accounting) and ships no K2 code.  These two calls keep FlashMLA's argument
names and shapes so a FlashMLA caller switches by changing the import:

    tile_md, num_splits = get_mla_metadata(cache_seqlens, s_q * h_q // h_kv, h_kv)
    out, lse = flash_mla_with_kvcache(q, k_cache, block_table, cache_seqlens, 512,
                                      tile_md, num_splits, softmax_scale, causal)

q [B, s_q, h_q, 576] bf16, k_cache [num_blocks, 64, 1, 576] bf16 (V = dims
0..511), block_table [B, max_blocks] int32, cache_seqlens [B] int32 ->
out [B, s_q, h_q, 512] bf16, lse [B, h_q, s_q] fp32.  The kernel is
tcgen05-only (sm_100a); there is no fallback.
"""

import threading

import torch

from binding import _ext

_NUM_SMS = {}
_ws_lock = threading.Lock()
_ws_cache = {}


def workspace(device, nbytes):
    """Split-state workspace of at least nbytes, cached per device.  Kept
    apart from binding.workspace, so a GQA decode and an MLA decode never
    overwrite each other's partial states.  Every stream of the
    device shares it: decodes that may run at the same time on different
    streams must not both come through this module (use the C ABI with a
    workspace each, or order the streams)."""
    device = torch.device(device)
    key = (device.type, device.index)
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=device)
            _ws_cache[key] = ws
        return ws


def _num_sms(device):
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    if idx not in _NUM_SMS:
        _NUM_SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _NUM_SMS[idx]


def get_mla_metadata(cache_seqlens, num_heads_per_head_k, num_heads_k, max_pages=None):
    """Split plan for a batch.  Returns (tile_scheduler_metadata, num_splits)
    like FlashMLA: metadata is a CPU int32 tensor [1, 8] whose first entry is
    the split count the decode uses (no device synchronisation: the count
    depends on the batch size and head count; pass max_pages to cap it by the
    longest request), num_splits the cumulative splits per request [B + 1]."""
    if num_heads_k != 1:
        raise ValueError("MLA has one latent kv head (num_heads_k == 1)")
    B = int(cache_seqlens.shape[0])
    rows = int(num_heads_per_head_k)
    ns = int(_ext.mla_pick_splits(B, 1, rows, int(max_pages) if max_pages else 1 << 20,
                                  _num_sms(cache_seqlens.device)))
    md = torch.zeros((1, 8), dtype=torch.int32)
    md[0, 0] = ns
    md[0, 1] = rows
    cum = torch.arange(0, (B + 1) * ns, ns, dtype=torch.int32, device=cache_seqlens.device)
    return md, cum


def flash_mla_with_kvcache(q, k_cache, block_table, cache_seqlens, head_dim_v,
                           tile_scheduler_metadata, num_splits, softmax_scale=None, causal=False):
    """(out [B, s_q, h_q, 512] bf16, softmax_lse [B, h_q, s_q] fp32)."""
    if head_dim_v != 512:
        raise ValueError("head_dim_v must be 512")
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    ns = int(tile_scheduler_metadata[0, 0])
    B, s_q, h_q = q.shape[0], q.shape[1], q.shape[2]
    nbytes = int(_ext.mla_workspace_bytes(B, s_q, h_q, ns))
    ws = workspace(q.device, nbytes) if nbytes else torch.empty(0, dtype=torch.uint8,
                                                                 device=q.device)
    out, lse = _ext.mla_decode(q, k_cache, block_table, cache_seqlens, float(softmax_scale),
                               bool(causal), ns, ws)
    return out, lse


def mla_decode(q, k_cache, block_table, cache_seqlens, softmax_scale, causal=False,
               num_splits=0):
    """Direct entry: num_splits = 0 picks the split count."""
    B, s_q, h_q = q.shape[0], q.shape[1], q.shape[2]
    if num_splits == 0:
        num_splits = int(_ext.mla_pick_splits(B, s_q, h_q, block_table.shape[1],
                                              _num_sms(q.device)))
    nbytes = int(_ext.mla_workspace_bytes(B, s_q, h_q, num_splits))
    ws = workspace(q.device, nbytes) if nbytes else torch.empty(0, dtype=torch.uint8,
                                                                 device=q.device)
    return _ext.mla_decode(q, k_cache, block_table, cache_seqlens, float(softmax_scale),
                           bool(causal), int(num_splits), ws)


get_status = _ext.mla_get_status
