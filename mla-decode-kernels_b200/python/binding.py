"""PyTorch entry points of the B200 paged GQA decode engine.

Drop-in for the reference's python/binding.py (yuqiz7/mla-decode-kernels):
``gqa_decode_v0``, ``gqa_decode_v1``, ``gqa_decode_v2(..., num_splits=8)``
and the ``KERNELS`` registry (reference binding.py:25-31), with the same
argument names, defaults and validation errors.  The reference JIT-builds an
sm_90a extension at import; this module loads the in-tree sm_100a build
(building it first if it is missing) and fails loudly if that is impossible -
there is no CPU or eager fallback.

Additions:
  * ``gqa_decode(..., num_splits=0)``: the balanced single-launch schedule
    (``num_splits=0``) or fixed splits, with a cached per-device workspace;
    ``gqa_decode_v2(..., num_splits="auto")`` routes there too.
  * ``gqa_decode_partial`` / ``merge_states``: unnormalised softmax states
    for sharding one request's KV range across GPUs.
"""

import importlib.util
import os
import sys
import threading

import torch

_PY_DIR = os.path.dirname(os.path.abspath(__file__))
if _PY_DIR not in sys.path:
    sys.path.insert(0, _PY_DIR)

import gqa_build as _build  # noqa: E402


def _load_ext():
    if not os.path.exists(_build.LIB_PATH):
        _build.build_lib()
    _build.preload_lib()
    if not os.path.exists(_build.EXT_PATH):
        _build.build_ext()
    spec = importlib.util.spec_from_file_location(_build.EXT_NAME, _build.EXT_PATH)
    if spec is None:
        raise ImportError(f"cannot load {_build.EXT_PATH}")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


_ext = _load_ext()

LIB_PATH = _build.LIB_PATH
EXT_PATH = _build.EXT_PATH

gqa_decode_v0 = _ext.gqa_decode_v0
gqa_decode_v1 = _ext.gqa_decode_v1
merge_states = _ext.merge_states
get_status = _ext.get_status
pick_splits = _ext.pick_splits

_ws_lock = threading.Lock()
_ws_cache = {}


def workspace(device, nbytes):
    """uint8 workspace of at least nbytes on device, cached.

    The balanced schedule keeps its per-launch records and partial states
    there (every launch writes what it reads, so no zeroing is needed).
    Every stream of the device shares it: decodes that may run at the same
    time on different streams must not both use it (pass each its own
    workspace through the C ABI, or order the streams).
    """
    device = torch.device(device)
    key = (device.type, device.index)
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(int(nbytes), 1 << 20)
            if ws is not None:
                size = max(size, 2 * ws.numel())
            ws = torch.zeros(size, dtype=torch.uint8, device=device)
            _ws_cache[key] = ws
        return ws


def gqa_decode(q, k_cache, v_cache, block_table, seq_lens, scale, num_splits=0,
               check_blocks=True, out=None):
    """Paged GQA decode; num_splits=0 picks the balanced schedule.

    check_blocks validates every block id against k_cache.shape[0] in the
    kernel (an out-of-range id sets bit 1 of ``get_status()``).
    """
    if num_splits == "auto":
        num_splits = 0
    nbytes = _ext.workspace_bytes(q.shape[0], q.shape[1], k_cache.shape[2], int(num_splits)) \
        if q.is_cuda else 0
    ws = workspace(q.device, nbytes) if q.is_cuda else torch.empty(0, dtype=torch.uint8)
    return _ext.gqa_decode(q, k_cache, v_cache, block_table, seq_lens, float(scale),
                           int(num_splits), ws, bool(check_blocks), out)


def gqa_decode_v2(q, k_cache, v_cache, block_table, seq_lens, scale, num_splits=8):
    """Split-KV decode; identical contract to the reference's v2 (num_splits
    in [1, 512], default 8).  num_splits="auto" selects the balanced
    schedule of :func:`gqa_decode`."""
    if num_splits == "auto":
        return gqa_decode(q, k_cache, v_cache, block_table, seq_lens, scale, 0)
    return _ext.gqa_decode_v2(q, k_cache, v_cache, block_table, seq_lens, scale,
                              num_splits=num_splits)


def gqa_decode_partial(q, k_cache, v_cache, block_table, seq_lens, scale, check_blocks=True):
    """Unnormalised states (m, l, acc) per (request, q head): m and l [B, Hq]
    in the log2 domain (m = max score*scale*log2(e)), acc [B, Hq, 128]."""
    nbytes = _ext.workspace_bytes(q.shape[0], q.shape[1], k_cache.shape[2], 0)
    ws = workspace(q.device, nbytes)
    return _ext.gqa_decode_partial(q, k_cache, v_cache, block_table, seq_lens, float(scale), ws,
                                   bool(check_blocks))


kvshard_buffer_bytes = _ext.kvshard_buffer_bytes


def gqa_decode_kvshard(q, k_cache, v_cache, block_table, seq_lens, scale, rank, world,
                       peer_ptrs, epoch, check_blocks=True, out=None):
    """KV-range sharded decode with the cross-rank merge fused into the
    decode's merge kernel (epoch-tagged peer stores over NVLink); see
    sharding.P2PKVRangeDecoder.  out: optional [B, Hq, 128] bf16 to write."""
    nbytes = _ext.workspace_bytes(q.shape[0], q.shape[1], k_cache.shape[2], 0)
    ws = workspace(q.device, nbytes)
    return _ext.gqa_decode_kvshard(q, k_cache, v_cache, block_table, seq_lens, float(scale),
                                   int(rank), int(world), [int(x) for x in peer_ptrs], int(epoch),
                                   ws, bool(check_blocks), out)


def block_table_to_paged(block_table, seq_lens, page_size):
    """(kv_indptr [B+1], kv_indices [sum n_b], kv_last_page_len [B]) int32 on
    block_table's device, from a dense page table: the reference's helper
    (bench/baselines/flashinfer_adapter.py:33-51) computed by one GPU kernel.
    Reads kv_indptr[B] back to size kv_indices (one host synchronisation)."""
    indptr, indices, last = _ext.block_table_to_csr(block_table, seq_lens, int(page_size))
    n = int(indptr[-1].item())
    return indptr, indices[:n], last


class BatchDecodeWithPagedKVCacheWrapper:
    """plan() / run() over a CSR page table, shaped like the FlashInfer
    wrapper the reference benchmarks against (bench/baselines/
    flashinfer_adapter.py:24-66: NHD caches passed as (k_cache, v_cache),
    plan() once per batch shape, run() per decode).  plan() runs on the GPU
    without a host synchronisation; run() only launches, so it can be
    captured in a CUDA graph and repeated (e.g. once per layer) while the
    plan's lengths stay valid."""

    def __init__(self, workspace_buffer=None, kv_layout="NHD"):
        if kv_layout != "NHD":
            raise ValueError("only the NHD page layout [num_blocks, page, Hkv, 128] is supported")
        self._user_ws = workspace_buffer
        self._user_ws_zeroed = False
        self._ws = None
        self._planned = None

    def plan(self, indptr, indices, last_page_len, num_qo_heads, num_kv_heads, head_dim,
             page_size, sm_scale=None, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
             num_blocks=0):
        if head_dim != 128:
            raise ValueError("head_dim must be 128")
        if q_data_type != torch.bfloat16 or kv_data_type != torch.bfloat16:
            raise ValueError("q and kv must be bf16")
        B = last_page_len.shape[0]
        nbytes = _ext.workspace_bytes(B, num_qo_heads, num_kv_heads, 0)
        # The plan and each run's records and partial states live in the
        # workspace, so every wrapper keeps its own: two wrappers planned for
        # different batches (or run on different streams) never share one.
        if self._user_ws is not None:
            if self._user_ws.numel() * self._user_ws.element_size() < nbytes:
                raise ValueError(f"workspace_buffer needs {nbytes} bytes")
            if not self._user_ws_zeroed:
                self._user_ws.zero_()
                self._user_ws_zeroed = True
            self._ws = self._user_ws
        elif self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8,
                                   device=indptr.device)
        _ext.plan_csr(indptr, indices, last_page_len, int(num_qo_heads), int(num_kv_heads),
                      int(page_size), int(num_blocks), self._ws)
        self._planned = (indptr, indices, last_page_len, num_qo_heads, num_kv_heads, page_size,
                         1.0 / 128 ** 0.5 if sm_scale is None else float(sm_scale))

    def run(self, q, paged_kv_cache, out=None, check_blocks=True):
        if self._planned is None:
            raise RuntimeError("plan() must be called before run()")
        indptr, indices, last, Hq, Hkv, page_size, scale = self._planned
        k_cache, v_cache = paged_kv_cache
        if q.shape[1] != Hq or k_cache.shape[2] != Hkv or k_cache.shape[1] != page_size:
            raise ValueError("q / cache shapes differ from the plan")
        return _ext.run_csr(q, k_cache, v_cache, indptr, indices, last, scale, self._ws,
                            bool(check_blocks), out)


# Reference registry (binding.py:31) plus the balanced schedule.
KERNELS = {
    "v0": gqa_decode_v0,
    "v1": gqa_decode_v1,
    "v2": gqa_decode_v2,
    "auto": gqa_decode,
}
