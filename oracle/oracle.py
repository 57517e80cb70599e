"""ctypes front end of the CPU oracle (gqa_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker.  It restates the reference's
python/reference.py (gather_kv :7-18, attention_ref :21-40) in C; its
outputs are pinned against reference.py itself through the fixtures in
tests/golden/.
"""

import ctypes
import json
import os
import subprocess

import numpy as np
import torch

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(ORACLE_DIR, "_build")
REF_LIB = os.path.join(ORACLE_DIR, "_ref", "libref_gqa.so")


def _cpu_has_avx2_fma():
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return " avx2" in flags and " fma" in flags
    except OSError:
        return False


def reference_checkout():
    """Directory of a reference checkout to build checkers from, or None.

    Taken from the GQA_REFERENCE_DIR environment variable, else from the
    "reference_path" BASELINE.json records at the repository root; either
    must be an existing directory holding include/gqa_decode.h.  On a
    machine without the checkout this returns None and the callers skip.
    """
    cand = os.environ.get("GQA_REFERENCE_DIR")
    if not cand:
        try:
            with open(os.path.join(os.path.dirname(ORACLE_DIR), "BASELINE.json")) as f:
                cand = json.load(f).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if cand and os.path.isfile(os.path.join(cand, "include", "gqa_decode.h")):
        return cand
    return None


def build(reference_dir=None):
    """make the oracle (and, with a reference checkout, the _ref kernels)."""
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)
    if reference_dir and os.path.isdir(reference_dir):
        subprocess.run(["make", "-s", "-C", ORACLE_DIR, "ref", f"REF={reference_dir}"], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        name = "liboracle_avx2.so" if _cpu_has_avx2_fma() else "liboracle_base.so"
        path = os.path.join(BUILD_DIR, name)
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        p = ctypes.c_void_p
        i = ctypes.c_int
        f = ctypes.c_float
        L.oracle_attention_ref.argtypes = [p, p, p, p, p, i, i, i, i, i, f, p, i]
        L.oracle_attention_ref.restype = None
        L.oracle_attention_state.argtypes = [p, p, p, p, p, i, i, i, i, i, f, p, p, p, i]
        L.oracle_attention_state.restype = None
        L.oracle_online_softmax.argtypes = [p, p, i, i, p, p, p]
        L.oracle_online_softmax.restype = None
        L.oracle_merge_states.argtypes = [p, p, p, i, i, p, p, p]
        L.oracle_merge_states.restype = None
        i64 = ctypes.c_int64
        L.oracle_nhd_index.argtypes = [i64, i64, i64, i64, i64, i64]
        L.oracle_nhd_index.restype = i64
        L.oracle_mla_ref.argtypes = [p, p, p, p, i, i, i, i, i, f, i, p, p, i]
        L.oracle_mla_ref.restype = None
        L.oracle_dsa_scores.argtypes = [p, p, p, p, p, i, i, i, i, i, i, i, p, i]
        L.oracle_dsa_scores.restype = None
        _lib = L
    return _lib


def default_threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def _bits(t):
    """CPU contiguous uint16 numpy view of a bf16 tensor."""
    t = t.detach().to("cpu").contiguous()
    assert t.dtype == torch.bfloat16
    return t.view(torch.int16).numpy().view(np.uint16)


def _i32(t):
    return np.ascontiguousarray(t.detach().to("cpu").numpy().astype(np.int32, copy=False))


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def attention_ref(q, k_cache, v_cache, block_table, seq_lens, scale, nthreads=None):
    """fp32 out [B, Hq, 128] (torch CPU tensor), reference.py semantics."""
    B, Hq, D = q.shape
    assert D == 128
    Hkv, bs = k_cache.shape[2], k_cache.shape[1]
    qb, kb, vb = _bits(q), _bits(k_cache), _bits(v_cache)
    bt, sl = _i32(block_table), _i32(seq_lens)
    out = np.empty((B, Hq, D), dtype=np.float32)
    lib().oracle_attention_ref(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(bt), _ptr(sl), B, Hq, Hkv, bs,
                               bt.shape[1], float(scale), _ptr(out),
                               nthreads or default_threads())
    return torch.from_numpy(out)


def attention_state(q, k_cache, v_cache, block_table, seq_lens, scale, nthreads=None):
    """Unnormalised (m, l, acc) in natural-log units: m, l [B, Hq], acc [B, Hq, 128]."""
    B, Hq, D = q.shape
    Hkv, bs = k_cache.shape[2], k_cache.shape[1]
    qb, kb, vb = _bits(q), _bits(k_cache), _bits(v_cache)
    bt, sl = _i32(block_table), _i32(seq_lens)
    m = np.empty((B, Hq), dtype=np.float32)
    l = np.empty((B, Hq), dtype=np.float32)
    acc = np.empty((B, Hq, D), dtype=np.float32)
    lib().oracle_attention_state(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(bt), _ptr(sl), B, Hq, Hkv,
                                 bs, bt.shape[1], float(scale), _ptr(m), _ptr(l), _ptr(acc),
                                 nthreads or default_threads())
    return torch.from_numpy(m), torch.from_numpy(l), torch.from_numpy(acc)


def mla_ref(q, kv_cache, block_table, seq_lens, scale, causal=False, nthreads=None):
    """MLA absorbed-path decode on a latent cache (gqa_oracle.c: oracle_mla_ref):
    q [B, s_q, h_q, 576] bf16, kv_cache [num_blocks, page, 1, 576] bf16 ->
    out [B, s_q, h_q, 512] fp32, lse [B, h_q, s_q] fp32 (natural log)."""
    B, s_q, h_q, D = q.shape
    assert D == 576 and kv_cache.shape[-1] == 576 and kv_cache.shape[2] == 1
    page = kv_cache.shape[1]
    qb, kb = _bits(q), _bits(kv_cache)
    bt, sl = _i32(block_table), _i32(seq_lens)
    out = np.empty((B, s_q, h_q, 512), dtype=np.float32)
    lse = np.empty((B, h_q, s_q), dtype=np.float32)
    lib().oracle_mla_ref(_ptr(qb), _ptr(kb), _ptr(bt), _ptr(sl), B, s_q, h_q, page, bt.shape[1],
                         float(scale), int(bool(causal)), _ptr(out), _ptr(lse),
                         nthreads or default_threads())
    return torch.from_numpy(out), torch.from_numpy(lse)


def dsa_scores(q_idx, w_idx, k_idx_cache, block_table, seq_lens, causal=False, smax=None,
               nthreads=None):
    """Indexer scores (gqa_oracle.c: oracle_dsa_scores): q_idx [B, s_q, H, 128]
    bf16, w_idx [B, s_q, H] fp32, k_idx_cache [num_blocks, page, 128] bf16 ->
    [B, s_q, smax] fp32, -inf where the query cannot see the token."""
    B, s_q, H, D = q_idx.shape
    assert D == 128
    page = k_idx_cache.shape[1]
    sl = _i32(seq_lens)
    smax = int(smax if smax is not None else max(1, int(sl.max()) if sl.size else 1))
    qb, kb = _bits(q_idx), _bits(k_idx_cache)
    w = np.ascontiguousarray(w_idx.detach().cpu().numpy().astype(np.float32))
    bt = _i32(block_table)
    out = np.empty((B, s_q, smax), dtype=np.float32)
    lib().oracle_dsa_scores(_ptr(qb), _ptr(w), _ptr(kb), _ptr(bt), _ptr(sl), B, s_q, H, page,
                            bt.shape[1], int(bool(causal)), smax, _ptr(out),
                            nthreads or default_threads())
    return torch.from_numpy(out)


def dsa_topk(scores, k):
    """Top-k token indices per query row of a [..., S] score array: the k
    largest finite scores, ties to the lower token index, returned in
    ascending token order and padded with -1 (numpy restatement of the
    selection; -inf scores are never selected)."""
    sc = np.asarray(scores.detach().cpu().numpy() if hasattr(scores, "detach") else scores,
                    dtype=np.float32)
    flat = sc.reshape(-1, sc.shape[-1])
    out = np.full((flat.shape[0], k), -1, dtype=np.int32)
    idx = np.arange(flat.shape[1])
    for r, row in enumerate(flat):
        fin = np.isfinite(row)
        cand = idx[fin]
        order = np.lexsort((cand, -row[fin]))[:k]
        sel = np.sort(cand[order])
        out[r, :len(sel)] = sel
    return out.reshape(sc.shape[:-1] + (k,))


def dsa_sparse_ref(q, kv_cache, block_table, indices, scale, nthreads=None):
    """Attention of each query position over its selected tokens only:
    q [B, s_q, h_q, 576] bf16, kv_cache [num_blocks, page, 1, 576] bf16,
    indices [B, s_q, k] token positions (-1 = none) -> out [B, s_q, h_q, 512]
    fp32, lse [B, h_q, s_q] fp32.  The selected rows of (b, i) are copied
    into a one-page cache of their own and decoded by oracle_mla_ref, whose
    result does not depend on the order of the tokens beyond rounding."""
    B, s_q, h_q, D = q.shape
    page = kv_cache.shape[1]
    idx = _i32(indices).reshape(B * s_q, -1)
    bt = _i32(block_table)
    k = idx.shape[1]
    kv = kv_cache.reshape(-1, 576)
    rows = torch.zeros((B * s_q, max(k, 1), 1, 576), dtype=kv_cache.dtype)
    counts = np.zeros(B * s_q, dtype=np.int32)
    for r in range(B * s_q):
        sel = idx[r][idx[r] >= 0]
        b = r // s_q
        phys = bt[b, sel // page].astype(np.int64) * page + sel % page
        rows[r, :len(sel), 0] = kv[torch.from_numpy(phys)]
        counts[r] = len(sel)
    table = torch.arange(B * s_q, dtype=torch.int32).view(B * s_q, 1)
    out, lse = mla_ref(q.reshape(B * s_q, 1, h_q, D), rows, table, torch.from_numpy(counts),
                       scale, causal=False, nthreads=nthreads)
    return out.view(B, s_q, h_q, 512), lse.view(B, s_q, h_q).permute(0, 2, 1).contiguous()


def online_softmax(scores, values):
    s = np.ascontiguousarray(scores, dtype=np.float32)
    v = np.ascontiguousarray(values, dtype=np.float32)
    n, dv = v.shape
    m = np.zeros(1, np.float32)
    l = np.zeros(1, np.float32)
    acc = np.zeros(dv, np.float32)
    lib().oracle_online_softmax(_ptr(s), _ptr(v), n, dv, _ptr(m), _ptr(l), _ptr(acc))
    return float(m[0]), float(l[0]), acc


def merge_states(m, l, acc):
    m = np.ascontiguousarray(m, dtype=np.float32)
    l = np.ascontiguousarray(l, dtype=np.float32)
    acc = np.ascontiguousarray(acc, dtype=np.float32)
    n, dv = acc.shape
    mo = np.zeros(1, np.float32)
    lo = np.zeros(1, np.float32)
    ao = np.zeros(dv, np.float32)
    lib().oracle_merge_states(_ptr(m), _ptr(l), _ptr(acc), n, dv, _ptr(mo), _ptr(lo), _ptr(ao))
    return float(mo[0]), float(lo[0]), ao


def nhd_index(p, s, bs, Hkv, h, j):
    return int(lib().oracle_nhd_index(p, s, bs, Hkv, h, j))


def block_table_to_paged(block_table, seq_lens, page_size):
    """CSR form of a dense page table, restating the reference helper
    (bench/baselines/flashinfer_adapter.py:33-51) in numpy:
    n_b = ceil(S_b / page), indptr = [0, cumsum(n)], indices = the first n_b
    ids of each row, last_page_len = S - (n - 1) * page."""
    bt = np.asarray(block_table.detach().cpu().numpy() if hasattr(block_table, "detach")
                    else block_table, dtype=np.int64)
    sl = np.asarray(seq_lens.detach().cpu().numpy() if hasattr(seq_lens, "detach")
                    else seq_lens, dtype=np.int64)
    n = (sl + page_size - 1) // page_size
    indptr = np.zeros(len(sl) + 1, dtype=np.int32)
    indptr[1:] = np.cumsum(n)
    indices = np.concatenate([bt[b, :n[b]] for b in range(len(sl))] or [np.zeros(0)])
    last = (sl - (n - 1) * page_size).astype(np.int32)
    return indptr, indices.astype(np.int32), last


def ref_kernels():
    """The reference's own v1/v2 kernels built for sm_100a (oracle/_ref), or None."""
    if not os.path.exists(REF_LIB):
        return None
    L = ctypes.CDLL(REF_LIB)
    p = ctypes.c_void_p
    i = ctypes.c_int
    f = ctypes.c_float
    L.ref_gqa_decode_v1.argtypes = [p, p, p, p, p, p, i, i, i, i, i, f, p]
    L.ref_gqa_decode_v1.restype = i
    L.ref_gqa_decode_v2.argtypes = [p, p, p, p, p, p, i, i, i, i, i, f, i, p, p, p, p]
    L.ref_gqa_decode_v2.restype = i
    return L
