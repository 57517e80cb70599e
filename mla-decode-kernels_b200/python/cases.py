"""Seeded synthetic paged-KV decode inputs.

The reference measures on synthetic data only (bench/common.py:16-46,
tests/test_gqa_decode.py:27-69); nothing here stands in for a dataset.  One
recipe builds every case, on CPU (bit-identical inputs for the CPU oracle)
or directly on a GPU for the large configurations:

  gen = torch.Generator(gen_device).manual_seed(seed)
  q  = randn(B, Hq, 128)                 * value_scale          -> bf16
  K  = randn(pool, bs, Hkv, 128)         * value_scale * k_scale -> bf16
  V  = randn(pool, bs, Hkv, 128)         * value_scale          -> bf16
  perm = randperm(pool)                   (physical block order)
  block_table[b, :n_b] = next n_b entries of perm, -1 after
  poison: unused blocks and the tail slots of each last block = NaN,
          so any read outside a request's tokens poisons its output.

Named configurations follow BASELINE.json's five configs and the
reference's test case table (tests/test_gqa_decode.py:89-98).
"""

import math

import torch

D = 128


def _randn_bf16(shape, gen, scale, device, chunk_rows=2048):
    """randn(shape) * scale as bf16, generated in chunks of the first dim so
    the fp32 temporary stays small for multi-GiB caches."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=device)
    n = shape[0]
    for s in range(0, n, chunk_rows):
        e = min(n, s + chunk_rows)
        t = torch.randn((e - s,) + tuple(shape[1:]), generator=gen, device=device)
        if scale != 1.0:
            t.mul_(scale)
        out[s:e].copy_(t)
    return out


def make_case(seq_lens, Hq, Hkv, bs, *, seed=0, pool_factor=2.0, pool_blocks=None,
              extra_blocks=0, poison=True, value_scale=1.0, k_scale=1.0, device="cpu",
              gen=None):
    """Build (q, k_cache, v_cache, block_table, seq_lens) per the recipe above.

    pool = pool_blocks if given, else ceil(need * pool_factor) + extra_blocks.
    """
    seq_lens = [int(s) for s in seq_lens]
    B = len(seq_lens)
    device = torch.device(device)
    if gen is None:
        gen = torch.Generator(device=device).manual_seed(seed)
    n_blocks = [(s + bs - 1) // bs for s in seq_lens]
    need = sum(n_blocks)
    if pool_blocks is None:
        pool = max(need, int(math.ceil(need * pool_factor))) + extra_blocks
    else:
        pool = int(pool_blocks)
    assert pool >= need and pool >= 1
    max_blocks = max(1, max(n_blocks) if n_blocks else 1)

    q = _randn_bf16((B, Hq, D), gen, value_scale, device)
    k_cache = _randn_bf16((pool, bs, Hkv, D), gen, value_scale * k_scale, device)
    v_cache = _randn_bf16((pool, bs, Hkv, D), gen, value_scale, device)

    perm = torch.randperm(pool, generator=gen, device=device).to(torch.int32)
    block_table = torch.full((B, max_blocks), -1, dtype=torch.int32, device=device)
    rows = torch.repeat_interleave(torch.arange(B, device=device),
                                   torch.tensor(n_blocks, device=device, dtype=torch.long))
    cols = torch.cat([torch.arange(n, device=device) for n in n_blocks]) if need else \
        torch.empty(0, dtype=torch.long, device=device)
    if need:
        block_table[rows, cols] = perm[:need]
    if poison:
        unused = perm[need:].long()
        if unused.numel():
            k_cache[unused] = float("nan")
            v_cache[unused] = float("nan")
        for b, s in enumerate(seq_lens):
            rem = s % bs
            if s > 0 and rem:
                last = int(block_table[b, n_blocks[b] - 1])
                k_cache[last, rem:] = float("nan")
                v_cache[last, rem:] = float("nan")
    sl = torch.tensor(seq_lens, dtype=torch.int32, device=device)
    return q, k_cache, v_cache, block_table, sl


def subset(case, requests):
    """CPU copy of the given requests with a compact block pool, for the
    oracle when the full case lives on a GPU."""
    q, k_cache, v_cache, block_table, seq_lens = case
    idx = torch.as_tensor(list(requests), dtype=torch.long, device=q.device)
    sl = seq_lens[idx].to("cpu")
    bs = k_cache.shape[1]
    n_blocks = [(int(s) + bs - 1) // bs for s in sl]
    max_blocks = max(1, max(n_blocks))
    bt = block_table[idx][:, :max_blocks].to("cpu")
    blocks = torch.cat([bt[i, :n] for i, n in enumerate(n_blocks)]).long()
    k_small = k_cache[blocks.to(k_cache.device)].to("cpu")
    v_small = v_cache[blocks.to(v_cache.device)].to("cpu")
    bt_new = torch.full((len(n_blocks), max_blocks), -1, dtype=torch.int32)
    off = 0
    for i, n in enumerate(n_blocks):
        bt_new[i, :n] = torch.arange(off, off + n, dtype=torch.int32)
        off += n
    return q[idx].to("cpu"), k_small, v_small, bt_new, sl


def kv_bytes(seq_lens, Hkv):
    """Algorithmic KV bytes of one decode step: sum_b S_b * Hkv * 128 * 2 (K, V) * 2 B
    (bench/common.py:67-68 for uniform S)."""
    total = int(torch.as_tensor(seq_lens, dtype=torch.int64).clamp_min(0).sum())
    return total * Hkv * D * 2 * 2


# ---- the reference's GPU test cases (tests/test_gqa_decode.py:89-98) -------

REF_CASES = {
    "a_base": dict(S_list=[100, 257, 512, 33], Hq=32, Hkv=8, bs=16),
    "b_long": dict(S_list=[1000], Hq=32, Hkv=8, bs=16),
    "c_len1": dict(S_list=[1], Hq=32, Hkv=8, bs=16),
    "d_exact_blocks": dict(S_list=[16, 64], Hq=32, Hkv=8, bs=16),
    "e_partial_blocks": dict(S_list=[17, 65], Hq=32, Hkv=8, bs=16),
    "f_bs64": dict(S_list=[100, 257, 512, 33], Hq=32, Hkv=8, bs=64),
    "g_hq64": dict(S_list=[100, 257, 512, 33], Hq=64, Hkv=8, bs=16),
    "i_8k": dict(S_list=[8192, 8192], Hq=32, Hkv=8, bs=16),
}


def ref_case(name, seed=0, device="cpu"):
    """A reference test case: N(0, 0.5^2) data, 2x pool, NaN poisoning."""
    c = REF_CASES[name]
    return make_case(c["S_list"], c["Hq"], c["Hkv"], c["bs"], seed=seed, pool_factor=2.0,
                     value_scale=0.5, device=device)


# ---- BASELINE.json configurations -------------------------------------------

def config1_seq_lens(seed=0):
    """Config 1: B=4, seq_lens uniform in [1, 512] from seed 0."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(1, 513, (4,), generator=g).tolist()


def config1(device="cpu", seed=0):
    """CPU oracle config: B=4, Hq=32, Hkv=8, bs=16, pool = sum(ceil(S/16)) + 16."""
    sl = config1_seq_lens(seed)
    need = sum((s + 15) // 16 for s in sl)
    return make_case(sl, 32, 8, 16, seed=seed, pool_blocks=need + 16, device=device)


def config2(device="cuda", seed=2, B=32, S=8192):
    """Representative: Hq=32, Hkv=8, bs=16, every S=8192, 16384 permuted blocks (1 GiB KV)."""
    return make_case([S] * B, 32, 8, 16, seed=seed, pool_factor=1.0, device=device)


def config3(device="cuda", seed=3, B=16, S=32768):
    """Wide group: Hq=64, Hkv=8, bs=64, S=32768 (16 requests per GPU; 2 GiB KV per 16)."""
    return make_case([S] * B, 64, 8, 64, seed=seed, pool_factor=1.0, device=device)


def config4_seq_lens(seed=1, B=256):
    """Config 4: seq_lens log-uniform in [64, 32768] from seed 1 (exp(U[ln 64, ln 32768]))."""
    g = torch.Generator().manual_seed(seed)
    u = torch.rand(B, generator=g, dtype=torch.float64)
    s = torch.exp(math.log(64) + u * (math.log(32768) - math.log(64)))
    return torch.round(s).to(torch.int64).clamp(64, 32768).tolist()


def config4(device="cuda", seed=1, B=256):
    """Ragged: Hq=32, Hkv=8, bs=16, pool = ceil(need / 0.9), unused blocks NaN-poisoned."""
    sl = config4_seq_lens(seed, B)
    need = sum((s + 15) // 16 for s in sl)
    return make_case(sl, 32, 8, 16, seed=seed, pool_blocks=int(math.ceil(need / 0.9)),
                     device=device)


def config5(device="cuda", seed=5, S=262144, k_scale=1.0):
    """Long context: B=1, S=262144, Hq=32, Hkv=8, bs=64 (4096 blocks, 1 GiB KV);
    k_scale=8 gives the peaked-softmax variant."""
    return make_case([S], 32, 8, 64, seed=seed, pool_factor=1.0, k_scale=k_scale,
                     device=device)


# ---- MLA latent-cache cases (K2) -------------------------------------------
#
# Same recipe on FlashMLA's layouts: q [B, s_q, h_q, 576], one latent kv head
# kv_cache [pool, page, 1, 576] (K = all 576 dims, V = the first 512), pages
# of 64 tokens, a permuted page table and NaN-poisoned unused slots.

MLA_D, MLA_DV = 576, 512


def make_mla_case(seq_lens, s_q, h_q, page=64, *, seed=0, pool_factor=2.0, poison=True,
                  value_scale=1.0, device="cpu", gen=None):
    seq_lens = [int(s) for s in seq_lens]
    B = len(seq_lens)
    device = torch.device(device)
    if gen is None:
        gen = torch.Generator(device=device).manual_seed(seed)
    n_blocks = [(s + page - 1) // page for s in seq_lens]
    need = sum(n_blocks)
    pool = max(need, int(math.ceil(need * pool_factor)), 1)
    max_blocks = max(1, max(n_blocks) if n_blocks else 1)
    q = _randn_bf16((B, s_q, h_q, MLA_D), gen, value_scale, device)
    kv = _randn_bf16((pool, page, 1, MLA_D), gen, value_scale, device)
    perm = torch.randperm(pool, generator=gen, device=device).to(torch.int32)
    block_table = torch.full((B, max_blocks), -1, dtype=torch.int32, device=device)
    off = 0
    for b, n in enumerate(n_blocks):
        block_table[b, :n] = perm[off:off + n]
        off += n
    if poison:
        unused = perm[need:].long()
        if unused.numel():
            kv[unused] = float("nan")
        for b, s in enumerate(seq_lens):
            rem = s % page
            if s > 0 and rem:
                kv[int(block_table[b, n_blocks[b] - 1]), rem:] = float("nan")
    return q, kv, block_table, torch.tensor(seq_lens, dtype=torch.int32, device=device)


def mla_subset(case, requests):
    """CPU copy of some requests of an MLA case with a compact page pool."""
    q, kv, block_table, seq_lens = case
    idx = torch.as_tensor(list(requests), dtype=torch.long, device=q.device)
    sl = seq_lens[idx].to("cpu")
    page = kv.shape[1]
    n_blocks = [(int(s) + page - 1) // page for s in sl]
    max_blocks = max(1, max(n_blocks))
    bt = block_table[idx][:, :max_blocks].to("cpu")
    blocks = torch.cat([bt[i, :n] for i, n in enumerate(n_blocks)]).long()
    kv_small = kv[blocks.to(kv.device)].to("cpu")
    bt_new = torch.full((len(n_blocks), max_blocks), -1, dtype=torch.int32)
    off = 0
    for i, n in enumerate(n_blocks):
        bt_new[i, :n] = torch.arange(off, off + n, dtype=torch.int32)
        off += n
    return q[idx].to("cpu"), kv_small, bt_new, sl


def mla_kv_bytes(seq_lens):
    """Latent-cache bytes one decode step reads: sum_b S_b * 576 * 2 B (FlashMLA's
    byte count without q and out, tests/test_flash_mla_dense_decoding.py:177-190
    as quoted in docs/k1/notes_w1.md:107-113)."""
    total = int(torch.as_tensor(seq_lens, dtype=torch.int64).clamp_min(0).sum())
    return total * MLA_D * 2


def mla_flops(seq_lens, s_q, h_q, causal=False):
    """FlashMLA's FLOP count: per query row 2 * S * (576 + 512) (no causal discount)."""
    total = int(torch.as_tensor(seq_lens, dtype=torch.int64).clamp_min(0).sum())
    return total * s_q * h_q * 2 * (MLA_D + MLA_DV)


# ---- DSA-style sparse decode cases (K3) -------------------------------------
#
# The MLA case plus DeepSeek-sparse-attention indexer inputs: index queries
# q_idx [B, s_q, H, 128], per-head weights w_idx [B, s_q, H] and an index-key
# cache k_idx [num_blocks, 64, 128] paged by the same block table.

DSA_D = 128


def make_dsa_case(seq_lens, s_q, h_q, n_idx_heads=64, page=64, *, seed=0, pool_factor=2.0,
                  poison=True, device="cpu"):
    gen = torch.Generator(device=torch.device(device)).manual_seed(seed)
    q, kv, bt, sl = make_mla_case(seq_lens, s_q, h_q, page, seed=seed, pool_factor=pool_factor,
                                  poison=poison, device=device, gen=gen)
    B = len(seq_lens)
    pool = kv.shape[0]
    q_idx = _randn_bf16((B, s_q, n_idx_heads, DSA_D), gen, 1.0, device)
    w_idx = (torch.randn((B, s_q, n_idx_heads), generator=gen, device=device)
             / math.sqrt(n_idx_heads)).float()
    k_idx = _randn_bf16((pool, page, DSA_D), gen, 1.0, device)
    if poison:
        used = torch.zeros(pool, dtype=torch.bool, device=device)
        for b, s in enumerate(seq_lens):
            n = (int(s) + page - 1) // page
            used[bt[b, :n].long()] = True
            rem = int(s) % page
            if s > 0 and rem:
                k_idx[int(bt[b, n - 1]), rem:] = float("nan")
        k_idx[~used] = float("nan")
    return q, kv, q_idx, w_idx, k_idx, bt, sl
