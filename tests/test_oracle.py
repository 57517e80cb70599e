"""CPU: the oracle pinned against the reference's own outputs and worked examples.

* golden.npz holds python/reference.py:attention_ref outputs (made by
  tests/golden/make_golden.py from the unmodified reference);
* known-answer traces from docs/k1/notes_w1.md (online softmax :74-86,
  split merge :88-95, NHD index :55-68);
* the SDPA cross-check of tests/test_reference.py:13-23.
"""

import math
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import cases
import oracle
from golden.make_golden import golden_cases, input_digest, q_transform

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
SCALE = 1.0 / math.sqrt(128)
# fp32 vs fp32 with a different summation order (the reference's own
# oracle-vs-SDPA check uses 1e-5 max-abs, tests/test_reference.py:23).
PIN_ATOL = 2e-5
PIN_RTOL = 1e-5


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name", list(golden_cases().keys()))
def test_oracle_matches_reference_outputs(golden, name):
    builder, _ = golden_cases()[name]
    q, k, v, bt, sl = builder()
    q = q_transform(name, q)
    assert input_digest((q, k, v, bt, sl)) == str(golden[name + "/digest"]), \
        "regenerated inputs differ from the ones the fixture was made from"
    out = oracle.attention_ref(q, k, v, bt, sl, SCALE).numpy()
    ref = golden[name + "/out"]
    assert np.isfinite(ref).all()
    np.testing.assert_allclose(out, ref, atol=PIN_ATOL, rtol=PIN_RTOL)


def test_empty_request_is_zero(golden):
    # reference.py returns zeros for seq_len == 0 (softmax of an empty row).
    ref = golden["empty_request/out"]
    assert np.all(ref[1] == 0.0)


def test_online_softmax_trace():
    # docs/k1/notes_w1.md:74-86: scores [2,5,1,6], 2-d values.
    scores = [2.0, 5.0, 1.0, 6.0]
    values = [[1, 0], [0, 1], [1, 1], [2, 0]]
    m, l, acc = oracle.online_softmax(scores, values)
    assert m == 6.0
    assert l == pytest.approx(1.392933, abs=1e-6)
    np.testing.assert_allclose(acc, [2.025054, 0.374618], atol=1e-6)
    np.testing.assert_allclose(acc / l, [1.4538, 0.2689], atol=1e-4)


def test_split_merge_trace():
    # docs/k1/notes_w1.md:88-95: split {t0,t1} and {t2,t3}, merged.
    values = np.array([[1, 0], [0, 1], [1, 1], [2, 0]], dtype=np.float32)
    m1, l1, a1 = oracle.online_softmax([2.0, 5.0], values[:2])
    m2, l2, a2 = oracle.online_softmax([1.0, 6.0], values[2:])
    assert (m1, m2) == (5.0, 6.0)
    assert l1 == pytest.approx(1.049787, abs=1e-6)
    assert l2 == pytest.approx(1.006738, abs=1e-6)
    np.testing.assert_allclose(a1, [0.049787, 1.0], atol=1e-6)
    np.testing.assert_allclose(a2, [2.006738, 0.006738], atol=1e-6)
    M, L, A = oracle.merge_states([m1, m2], [l1, l2], np.stack([a1, a2]))
    assert M == 6.0
    assert L == pytest.approx(1.392933, abs=1e-6)
    np.testing.assert_allclose(A, [2.025054, 0.374617], atol=2e-6)
    np.testing.assert_allclose(A / L, [1.4538, 0.2689], atol=1e-4)


def test_merge_all_empty_is_neutral():
    M, L, A = oracle.merge_states([-np.inf, -np.inf], [0.0, 0.0], np.zeros((2, 3)))
    assert M == -np.inf and L == 0.0 and np.all(A == 0)


def test_nhd_index_worked_example():
    # docs/k1/notes_w1.md:59-68: bs=16, Hkv=8, h=3, t=20, block_table=[9,2,14].
    bt = [9, 2, 14]
    t, bs = 20, 16
    idx = oracle.nhd_index(bt[t // bs], t % bs, bs, 8, 3, 0)
    assert idx == 37248
    assert idx * 2 == 74496
    # int32 overflow point noted at notes_w1.md:70-72: 2^32 elements.
    assert oracle.nhd_index(128 * 32768 // 16, 0, 16, 8, 0, 0) == 2 ** 32


@pytest.mark.parametrize("B,S,Hq,Hkv", [(2, [37, 100], 32, 8), (1, [1], 32, 8),
                                        (3, [16, 17, 64], 64, 8)])
def test_oracle_matches_sdpa(B, S, Hq, Hkv):
    # Shapes of tests/test_reference.py:14-20, identity block table.
    g = torch.Generator().manual_seed(0)
    bs = 16
    max_blocks = (max(S) + bs - 1) // bs
    nblk = B * max_blocks
    q = torch.randn(B, Hq, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(nblk, bs, Hkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(nblk, bs, Hkv, 128, generator=g).to(torch.bfloat16)
    bt = torch.arange(nblk, dtype=torch.int32).reshape(B, max_blocks)
    sl = torch.tensor(S, dtype=torch.int32)
    out = oracle.attention_ref(q, k, v, bt, sl, SCALE)
    grp = Hq // Hkv
    for b in range(B):
        Kb = k.float()[bt[b].long()].reshape(-1, Hkv, 128)[:S[b]]
        Vb = v.float()[bt[b].long()].reshape(-1, Hkv, 128)[:S[b]]
        Ke = Kb.permute(1, 0, 2).repeat_interleave(grp, dim=0)
        Ve = Vb.permute(1, 0, 2).repeat_interleave(grp, dim=0)
        o = F.scaled_dot_product_attention(q[b].float().unsqueeze(1), Ke, Ve, scale=SCALE)
        assert (o.squeeze(1) - out[b]).abs().max().item() < 1e-5


def test_state_split_merge_equals_full():
    # Splitting one request's tokens into page ranges and merging the states
    # reproduces the full softmax (the identity the GPU merge relies on).
    q, k, v, bt, sl = cases.make_case([1000], 32, 8, 16, seed=21, poison=False)
    full = oracle.attention_ref(q, k, v, bt, sl, SCALE)
    parts = []
    for t0, t1 in [(0, 320), (320, 656), (656, 1000)]:
        p0, p1 = t0 // 16, (t1 + 15) // 16
        bt_part = bt[:, p0:p1].contiguous()
        parts.append(oracle.attention_state(q, k, v, bt_part,
                                            torch.tensor([t1 - t0], dtype=torch.int32), SCALE))
    for h in range(32):
        M, L, A = oracle.merge_states([p[0][0, h] for p in parts], [p[1][0, h] for p in parts],
                                      np.stack([p[2][0, h].numpy() for p in parts]))
        np.testing.assert_allclose(A / L, full[0, h].numpy(), atol=1e-5, rtol=1e-5)


def test_case_recipe_poisons_unused_storage():
    q, k, v, bt, sl = cases.make_case([17, 65], 32, 8, 16, seed=0)
    used = set(int(x) for x in bt.flatten() if x >= 0)
    for p in range(k.shape[0]):
        if p not in used:
            assert torch.isnan(k[p].float()).all() and torch.isnan(v[p].float()).all()
    last = int(bt[0, 1])
    assert torch.isnan(k[last, 1:].float()).all() and not torch.isnan(k[last, 0].float()).any()


def test_config_recipes():
    sl1 = cases.config1_seq_lens()
    assert len(sl1) == 4 and all(1 <= s <= 512 for s in sl1)
    q, k, v, bt, sl = cases.config1()
    assert k.shape[0] == sum((s + 15) // 16 for s in sl1) + 16
    sl4 = cases.config4_seq_lens()
    assert len(sl4) == 256 and min(sl4) >= 64 and max(sl4) <= 32768
    assert cases.kv_bytes([8192] * 32, 8) == 1 << 30
    assert cases.kv_bytes([262144], 8) == 1 << 30
    assert cases.kv_bytes([32768] * 128, 8) == 16 << 30


def test_block_table_to_paged_known_answer():
    # tests/test_flashinfer_baseline.py:20-31 of the reference.
    bt = np.array([[5, 1, 3], [0, 4, -1]], dtype=np.int32)
    sl = np.array([37, 22], dtype=np.int32)
    indptr, indices, last = oracle.block_table_to_paged(bt, sl, page_size=16)
    assert indptr.tolist() == [0, 3, 5]
    assert indices.tolist() == [5, 1, 3, 0, 4]
    assert last.tolist() == [5, 6]


@pytest.mark.parametrize("S,s_q,h_q,causal", [([1, 70, 200], 1, 16, False),
                                              ([130, 64], 2, 16, True),
                                              ([257], 1, 128, False),
                                              ([5, 300], 2, 32, False)])
def test_mla_oracle_matches_sdpa(S, s_q, h_q, causal):
    # the MLA restatement against torch's fp32 SDPA on the gathered latent cache
    q, kv, bt, sl = cases.make_mla_case(S, s_q, h_q, seed=4, poison=True)
    scale = 1.0 / math.sqrt(192)
    out, lse = oracle.mla_ref(q, kv, bt, sl, scale, causal=causal)
    page = kv.shape[1]
    for b, Sb in enumerate(S):
        n = (Sb + page - 1) // page
        K = kv.float()[bt[b, :n].long()].reshape(-1, 576)[:Sb]
        qb = q[b].float()  # [s_q, h_q, 576]
        sc = torch.einsum("ihd,td->iht", qb, K) * scale
        if causal:
            t = torch.arange(Sb)
            mask = t[None, :] < (Sb - s_q + 1 + torch.arange(s_q))[:, None]
            sc = sc.masked_fill(~mask[:, None, :], float("-inf"))
        ref = torch.softmax(sc, dim=-1) @ K[:, :512]
        np.testing.assert_allclose(out[b].numpy(), ref.numpy(), atol=2e-5, rtol=1e-4)
        ref_lse = torch.logsumexp(sc, dim=-1).transpose(0, 1)  # [h_q, s_q]
        np.testing.assert_allclose(lse[b].numpy(), ref_lse.numpy(), atol=1e-4, rtol=1e-5)


def test_mla_oracle_empty_request():
    q, kv, bt, sl = cases.make_mla_case([0, 10], 1, 16, seed=5)
    out, lse = oracle.mla_ref(q, kv, bt, sl, 0.07)
    assert torch.all(out[0] == 0) and torch.all(torch.isinf(lse[0])) and torch.all(lse[0] < 0)
    assert torch.isfinite(out[1]).all()


@pytest.mark.parametrize("S,s_q,causal", [([5, 130, 64], 1, False), ([70, 200], 2, True)])
def test_dsa_scores_match_torch(S, s_q, causal):
    q, kv, q_idx, w_idx, k_idx, bt, sl = cases.make_dsa_case(S, s_q, 16, n_idx_heads=8, seed=6)
    sc = oracle.dsa_scores(q_idx, w_idx, k_idx, bt, sl, causal=causal)
    page = k_idx.shape[1]
    for b, Sb in enumerate(S):
        n = (Sb + page - 1) // page
        K = k_idx.float()[bt[b, :n].long()].reshape(-1, 128)[:Sb]
        dots = torch.einsum("ihd,td->iht", q_idx[b].float(), K).clamp_min(0)
        ref = torch.einsum("ih,iht->it", w_idx[b], dots)
        for i in range(s_q):
            vis = Sb - s_q + 1 + i if causal else Sb
            np.testing.assert_allclose(sc[b, i, :vis].numpy(), ref[i, :vis].numpy(), rtol=1e-4,
                                       atol=1e-4)
            assert torch.all(torch.isinf(sc[b, i, vis:]))


def test_dsa_topk_ties_order_and_padding():
    row = np.array([1.0, 3.0, 3.0, -np.inf, 2.0, 3.0, 0.5], dtype=np.float32)
    # three 3.0 ties: the lower indices win when only two fit
    assert oracle.dsa_topk(row[None], 2).tolist() == [[1, 2]]
    assert oracle.dsa_topk(row[None], 4).tolist() == [[1, 2, 4, 5]]
    # more slots than finite scores: -1 padding, -inf never selected
    assert oracle.dsa_topk(row[None], 8).tolist() == [[0, 1, 2, 4, 5, 6, -1, -1]]


def test_dsa_sparse_ref_matches_torch():
    S, s_q, h_q = [90, 3, 200], 2, 16
    q, kv, q_idx, w_idx, k_idx, bt, sl = cases.make_dsa_case(S, s_q, h_q, n_idx_heads=8, seed=7)
    sc = oracle.dsa_scores(q_idx, w_idx, k_idx, bt, sl, causal=True)
    idx = torch.from_numpy(oracle.dsa_topk(sc, 40))
    scale = 0.05
    out, lse = oracle.dsa_sparse_ref(q, kv, bt, idx, scale)
    page = kv.shape[1]
    for b in range(len(S)):
        for i in range(s_q):
            sel = idx[b, i][idx[b, i] >= 0].long()
            assert len(sel) == min(40, S[b] - s_q + 1 + i)
            rows = kv[bt[b, sel // page].long(), sel % page, 0].float()
            s = q[b, i].float() @ rows.T * scale
            p = torch.softmax(s, -1)
            np.testing.assert_allclose(out[b, i].numpy(), (p @ rows[:, :512]).numpy(),
                                       rtol=1e-4, atol=1e-5)
            np.testing.assert_allclose(lse[b, :, i].numpy(), torch.logsumexp(s, -1).numpy(),
                                       rtol=1e-5, atol=1e-5)
