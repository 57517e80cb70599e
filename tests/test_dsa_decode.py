"""GPU: DSA-style sparse decode (indexer, top-k, gather, attention over the
selected tokens) against the CPU restatement.

* indexer scores vs oracle.dsa_scores, rtol 1e-4 / atol 1e-3 (fp32 sums of
  bf16 products in a different order);
* top-k indices bit-exact vs oracle.dsa_topk run on the GPU's own scores
  (the selection is integer work: ties, ordering and -1 padding must agree),
  and on hand-made score rows full of ties;
* gathered rows bit-exact vs the cache rows they name;
* attention out atol = rtol = 1e-2, lse 1e-3 vs oracle.dsa_sparse_ref on the
  same selection; with topk >= S the sparse step equals the dense decode.
Caches are NaN-poisoned past every request's tokens, so a read outside the
visible range shows.
"""

import math

import numpy as np
import pytest
import torch

import cases
import dsa_decode
import mla_decode
import oracle

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(192)


def _cuda(case):
    return tuple(t.cuda() for t in case)


def _scores_visible(scores, S, s_q, causal):
    """GPU scores as a CPU array with the unwritten columns (t >= S_b) set to
    -inf, the oracle's convention."""
    sc = scores.cpu().clone()
    for b, Sb in enumerate(S):
        sc[b, :, Sb:] = -math.inf
    return sc


def _check_status():
    torch.cuda.synchronize()
    assert dsa_decode.get_status(True) == 0
    assert mla_decode.get_status(True) == 0


@pytest.mark.parametrize("S,s_q,H,causal", [
    ([64, 1, 37, 129, 1000], 1, 64, False),
    ([300, 2049, 5], 2, 64, True),
    ([4096, 3, 130], 1, 128, False),
    ([777, 64, 2], 2, 32, True),
])
def test_indexer_matches_oracle(S, s_q, H, causal):
    case = cases.make_dsa_case(S, s_q, 16, n_idx_heads=H, seed=11)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, causal)
    _check_status()
    ref = oracle.dsa_scores(*case[2:], causal=causal, smax=scores.shape[2])
    got = scores.cpu()
    for b, Sb in enumerate(S):
        for i in range(s_q):
            vis = max(0, Sb - s_q + 1 + i) if causal else Sb
            np.testing.assert_allclose(got[b, i, :vis].numpy(), ref[b, i, :vis].numpy(),
                                       rtol=1e-4, atol=1e-3)
            assert torch.all(torch.isneginf(got[b, i, vis:Sb]))


@pytest.mark.parametrize("S,s_q,k,causal", [
    ([5000, 100, 2048, 0], 1, 2048, False),
    ([3000, 9, 700], 2, 512, True),
    ([20000], 1, 64, False),
])
def test_topk_matches_oracle_on_indexer_scores(S, s_q, k, causal):
    case = cases.make_dsa_case(S, s_q, 16, n_idx_heads=64 // s_q, seed=12)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, causal)
    idx, counts = dsa_decode.dsa_topk(scores, sl, k, causal)
    _check_status()
    ref = oracle.dsa_topk(_scores_visible(scores, S, s_q, causal), k)
    assert np.array_equal(idx.cpu().numpy(), ref)
    assert np.array_equal(counts.cpu().numpy(), (ref >= 0).sum(-1))


@pytest.mark.parametrize("levels", [1, 3, 50])
def test_topk_ties(levels):
    # few distinct values (one level: every score ties), +0 and -0 together,
    # negative scores: selection must still take the lowest positions first
    gen = torch.Generator().manual_seed(levels)
    B, s_q, Smax, k = 3, 2, 5000, 1000
    sc = (torch.randint(0, levels, (B, s_q, Smax), generator=gen).float() - levels // 2) * 0.5
    sc[0, 0, ::7] = -0.0
    sl = torch.tensor([5000, 999, 2500], dtype=torch.int32)
    for causal in (False, True):
        idx, counts = dsa_decode.dsa_topk(sc.cuda(), sl.cuda(), k, causal)
        _check_status()
        vis = sc.clone()
        for b in range(B):
            for i in range(s_q):
                v = int(sl[b]) - s_q + 1 + i if causal else int(sl[b])
                vis[b, i, v:] = -math.inf
        assert np.array_equal(idx.cpu().numpy(), oracle.dsa_topk(vis, k))


def test_gather_rows():
    S = [300, 64, 1]
    case = cases.make_dsa_case(S, 1, 16, seed=13)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    idx = torch.full((3, 1, 100), -1, dtype=torch.int32)
    idx[0, 0, :100] = torch.arange(0, 300, 3)
    idx[1, 0, :64] = torch.arange(64)
    idx[2, 0, 0] = 0
    pages = dsa_decode.dsa_gather(kv, bt, idx.cuda())
    _check_status()
    got = pages.cpu().view(3, 128, 576)
    kv_c, bt_c = case[1], case[5]
    for b in range(3):
        for s in range(128):
            t = int(idx[b, 0, s]) if s < 100 else -1
            want = (kv_c[bt_c[b, t // 64].long(), t % 64, 0] if t >= 0
                    else torch.zeros(576, dtype=torch.bfloat16))
            assert torch.equal(got[b, s], want), (b, s)


def _run_sparse(S, s_q, h_q, topk, causal, seed, num_splits=0):
    case = cases.make_dsa_case(S, s_q, h_q, seed=seed)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    out, lse, idx = dsa_decode.sparse_decode(q, kv, q_idx, w_idx, k_idx, bt, sl, topk, SCALE,
                                             causal, num_splits)
    _check_status()
    return case, out.float().cpu(), lse.cpu(), idx.cpu()


def _check_attention(case, out, lse, idx):
    ref_out, ref_lse = oracle.dsa_sparse_ref(case[0], case[1], case[5], idx, SCALE)
    assert torch.isfinite(out).all()
    np.testing.assert_allclose(out.numpy(), ref_out.numpy(), atol=1e-2, rtol=1e-2)
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse), fin)
    np.testing.assert_allclose(lse[fin].numpy(), ref_lse[fin].numpy(), atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("h_q", [16, 64, 128])
def test_sparse_decode(h_q):
    S = [8192, 3000, 2048, 100]
    case, out, lse, idx = _run_sparse(S, 1, h_q, 2048, False, seed=14)
    # the selection is the oracle's on the same (deterministic) scores
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, False)
    ref_idx = oracle.dsa_topk(_scores_visible(scores, S, 1, False), 2048)
    assert np.array_equal(idx.numpy(), ref_idx)
    _check_attention(case, out, lse, idx)


@pytest.mark.parametrize("h_q", [16, 128])
def test_sparse_decode_mtp_causal(h_q):
    case, out, lse, idx = _run_sparse([4000, 700, 3], 2, h_q, 512, True, seed=15)
    assert int(idx[2, 0, 1]) == 1 and int(idx[2, 0, 2]) == -1  # query 0 sees 2 tokens
    _check_attention(case, out, lse, idx)


def test_sparse_with_topk_above_length_is_dense():
    S = [1000, 64, 1, 0]
    case, out, lse, idx = _run_sparse(S, 1, 64, 1024, False, seed=16)
    for b, Sb in enumerate(S):
        assert idx[b, 0, :Sb].tolist() == list(range(Sb))
        assert torch.all(idx[b, 0, Sb:] == -1)
    q, kv, bt, sl = (t.cuda() for t in (case[0], case[1], case[5], case[6]))
    dense_out, dense_lse = mla_decode.mla_decode(q, kv, bt, sl, SCALE)
    _check_status()
    np.testing.assert_allclose(out.numpy(), dense_out.float().cpu().numpy(), atol=1e-2, rtol=1e-2)
    fin = torch.isfinite(dense_lse.cpu())
    np.testing.assert_allclose(lse[fin].numpy(), dense_lse.cpu()[fin].numpy(), atol=1e-3)


def test_indexer_batches_above_one_launch():
    # more requests than one launch takes (4096): the host splits the batch
    gen = torch.Generator().manual_seed(21)
    S = torch.randint(0, 200, (4100,), generator=gen).tolist()
    S[0], S[-1] = 0, 129
    case = cases.make_dsa_case(S, 1, 16, n_idx_heads=64, seed=21, pool_factor=1.2, poison=False)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, False)
    _check_status()
    got = scores.cpu()
    for b in (1, 2, 4095, 4096, 4097, 4099):
        ref = oracle.dsa_scores(case[2][b:b + 1], case[3][b:b + 1], case[4], case[5][b:b + 1],
                                case[6][b:b + 1], smax=max(1, S[b]))
        np.testing.assert_allclose(got[b, 0, :S[b]].numpy(), ref[0, 0, :S[b]].numpy(),
                                   rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("causal", [False, True])
def test_topk_long_rows_from_global_scores(causal):
    # rows longer than the shared-memory key capacity (40960) read the scores
    gen = torch.Generator().manual_seed(22)
    B, s_q, Smax, k = 2, 2, 50000, 2048
    sc = (torch.randint(0, 300, (B, s_q, Smax), generator=gen).float() - 150) * 0.25
    sl = torch.tensor([50000, 41000], dtype=torch.int32)
    idx, counts = dsa_decode.dsa_topk(sc.cuda(), sl.cuda(), k, causal)
    _check_status()
    vis = sc.clone()
    for b in range(B):
        for i in range(s_q):
            v = int(sl[b]) - s_q + 1 + i if causal else int(sl[b])
            vis[b, i, v:] = -math.inf
    assert np.array_equal(idx.cpu().numpy(), oracle.dsa_topk(vis, k))


@pytest.mark.parametrize("s_q,causal", [(1, False), (2, True)])
def test_fused_row_gather_equals_gathered_pages(s_q, causal):
    # the MLA kernel fetching the selected rows itself (TMA gather) and the
    # same kernel over pre-gathered pages run identical tiles in the same
    # order: bit-identical results
    case = cases.make_dsa_case([3000, 700, 100, 2], s_q, 128, seed=23)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, causal)
    idx, counts = dsa_decode.dsa_topk(scores, sl, 640, causal)
    fo, fl = dsa_decode.sparse_mla_decode(q, kv, bt, idx, counts, SCALE, fused=True)
    go, gl = dsa_decode.sparse_mla_decode(q, kv, bt, idx, counts, SCALE, fused=False)
    _check_status()
    assert torch.equal(fo, go)
    assert torch.equal(torch.isfinite(fl), torch.isfinite(gl))
    assert torch.equal(fl[torch.isfinite(fl)], gl[torch.isfinite(gl)])


@pytest.mark.parametrize("h_q,num_splits", [(128, 3), (256, 2)])
def test_fused_row_gather_splits_and_wide_heads(h_q, num_splits):
    # split selections (partial states + combine) and two 128-row groups per
    # query position: still bit-identical to decoding gathered pages, and
    # within tolerance of the oracle
    case = cases.make_dsa_case([5000, 900, 70], 1, h_q, seed=24)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, False)
    idx, counts = dsa_decode.dsa_topk(scores, sl, 1024, False)
    fo, fl = dsa_decode.sparse_mla_decode(q, kv, bt, idx, counts, SCALE, num_splits, fused=True)
    go, gl = dsa_decode.sparse_mla_decode(q, kv, bt, idx, counts, SCALE, num_splits, fused=False)
    _check_status()
    assert torch.equal(fo, go)
    assert torch.equal(fl, gl)
    _check_attention(case, fo.float().cpu(), fl.cpu(), idx.cpu())


@pytest.mark.parametrize("S,s_q,k,causal", [
    ([5000, 100, 2048, 0], 1, 2048, False),
    ([3000, 9, 700], 2, 512, True),
])
def test_topk_rows_resolve_the_page_table(S, s_q, k, causal):
    # the top-k kernel's row output: the same selection as dsa_topk, and each
    # selected token t of request b mapped to block_table[b, t // 64] * 64 +
    # t % 64 (integer work: bit-exact), -1 where the selection is padded
    case = cases.make_dsa_case(S, s_q, 16, n_idx_heads=64 // s_q, seed=25)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, causal)
    idx, counts = dsa_decode.dsa_topk(scores, sl, k, causal)
    idx2, counts2, rows = dsa_decode.dsa_topk_rows(scores, sl, k, bt, kv.shape[0], causal)
    _check_status()
    assert torch.equal(idx, idx2) and torch.equal(counts, counts2)
    tok = idx.long().cpu()
    btc = bt.long().cpu()
    expect = torch.full_like(tok, -1)
    for b in range(tok.shape[0]):
        sel = tok[b] >= 0
        expect[b][sel] = btc[b][tok[b][sel] // 64] * 64 + tok[b][sel] % 64
    assert torch.equal(rows.long().cpu(), expect)


@pytest.mark.parametrize("h_q,num_splits", [(128, 0), (128, 3), (256, 2)])
def test_sparse_decode_over_resolved_rows_equals_token_path(h_q, num_splits):
    # the MLA kernel reading the rows resolved by top-k and the one resolving
    # token -> block -> row itself copy the same rows into the same tiles:
    # bit-identical outputs; the one-call sparse_decode takes the row path
    case = cases.make_dsa_case([5000, 900, 70, 2048], 1, h_q, seed=26)
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, False)
    idx, counts, rows = dsa_decode.dsa_topk_rows(scores, sl, 1024, bt, kv.shape[0], False)
    ro, rl = dsa_decode.sparse_mla_decode_rows(q, kv, rows, counts, SCALE, num_splits)
    to, tl = dsa_decode.sparse_mla_decode(q, kv, bt, idx, counts, SCALE, num_splits, fused=True)
    so, sl2, sidx = dsa_decode.sparse_decode(q, kv, q_idx, w_idx, k_idx, bt, sl, 1024, SCALE,
                                             num_splits=num_splits)
    _check_status()
    assert torch.equal(ro, to) and torch.equal(rl, tl)
    assert torch.equal(so, ro) and torch.equal(sidx, idx)
    _check_attention(case, ro.float().cpu(), rl.cpu(), idx.cpu())


def test_every_device_of_one_process():
    # kernel shared-memory limits are per device: a process that decodes on
    # a second GPU gets the same bits as on the first
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs visible to one process")
    case = cases.make_dsa_case([3000, 2048, 100], 1, 128, seed=16)
    mcase = cases.make_mla_case([700, 64, 2049], 1, 64, seed=17)
    got = []
    for d in range(2):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            q, kv, q_idx, w_idx, k_idx, bt, sl = (t.to(dev) for t in case)
            out, lse, idx = dsa_decode.sparse_decode(q, kv, q_idx, w_idx, k_idx, bt, sl, 2048,
                                                     SCALE, False, 0)
            mq, mkv, mbt, msl = (t.to(dev) for t in mcase)
            mout, mlse = mla_decode.mla_decode(mq, mkv, mbt, msl, SCALE)
            _check_status()
            got.append([t.cpu() for t in (out, lse, idx, mout, mlse)])
    for a, b in zip(*got):
        assert torch.equal(a, b)


def test_rows_out_of_range_raise_status_and_read_block_zero():
    # integer bounds checks of the row path: a block id outside the cache
    # (top-k's resolve) and a row id outside it (the MLA copy warp) each set
    # status bit 1 and read block / row 0 instead; nothing reads outside
    case = cases.make_dsa_case([3000, 900], 1, 128, seed=27, poison=False)  # block 0 is finite
    q, kv, q_idx, w_idx, k_idx, bt, sl = _cuda(case)
    nb = kv.shape[0]
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl, False)
    idx, counts, rows = dsa_decode.dsa_topk_rows(scores, sl, 512, bt, nb, False)
    _check_status()
    bad_bt = bt.clone()
    bad_bt[1, 3] = nb + 5  # request 1, tokens 192..255
    _, _, rows_bad = dsa_decode.dsa_topk_rows(scores, sl, 512, bad_bt, nb, False)
    torch.cuda.synchronize()
    assert dsa_decode.get_status(True) == 2
    tok = idx[1].long()
    hit = (tok >= 192) & (tok < 256)
    assert hit.any()
    assert torch.equal(rows_bad[1][hit].long(), tok[hit] % 64)
    assert torch.equal(rows_bad[1][~hit], rows[1][~hit]) and torch.equal(rows_bad[0], rows[0])
    bad_rows = rows.clone()
    bad_rows[0, 0, 5] = nb * 64 + 7
    out, _ = dsa_decode.sparse_mla_decode_rows(q, kv, bad_rows, counts, SCALE)
    torch.cuda.synchronize()
    assert mla_decode.get_status(True) == 2
    assert torch.isfinite(out.float()).all()
