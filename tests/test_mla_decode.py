"""GPU: MLA latent-cache decode (tcgen05) against the CPU restatement.

Cases follow FlashMLA's dense-decoding test grid (h_q 16 / 32 / 64 / 128,
s_q 1 and 2 with causal masking, ragged cache lengths including partial
pages and one-token requests), on NaN-poisoned caches so any read outside a
request's tokens shows.  Tolerances: out atol = rtol = 1e-2 (bf16 P and
output), lse 1e-3 absolute (fp32 path).
"""

import math

import numpy as np
import pytest
import torch

import cases
import mla_decode
import oracle

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(192)


def run_case(S, s_q, h_q, causal=False, num_splits=1, seed=0):
    case_cpu = cases.make_mla_case(S, s_q, h_q, seed=seed)
    q, kv, bt, sl = (t.cuda() for t in case_cpu)
    out, lse = mla_decode.mla_decode(q, kv, bt, sl, SCALE, causal=causal, num_splits=num_splits)
    torch.cuda.synchronize()
    assert mla_decode.get_status(True) == 0
    ref_out, ref_lse = oracle.mla_ref(*case_cpu, SCALE, causal=causal)
    return out.float().cpu(), lse.cpu(), ref_out, ref_lse


def check(out, lse, ref_out, ref_lse):
    assert torch.isfinite(out).all()
    np.testing.assert_allclose(out.numpy(), ref_out.numpy(), atol=1e-2, rtol=1e-2)
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse), fin)
    np.testing.assert_allclose(lse[fin].numpy(), ref_lse[fin].numpy(), atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("h_q", [16, 32, 64, 128])
def test_single_page_and_partial(h_q):
    check(*run_case([64, 1, 37, 129], 1, h_q))


@pytest.mark.parametrize("h_q", [16, 64, 128])
@pytest.mark.parametrize("num_splits", [1, 3])
def test_long_ragged(h_q, num_splits):
    check(*run_case([1000, 4096, 3, 2049], 1, h_q, num_splits=num_splits, seed=1))


@pytest.mark.parametrize("h_q", [16, 64, 128])
def test_mtp_causal(h_q):
    # s_q = 2 (speculative / MTP decode): query 0 does not see the last token
    check(*run_case([65, 700, 2], 2, h_q, causal=True, seed=2))


def test_empty_request_and_auto_splits():
    case_cpu = cases.make_mla_case([0, 300, 5000], 1, 64, seed=3)
    q, kv, bt, sl = (t.cuda() for t in case_cpu)
    md, cum = mla_decode.get_mla_metadata(sl, 64, 1)
    out, lse = mla_decode.flash_mla_with_kvcache(q, kv, bt, sl, 512, md, cum, SCALE)
    torch.cuda.synchronize()
    assert mla_decode.get_status(True) == 0
    ref_out, ref_lse = oracle.mla_ref(*case_cpu, SCALE)
    check(out.float().cpu(), lse.cpu(), ref_out, ref_lse)
    assert torch.all(out[0] == 0)


@pytest.mark.parametrize("s_q,h_q,causal", [(1, 1, False), (1, 3, False), (2, 63, True),
                                             (1, 100, False), (2, 9, True)])
def test_any_head_count(s_q, h_q, causal):
    # FlashMLA's test grid also covers head counts that are not multiples of
    # 16 (h_q 1, 3, 9, 63, 126): the last row group of a request is padded
    check(*run_case([129, 64, 1000], s_q, h_q, causal=causal, num_splits=2, seed=5))


def test_splits_agree():
    # the same request decoded with 1, 2 and 5 splits (combine kernel)
    case = tuple(t.cuda() for t in cases.make_mla_case([3000, 777], 1, 32, seed=4))
    outs = [mla_decode.mla_decode(*case, SCALE, num_splits=n)[0].float() for n in (1, 2, 5)]
    for o in outs[1:]:
        torch.testing.assert_close(o, outs[0], atol=1e-2, rtol=1e-2)
