"""GPU: the CSR page-table front end and the plan/run split.

* gqa_decode_block_table_to_csr against the reference helper's known answer
  (tests/test_flashinfer_baseline.py:20-31 of the reference) and the
  oracle's restatement on ragged tables;
* planned runs (dense and CSR) bitwise equal to the one-launch balanced
  decode (same schedule, same arithmetic);
* the FlashInfer-shaped wrapper on the cases the reference checks its
  FlashInfer baseline on (tests/test_flashinfer_baseline.py:34-52), against
  the oracle at atol = rtol = 1e-2;
* one plan serving several runs (layers) and a CUDA-graph replay of run().
"""

import math

import numpy as np
import pytest
import torch

import binding
import capi
import cases
import oracle

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(128)


def to_gpu(case):
    return tuple(t.cuda() for t in case)


def test_block_table_to_paged_known_answer():
    bt = torch.tensor([[5, 1, 3], [0, 4, -1]], dtype=torch.int32, device="cuda")
    sl = torch.tensor([37, 22], dtype=torch.int32, device="cuda")
    indptr, indices, last = binding.block_table_to_paged(bt, sl, page_size=16)
    assert indptr.tolist() == [0, 3, 5]
    assert indices.tolist() == [5, 1, 3, 0, 4]
    assert last.tolist() == [5, 6]
    for t in (indptr, indices, last):
        assert t.dtype == torch.int32 and t.device == bt.device


@pytest.mark.parametrize("B", [1, 7, 256, 1500])
def test_block_table_to_paged_matches_oracle(B):
    sl = cases.config4_seq_lens(seed=3, B=B)
    bs = 16
    mb = max((s + bs - 1) // bs for s in sl)
    g = torch.Generator().manual_seed(B)
    bt = torch.randint(0, 1 << 20, (B, mb), generator=g, dtype=torch.int32)
    ind_o = oracle.block_table_to_paged(bt, torch.tensor(sl), bs)
    ind_g = binding.block_table_to_paged(bt.cuda(), torch.tensor(sl, dtype=torch.int32).cuda(), bs)
    for a, b in zip(ind_o, ind_g):
        assert np.array_equal(a, b.cpu().numpy())


def csr_of(case):
    q, k, v, bt, sl = case
    return binding.block_table_to_paged(bt, sl, k.shape[1])


@pytest.mark.parametrize("name", ["a_base", "e_partial_blocks", "f_bs64", "g_hq64", "i_8k"])
def test_planned_runs_equal_one_launch(name):
    case = to_gpu(cases.ref_case(name, seed=7))
    q, k, v, bt, sl = case
    expect = capi.auto(*case, SCALE)
    ws = binding.workspace(q.device, binding._ext.workspace_bytes(q.shape[0], q.shape[1],
                                                                 k.shape[2], 0))
    binding._ext.plan_dense(bt, sl, q.shape[1], k.shape[2], k.shape[1], k.shape[0], ws)
    dense = binding._ext.run_dense(q, k, v, bt, sl, SCALE, ws)
    indptr, indices, last = csr_of(case)
    binding._ext.plan_csr(indptr, indices, last, q.shape[1], k.shape[2], k.shape[1], k.shape[0],
                          ws)
    csr = binding._ext.run_csr(q, k, v, indptr, indices, last, SCALE, ws)
    torch.cuda.synchronize()
    assert capi.status() == 0
    assert torch.equal(dense, expect)
    assert torch.equal(csr, expect)


def test_planned_csr_ragged_with_empty_requests():
    sl = cases.config4_seq_lens(seed=1, B=40)
    sl[3] = 0
    sl[17] = 1
    case = to_gpu(cases.make_case(sl, 32, 8, 16, seed=8, pool_factor=1.0 / 0.9))
    q, k, v, bt, sl_t = case
    w = binding.BatchDecodeWithPagedKVCacheWrapper()
    indptr, indices, last = csr_of(case)
    w.plan(indptr, indices, last, 32, 8, 128, 16, sm_scale=SCALE, num_blocks=k.shape[0])
    out = w.run(q, (k, v))
    torch.cuda.synchronize()
    assert capi.status() == 0
    assert torch.equal(out, capi.auto(*case, SCALE))
    assert torch.all(out[3].float() == 0)
    sub = cases.subset(case, [0, 3, 17, 39])
    ref = oracle.attention_ref(*sub, SCALE)
    assert torch.allclose(out[[0, 3, 17, 39]].float().cpu(), ref, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("name", ["a_base", "e_partial_blocks", "g_hq64", "f_bs64"])
def test_wrapper_vs_reference(name):
    # the reference's FlashInfer-baseline cases (tests/test_flashinfer_baseline.py:34-52)
    case_cpu = cases.ref_case(name, seed=0)
    q, k, v, bt, sl = to_gpu(case_cpu)
    indptr, indices, last = binding.block_table_to_paged(bt, sl, k.shape[1])
    w = binding.BatchDecodeWithPagedKVCacheWrapper()
    w.plan(indptr, indices, last, q.shape[1], k.shape[2], 128, k.shape[1], sm_scale=SCALE,
           q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
    out = w.run(q, (k, v))
    torch.cuda.synchronize()
    ref = oracle.attention_ref(*case_cpu, SCALE)
    assert torch.allclose(out.float().cpu(), ref, atol=1e-2, rtol=1e-2)


def test_one_plan_many_runs_and_graph_replay():
    # one plan, several "layers" (fresh q / caches of the same shape and page
    # table), each run inside one captured CUDA graph
    base = to_gpu(cases.make_case([900, 33, 4100], 32, 8, 16, seed=60, poison=False))
    bt, sl = base[3], base[4]
    layers = [base]
    for i in range(1, 3):
        q, k, v, _, _ = to_gpu(cases.make_case([900, 33, 4100], 32, 8, 16, seed=60 + i,
                                               poison=False))
        assert k.shape == base[1].shape
        layers.append((q, k, v, bt, sl))  # same page table and lengths, new data
    indptr, indices, last = binding.block_table_to_paged(bt, sl, 16)
    w = binding.BatchDecodeWithPagedKVCacheWrapper()
    w.plan(indptr, indices, last, 32, 8, 128, 16, sm_scale=SCALE)
    outs = [torch.empty_like(lay[0]) for lay in layers]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for lay, o in zip(layers, outs):
            w.run(lay[0], (lay[1], lay[2]), out=o)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for lay, o in zip(layers, outs):
            w.run(lay[0], (lay[1], lay[2]), out=o)
    for o in outs:
        o.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    for lay, o in zip(layers, outs):
        assert torch.equal(o, capi.auto(*lay, SCALE))


def test_two_wrappers_keep_their_own_plans():
    # two batches planned up front, then run alternately: each wrapper's plan
    # and partial states live in its own workspace, so neither clobbers the other
    a = to_gpu(cases.make_case([700, 5000, 64], 32, 8, 16, seed=61))
    b = to_gpu(cases.make_case([3000] * 9, 32, 8, 16, seed=62))
    wa, wb = binding.BatchDecodeWithPagedKVCacheWrapper(), binding.BatchDecodeWithPagedKVCacheWrapper()
    wa.plan(*csr_of(a), 32, 8, 128, 16, sm_scale=SCALE, num_blocks=a[1].shape[0])
    wb.plan(*csr_of(b), 32, 8, 128, 16, sm_scale=SCALE, num_blocks=b[1].shape[0])
    for _ in range(2):
        out_a = wa.run(a[0], (a[1], a[2]))
        out_b = wb.run(b[0], (b[1], b[2]))
    torch.cuda.synchronize()
    assert capi.status() == 0
    assert torch.equal(out_a, capi.auto(*a, SCALE))
    assert torch.equal(out_b, capi.auto(*b, SCALE))


def test_wrapper_user_workspace_starts_dirty():
    # FlashInfer callers hand over an uninitialised byte buffer; the wrapper
    # zeroes it once before the first plan
    case = to_gpu(cases.make_case([2500, 17, 9000], 32, 8, 16, seed=63))
    buf = torch.full((64 << 20,), 0xA5, dtype=torch.uint8, device="cuda")
    w = binding.BatchDecodeWithPagedKVCacheWrapper(buf)
    w.plan(*csr_of(case), 32, 8, 128, 16, sm_scale=SCALE, num_blocks=case[1].shape[0])
    out = w.run(case[0], (case[1], case[2]))
    torch.cuda.synchronize()
    assert capi.status() == 0
    assert torch.equal(out, capi.auto(*case, SCALE))
