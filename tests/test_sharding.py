"""CPU: multi-GPU host logic with world-size-2 gloo ranks.

* batch sharding (LPT) and KV-range cuts;
* the KV-range protocol end to end on CPU: each rank computes the softmax
  state of its page range (the oracle stands in for the GPU partial
  kernel), packs it, all-gathers, merges with the reference's identity
  (kernels/gqa_decode/v2_splitkv.cu:97-107) and must equal the unsharded
  oracle output;
* a rank that exits before the collective: the survivor's collective ends
  with an error within the process-group timeout instead of hanging.
"""

import math
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
import sharding

SCALE = 1.0 / math.sqrt(128)
LOG2E = math.log2(math.e)
HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_lpt_shards_balance_and_cover():
    sl = cases.config4_seq_lens(seed=1, B=256)
    for world in (1, 2, 4, 8):
        shards = sharding.lpt_shards(sl, world)
        assert sorted(i for s in shards for i in s) == list(range(256))
        loads = [sum(sl[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(sl)  # LPT bound
        assert max(loads) / (sum(sl) / world) < 1.02
        assert shards == sharding.lpt_shards(sl, world)  # deterministic


@pytest.mark.parametrize("S,bs", [(262144, 64), (1000, 16), (17, 16), (5, 64)])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_kv_range_cuts(S, bs, world):
    ranges = [sharding.kv_range(S, bs, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == S
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for t0, t1 in ranges:
        assert t0 % bs == 0 and t0 <= t1
    sizes = [t1 - t0 for t0, t1 in ranges]
    assert max(sizes) - min(sizes) <= bs + (S % bs)


def test_pack_unpack_roundtrip():
    g = torch.Generator().manual_seed(0)
    world, rows = 3, 10
    ms = [torch.randn(rows, generator=g) for _ in range(world)]
    ls = [torch.rand(rows, generator=g) for _ in range(world)]
    accs = [torch.randn(rows, 128, generator=g) for _ in range(world)]
    packed = torch.stack([sharding.pack_states(m, l, a) for m, l, a in zip(ms, ls, accs)])
    m, l, acc = sharding.unpack_states(packed, rows)
    assert torch.equal(m, torch.stack(ms)) and torch.equal(l, torch.stack(ls))
    assert torch.equal(acc, torch.stack(accs))


def _kv_worker(rank, world, port, S, bs, k_scale, result_path):
    sys.path[:0] = [os.path.join(os.path.dirname(HERE), "mla-decode-kernels_b200", "python"),
                    os.path.join(os.path.dirname(HERE), "oracle")]
    import cases as c
    import oracle
    import sharding as sh

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    sh.init_process_group("gloo", timeout_s=30)
    # every rank builds the same request, then keeps only its page range
    q, k, v, bt, sl = c.make_case([S], 32, 8, bs, seed=40, pool_factor=1.0, k_scale=k_scale)
    t0, t1 = sh.kv_range(S, bs, rank, world)
    bt_r = bt[:, t0 // bs:(t1 + bs - 1) // bs].contiguous()
    m, l, acc = oracle.attention_state(q, k, v, bt_r, torch.tensor([t1 - t0], dtype=torch.int32),
                                       SCALE, nthreads=2)
    buf = sh.pack_states(m * LOG2E, l, acc)  # the GPU kernel's log2-domain m
    gathered = torch.empty(world * buf.numel())
    dist.all_gather_into_tensor(gathered, buf)
    mm, ll, aa = sh.unpack_states(gathered.view(world, buf.numel()), 32)
    out = torch.empty(32, 128)
    for r in range(32):
        M, L, A = oracle.merge_states((mm[:, r] / LOG2E).numpy(), ll[:, r].numpy(),
                                      aa[:, r].numpy())
        out[r] = torch.from_numpy(A / L)
    if rank == 0:
        full = oracle.attention_ref(q, k, v, bt, sl, SCALE, nthreads=2)[0]
        np.save(result_path, np.stack([out.numpy(), full.numpy()]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("k_scale", [1.0, 8.0])
def test_kv_range_protocol_gloo(tmp_path, k_scale):
    path = str(tmp_path / "out.npy")
    mp.start_processes(_kv_worker, args=(2, free_port(), 4096 + 37, 64, k_scale, path), nprocs=2,
                       join=True, start_method="spawn")
    out, full = np.load(path)
    np.testing.assert_allclose(out, full, atol=1e-5, rtol=1e-4)


def _dying_worker(rank, world, port, result_path):
    sys.path[:0] = [os.path.join(os.path.dirname(HERE), "mla-decode-kernels_b200", "python")]
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, never reaches the collective
    buf = torch.ones(130)
    gathered = torch.empty(world * 130)
    try:
        dist.all_gather_into_tensor(gathered, buf)
        msg = "completed"
    except Exception as e:  # gloo reports the missing peer
        msg = "error: " + type(e).__name__
    with open(result_path, "w") as f:
        f.write(msg)
    os._exit(0)


def test_missing_rank_ends_collective_with_error(tmp_path):
    path = str(tmp_path / "msg.txt")
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, path)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung past the process-group timeout")
    with open(path) as f:
        assert f.read().startswith("error")
