"""GPU, 2+ devices: the two multi-GPU partitionings on real NCCL ranks.

* KV-range sharding (config-5 recipe, shortened): every rank holds one
  contiguous page range of a single request; KVRangeDecoder (local state,
  NCCL all-gather, merge kernel) and P2PKVRangeDecoder (one kernel per rank,
  states exchanged with peer stores + flags over NVLink) must both match the
  single-GPU decode of the whole request on every rank.
* Batch sharding: every rank decodes its LPT share of a ragged batch with
  the unsplit scan (v1), whose arithmetic for a request does not depend on
  the other requests in the launch; each output must equal, bitwise, the
  same request decoded inside the whole batch.

Ranks run as spawned child processes with NVLS off (NCCL_NVLS_ENABLE=0).
"""

import math
import os
import socket
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
SCALE = 1.0 / math.sqrt(128)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, k_scale, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    sys.path[:0] = [os.path.join(REPO, "mla-decode-kernels_b200", "python"),
                    os.path.join(REPO, "oracle"), HERE]
    import torch.distributed as dist

    import binding
    import cases
    import sharding

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    sharding.init_process_group("nccl", timeout_s=60)
    if mode in ("kvrange", "kvrange_p2p"):
        S, bs = 40000, 64
        # same request on every rank (same seed), each keeps its own page range
        q, k, v, bt, sl = cases.make_case([S], 32, 8, bs, seed=50, pool_factor=1.0,
                                          k_scale=k_scale, device=dev)
        t0, t1 = sharding.kv_range(S, bs, rank, world)
        bt_r = bt[:, t0 // bs:(t1 + bs - 1) // bs].contiguous()
        sl_r = torch.tensor([t1 - t0], dtype=torch.int32, device=dev)
        if mode == "kvrange":
            out = sharding.KVRangeDecoder().decode(q, k, v, bt_r, sl_r, SCALE)
        else:
            dec = sharding.P2PKVRangeDecoder(1, 32, 8, dev)
            for _ in range(3):  # several epochs: both parities, reused buffers
                out = dec.decode(q, k, v, bt_r, sl_r, SCALE)
            torch.cuda.synchronize()
            dec.close()
        full = binding.gqa_decode(q, k, v, bt, sl, SCALE)
        torch.cuda.synchronize()
        np.save(os.path.join(result_dir, f"{mode}_{rank}.npy"),
                np.stack([out.float().cpu().numpy(), full.float().cpu().numpy()]))
    else:
        sl_all = cases.config4_seq_lens(seed=1, B=24)
        mine = sharding.lpt_shards(sl_all, world)[rank]
        # the whole batch is built identically on every rank; each decodes its share
        q, k, v, bt, sl = cases.make_case(sl_all, 32, 8, 16, seed=51, pool_factor=1.0 / 0.9,
                                          device=dev)
        idx = torch.tensor(mine, dtype=torch.long, device=dev)
        out = binding.gqa_decode_v1(q[idx].contiguous(), k, v, bt[idx].contiguous(),
                                    sl[idx].contiguous(), SCALE)
        ref = binding.gqa_decode_v1(q, k, v, bt, sl, SCALE)[idx]
        torch.cuda.synchronize()
        np.save(os.path.join(result_dir, f"batch_{rank}.npy"),
                np.stack([out.float().cpu().numpy(), ref.float().cpu().numpy()]))
    assert binding.get_status(True) == 0
    dist.barrier()
    dist.destroy_process_group()


def _spawn(world, mode, k_scale, tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(world, _free_port(), mode, k_scale, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")


def _world():
    return min(4, torch.cuda.device_count())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["kvrange", "kvrange_p2p"])
@pytest.mark.parametrize("k_scale", [1.0, 8.0])
def test_kv_range_sharding(tmp_path, mode, k_scale):
    world = _world()
    _spawn(world, mode, k_scale, tmp_path)
    for r in range(world):
        out, full = np.load(tmp_path / f"{mode}_{r}.npy")
        assert np.isfinite(out).all()
        np.testing.assert_allclose(out, full, atol=1e-2, rtol=1e-2)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_batch_sharding_bitwise(tmp_path):
    world = _world()
    _spawn(world, "batch", 1.0, tmp_path)
    for r in range(world):
        out, ref = np.load(tmp_path / f"batch_{r}.npy")
        assert np.array_equal(out, ref)
