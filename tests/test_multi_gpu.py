"""GPU, 2+ devices: the two multi-GPU partitionings on real NCCL ranks.

* KV-range sharding (config-5 recipe, shortened): every rank holds one
  contiguous page range of a single request; KVRangeDecoder (local state,
  NCCL all-gather, merge kernel) and P2PKVRangeDecoder (one kernel per rank,
  states exchanged with peer stores + flags over NVLink) must both match the
  single-GPU decode of the whole request on every rank, with K x 1 and with
  K x 8 (a peaked softmax, which stresses the merge).
* Batch sharding: every rank decodes its LPT share of a ragged batch with
  the unsplit scan (v1), whose arithmetic for a request does not depend on
  the other requests in the launch; each output must equal, bitwise, the
  same request decoded inside the whole batch.

Every world size in {2, 4, 8} that the machine has GPUs for runs once, as
spawned child processes (one per GPU) with NVLS off (NCCL_NVLS_ENABLE=0);
each spawn runs every mode and every test reads its results.
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
WORLDS = [2, 4, 8]
KV_MODES = [("kvrange", 1.0), ("kvrange", 8.0), ("kvrange_p2p", 1.0), ("kvrange_p2p", 8.0)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
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
    S, bs = 40000, 64
    for mode, k_scale in KV_MODES:
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
            out = torch.full_like(q, float("nan"))
            for _ in range(3):  # several epochs: both parities, reused buffers
                dec.decode(q, k, v, bt_r, sl_r, SCALE, out=out)
            torch.cuda.synchronize()
            dec.close()
        full = binding.gqa_decode(q, k, v, bt, sl, SCALE)
        torch.cuda.synchronize()
        np.save(os.path.join(result_dir, f"{mode}_k{k_scale:g}_{rank}.npy"),
                np.stack([out.float().cpu().numpy(), full.float().cpu().numpy()]))
        del q, k, v, bt, sl
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
    status = binding.get_status(True)
    np.save(os.path.join(result_dir, f"status_{rank}.npy"), np.array([status]))
    dist.barrier()
    dist.destroy_process_group()


_RUNS = {}


def _results(world, tmp_path_factory):
    """Spawn `world` ranks once and return the directory of their results."""
    if world not in _RUNS:
        import torch.multiprocessing as mp

        d = tmp_path_factory.mktemp(f"world{world}")
        for attempt in range(3):
            try:
                mp.start_processes(_worker, args=(world, _free_port(), str(d)), nprocs=world,
                                   join=True, start_method="spawn")
                _RUNS[world] = d
                break
            except Exception as e:
                # the rendezvous port chosen may be taken before rank 0 binds it: retry
                # with another; any other failure fails every test of this world once
                if "EADDRINUSE" in str(e) and attempt < 2:
                    continue
                _RUNS[world] = RuntimeError(f"world {world} ranks failed: {e}")
                break
    if isinstance(_RUNS[world], Exception):
        raise _RUNS[world]
    return _RUNS[world]


def _need(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("mode,k_scale", KV_MODES)
def test_kv_range_sharding(tmp_path_factory, world, mode, k_scale):
    _need(world)
    d = _results(world, tmp_path_factory)
    for r in range(world):
        out, full = np.load(d / f"{mode}_k{k_scale:g}_{r}.npy")
        assert np.isfinite(out).all()
        np.testing.assert_allclose(out, full, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("world", WORLDS)
def test_batch_sharding_bitwise(tmp_path_factory, world):
    _need(world)
    d = _results(world, tmp_path_factory)
    for r in range(world):
        out, ref = np.load(d / f"batch_{r}.npy")
        assert np.array_equal(out, ref)


@pytest.mark.parametrize("world", WORLDS)
def test_no_device_status_on_any_rank(tmp_path_factory, world):
    _need(world)
    d = _results(world, tmp_path_factory)
    for r in range(world):
        assert int(np.load(d / f"status_{r}.npy")[0]) == 0
