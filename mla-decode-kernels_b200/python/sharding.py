"""Multi-GPU decode: one process per GPU, torch.distributed for the plumbing.

Two partitionings (the reference itself is single-GPU; its split-KV merge
identity, kernels/gqa_decode/v2_splitkv.cu:97-107, is what crosses GPUs):

* Batch sharding - independent requests are dealt to ranks (longest first,
  to the rank with the least total tokens), each rank decodes its own
  requests from its own KV pages.  No communication on the data path.

* KV-range sharding - one long request's pages are cut into contiguous
  ranges, one per rank.  Two exchanges of the per-rank softmax states:
  - P2PKVRangeDecoder (default): the decode's own merge kernel stores each
    rank's state straight into every rank's exchange buffer (CUDA IPC
    mappings of one cudaMalloc per rank, plain peer stores over NVLink, every
    64-bit word tagged with the decode's epoch) and merges all ranks' states
    once their words carry the epoch (bounded wait), so the all-gather and
    the merge happen inside the decode's kernels.
  - KVRangeDecoder: gqa_decode_partial, an NCCL all-gather of the packed
    states (Hq * 130 floats per request per rank: 16.6 KB at Hq = 32) and the
    merge kernel.  The collective-library baseline.
"""

import datetime
import heapq

import torch
import torch.distributed as dist


def lpt_shards(seq_lens, world):
    """Request indices per rank, balancing the sum of seq_lens (LPT greedy).

    Deterministic: ties are broken by request index and rank index.  Each
    rank's list is sorted ascending.
    """
    seq_lens = [int(s) for s in seq_lens]
    order = sorted(range(len(seq_lens)), key=lambda i: (-seq_lens[i], i))
    heap = [(0, r) for r in range(world)]
    shards = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + seq_lens[i], r))
    return [sorted(s) for s in shards]


def kv_range(seq_len, block_size, rank, world):
    """Token range [t0, t1) of `rank` when one request's pages are cut into
    `world` contiguous page ranges of near-equal size (page boundaries keep
    every rank's pages whole)."""
    n_pages = (seq_len + block_size - 1) // block_size
    p0 = n_pages * rank // world
    p1 = n_pages * (rank + 1) // world
    return min(seq_len, p0 * block_size), min(seq_len, p1 * block_size)


def pack_states(m, l, acc):
    """[m | l | acc] of one rank as a flat fp32 buffer of rows * 130 floats."""
    rows = m.numel()
    buf = torch.empty(rows * 130, dtype=torch.float32, device=m.device)
    buf[:rows].copy_(m.reshape(-1))
    buf[rows:2 * rows].copy_(l.reshape(-1))
    buf[2 * rows:].copy_(acc.reshape(-1))
    return buf


def unpack_states(gathered, rows):
    """Inverse of pack_states for gathered [world, rows * 130] buffers:
    m, l [world, rows] and acc [world, rows, 128], all contiguous."""
    world = gathered.shape[0]
    m = gathered[:, :rows].contiguous()
    l = gathered[:, rows:2 * rows].contiguous()
    acc = gathered[:, 2 * rows:].contiguous().view(world, rows, 128)
    return m, l, acc


def init_process_group(backend, timeout_s=60):
    """Process group from the torchrun environment with a short timeout, so a
    rank that never arrives ends the others' collectives with an error."""
    if not dist.is_initialized():
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
    return dist.group.WORLD


class KVRangeDecoder:
    """Decode requests whose KV range is split across the ranks of `group`.

    Each rank passes only its own pages (local k/v caches, block table and
    local token counts); decode() returns the full [B, Hq, 128] bf16 output
    on every rank.
    """

    def __init__(self, group=None):
        from binding import gqa_decode_partial, merge_states  # CUDA extension

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self._partial = gqa_decode_partial
        self._merge = merge_states
        self._gathered = None

    def decode(self, q, k_local, v_local, block_table_local, seq_lens_local, scale):
        m, l, acc = self._partial(q, k_local, v_local, block_table_local, seq_lens_local, scale)
        B, Hq = q.shape[0], q.shape[1]
        rows = B * Hq
        if self.world == 1:
            out = self._merge(m.view(1, rows), l.view(1, rows), acc.view(1, rows, 128))
            return out.view(B, Hq, 128)
        buf = pack_states(m, l, acc)
        n = buf.numel()
        if self._gathered is None or self._gathered.numel() != self.world * n:
            self._gathered = torch.empty(self.world * n, dtype=torch.float32, device=buf.device)
        dist.all_gather_into_tensor(self._gathered, buf, group=self.group)
        mm, ll, aa = unpack_states(self._gathered.view(self.world, n), rows)
        return self._merge(mm, ll, aa).view(B, Hq, 128)


def _cuda_check(err, what):
    from cuda.bindings import runtime as rt

    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"{what} failed: {err}")


class P2PKVRangeDecoder:
    """KV-range sharded decode with the cross-rank merge in the decode's
    merge kernel.

    Every rank allocates one exchange buffer (kvshard_buffer_bytes for the
    batch shape) with cudaMalloc, exports it with CUDA IPC and maps every
    peer's; the kernels then exchange states with plain peer stores.  Ranks
    must sit on distinct GPUs of one node (their kernels wait for each
    other).  decode() takes this rank's pages only and returns the full
    [B, Hq, 128] bf16 output on every rank.  Call close() (collectively)
    before the process group is destroyed.
    """

    def __init__(self, B, Hq, Hkv, device, group=None):
        from cuda.bindings import runtime as rt

        import binding

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("peer exchange supports up to 8 ranks")
        self.device = torch.device(device)
        self._binding = binding
        self.nbytes = binding.kvshard_buffer_bytes(B, Hq, Hkv, self.world)
        if self.nbytes <= 0:
            raise ValueError("invalid shape for the peer exchange")
        _cuda_check(rt.cudaSetDevice(self.device.index)[0], "cudaSetDevice")
        err, self._own = rt.cudaMalloc(self.nbytes)
        _cuda_check(err, "cudaMalloc")
        _cuda_check(rt.cudaMemset(self._own, 0, self.nbytes)[0], "cudaMemset")
        _cuda_check(rt.cudaDeviceSynchronize()[0], "cudaDeviceSynchronize")
        self._opened = []
        peers = [int(self._own)]
        if self.world > 1:
            err, handle = rt.cudaIpcGetMemHandle(self._own)
            _cuda_check(err, "cudaIpcGetMemHandle")
            uuid = str(torch.cuda.get_device_properties(self.device).uuid)
            info = [None] * self.world
            dist.all_gather_object(info, (bytes(handle.reserved), uuid), group=group)
            if len({u for _, u in info}) != self.world:
                raise RuntimeError("every rank of a peer exchange needs its own GPU")
            peers = []
            for r, (hb, _) in enumerate(info):
                if r == self.rank:
                    peers.append(int(self._own))
                    continue
                h = rt.cudaIpcMemHandle_t()
                h.reserved = hb
                err, ptr = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
                _cuda_check(err, "cudaIpcOpenMemHandle")
                self._opened.append(ptr)
                peers.append(int(ptr))
            dist.barrier(group=group)
        self.peers = peers
        self.epoch = 0

    def decode(self, q, k_local, v_local, block_table_local, seq_lens_local, scale, out=None):
        self.epoch = self.epoch + 1 if self.epoch < 0xFFFFFFFF else 1
        return self._binding.gqa_decode_kvshard(q, k_local, v_local, block_table_local,
                                                seq_lens_local, scale, self.rank, self.world,
                                                self.peers, self.epoch, out=out)

    def close(self):
        from cuda.bindings import runtime as rt

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for ptr in self._opened:
            rt.cudaIpcCloseMemHandle(ptr)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)
        rt.cudaFree(self._own)
        self._own = None
