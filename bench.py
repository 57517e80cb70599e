#!/usr/bin/env python
"""Decode-step benchmark: KV-bytes HBM GB/s and µs per decode step on 1..8 B200.

One "step" is one paged GQA decode over one batch (all requests, all heads),
inputs resident in HBM.  KV bytes per step = sum_b S_b * Hkv * 128 * 2 * 2
(the reference's accounting, bench/common.py:67-68); q / out / block_table
traffic is excluded from the metric, as in the reference.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload rep|wide|ragged|long|long_peaked|mla|dsa] [--num-splits auto|N]
                  [--kernel auto|v0|v1|v2] [--api block_table|csr|csr_replan]

N > 1 runs under torchrun, one rank per GPU.  Workloads (BASELINE.json
configs; seeded synthetic data, cases.py):
  rep          config 2 per GPU: B=32, S=8192, Hq=32, Hkv=8, bs=16 (1 GiB KV
               per GPU).  Batch sharding: weak scaling, no communication.
  wide         config 3 per GPU: B=16, S=32768, Hq=64, Hkv=8, bs=64 (2 GiB/GPU).
  ragged       config 4: B=256 log-uniform S in [64, 32768], LPT-sharded over
               the ranks (strong scaling, no communication).
  long         config 5: B=1, S=262144, bs=64, KV range split over the ranks,
               states all-gathered (NCCL) and merged (strong scaling).
  long_peaked  config 5 with K x 8.
  mla          MLA latent-cache decode (K2), FlashMLA grid: b=128, h_q=128,
               mean S=8192 (--mla-sq / --mla-hq / --mla-sk / --mla-causal).
  dsa          sparse decode (K3): indexer + top-k 2048 + gather + MLA over
               the selected tokens, same grid (--dsa-topk).
Every input set is larger than the 126 MB L2, so no flush is needed between
steps.  --impl reference times the CPU restatement of the reference's oracle
(oracle/, python/reference.py semantics) on the host cores instead.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_PY = os.path.join(REPO, "mla-decode-kernels_b200", "python")
ORACLE_DIR = os.path.join(REPO, "oracle")
for _p in (PKG_PY, ORACLE_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "KV-bytes HBM GB/s (% of SoL) and median us/decode step"
SCALE = 1.0 / math.sqrt(128)
# Reference's best published kernel at the rep shape: v2 splits=32,
# 1.1426 ms for 1 GiB on one H100 (bench/results/matrix_20260824_213534/
# cell_32x8_S8192_B32_bs16.json) = 939.7 GB/s.
BASELINE_GBS = (1 << 30) / 1.1426e-3 / 1e9
FALLBACK_HBM_GBS = 6650.0
E2E_PATHS = {
    "block_table": "binding.gqa_decode -> C ABI gqa_decode_launch; every step q, block_table "
                   "and seq_lens H2D from pinned host memory and out D2H",
    "csr": "BatchDecodeWithPagedKVCacheWrapper plan + run -> C ABI gqa_decode_plan / "
           "gqa_decode_run; every step q, indptr, indices and last_page_len H2D from pinned "
           "host memory, a fresh plan, and out D2H",
}
E2E_PATHS["csr_replan"] = E2E_PATHS["csr"]


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="rep",
                    choices=["rep", "wide", "ragged", "long", "long_peaked", "mla", "dsa"])
    ap.add_argument("--mla-sq", type=int, default=1, help="mla: query tokens per request")
    ap.add_argument("--mla-hq", type=int, default=128, help="mla: query heads")
    ap.add_argument("--mla-sk", type=int, default=8192, help="mla: mean cached tokens")
    ap.add_argument("--mla-causal", action="store_true")
    ap.add_argument("--dsa-topk", type=int, default=2048, help="dsa: tokens selected per query")
    ap.add_argument("--num-splits", default="auto",
                    help="auto = balanced schedule; an integer = fixed splits (v2)")
    ap.add_argument("--kernel", default="auto", choices=["auto", "v0", "v1", "v2"],
                    help="entry point timed: auto = gqa_decode (C ABI gqa_decode_launch); "
                         "v0/v1/v2 = the reference-compatible binding functions")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline budget (our arm, rank 0, N=1)")
    ap.add_argument("--ref-seconds", type=float, default=90.0,
                    help="total budget of the --impl reference arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="long workloads at N > 1: fused peer-memory merge or NCCL all-gather")
    ap.add_argument("--api", default="block_table", choices=["block_table", "csr", "csr_replan"],
                    help="batch workloads, --kernel auto: block_table = gqa_decode (one call); "
                         "csr = BatchDecodeWithPagedKVCacheWrapper.run on a CSR page table "
                         "planned once (plan amortised over layers); csr_replan = plan + run "
                         "every step")
    ap.add_argument("--batch", type=int, default=None,
                    help="requests per GPU for rep / wide (smaller cases for profiling)")
    return ap.parse_args()


# ---------------------------------------------------------------- environment

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_hbm_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "MEASURED_PEAKS.json hbm_gbs (copy, burst)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


# Archived ncu captures (profiles/<stem>.ncu.txt, written by ncu_report.py)
# of the dominant kernel of each timed configuration, on a smaller case of
# the same kernel; DRAM traffic scales with the KV bytes a launch processes.
CAPTURES = {
    ("rep", "auto"): ("gqa_decode_scan_kernel", "gqa_decode_scan_kernel_rep_b16"),
    ("wide", "auto"): ("gqa_decode_scan_kernel", "gqa_decode_scan_kernel_wide_b4"),
    ("rep", "v0"): ("gqa_decode_simt_kernel", "gqa_decode_simt_kernel_v0_b16"),
    ("rep", "v1"): ("gqa_decode_scan_kernel", "gqa_decode_scan_kernel_v1_b16"),
    ("rep", "v2"): ("gqa_decode_scan_kernel", "gqa_decode_scan_kernel_v2_ns8_b16"),
}


def dominant_kernel(args):
    kernel = "auto" if args.kernel == "auto" else args.kernel
    name, stem = CAPTURES.get((args.workload, kernel), ("gqa_decode_scan_kernel", None))
    if kernel == "v2" and args.num_splits not in ("8", "auto"):
        stem = None  # captured at num_splits=8 only
    return name, stem


def profiled_traffic(stem, kv_bytes_per_launch):
    """DRAM bytes per launch: the capture's DRAM bytes / algorithmic bytes
    ratio times this launch's KV bytes, or None without a capture."""
    if stem is None:
        return None
    import ncu_report

    r = ncu_report.traffic_ratio(stem)
    return None if r is None else int(r * kv_bytes_per_launch)


class ClockSampler:
    """nvidia-smi sampling during the timed region (the profiling recipe's
    clocks line), filtered to the given GPU UUIDs."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids):
        self.uuids = [u.lower().replace("gpu-", "") for u in uuids]
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            uuid = parts[1].lower().replace("gpu-", "")
            if self.uuids and uuid not in self.uuids:
                continue
            try:
                sm.append(float(parts[2]))
                smax.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[6:10]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- workloads

def build_workload(name, rank, world, device, batch=None):
    """Returns (case on device, description dict, kv bytes of this rank,
    decode function factory kind)."""
    import cases

    if name == "rep":
        B = batch or 32
        case = cases.config2(device=device, seed=2 + rank, B=B)
        cfg = {"workload": "config2_rep" if B == 32 else f"config2_rep_B{B}", "B_per_gpu": B,
               "seq_len": 8192, "Hq": 32, "Hkv": 8, "block_size": 16,
               "num_blocks_per_gpu": B * 512, "global_batch": B * world}
        kind = "batch"
    elif name == "wide":
        B = batch or 16
        case = cases.config3(device=device, seed=3 + rank, B=B)
        cfg = {"workload": "config3_wide", "B_per_gpu": B, "seq_len": 32768, "Hq": 64,
               "Hkv": 8, "block_size": 64, "global_batch": B * world}
        kind = "batch"
    elif name == "ragged":
        import sharding

        sl_all = cases.config4_seq_lens(seed=1, B=256)
        mine = sharding.lpt_shards(sl_all, world)[rank]
        sl = [sl_all[i] for i in mine]
        need = sum((s + 15) // 16 for s in sl)
        case = cases.make_case(sl, 32, 8, 16, seed=100 + rank,
                               pool_blocks=int(math.ceil(need / 0.9)), device=device)
        cfg = {"workload": "config4_ragged", "global_batch": 256, "Hq": 32, "Hkv": 8,
               "block_size": 16, "seq_lens": "log-uniform [64, 32768] seed 1",
               "sharding": "LPT by tokens", "requests_this_rank": len(sl)}
        kind = "batch"
    else:
        import sharding

        S, bs = 262144, 64
        t0, t1 = sharding.kv_range(S, bs, rank, world)
        case = cases.make_case([t1 - t0], 32, 8, bs, seed=5 + rank, pool_factor=1.0,
                               k_scale=8.0 if name == "long_peaked" else 1.0, device=device)
        cfg = {"workload": "config5_" + name, "global_batch": 1, "seq_len": S, "Hq": 32,
               "Hkv": 8, "block_size": bs, "sharding": f"KV range / {world}"}
        kind = "kvrange"
    return case, cfg, cases.kv_bytes(case[4].tolist(), case[1].shape[2]), kind


# ---------------------------------------------------------------- helpers

def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world, device):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# GPU cycles (~0.1 ms) of a spin kernel queued ahead of the start event, so
# the host has queued the start event and the first steps before the GPU
# reaches them: the timed region then holds the K steps back to back, not
# the host's latency to issue the first launch after the synchronize.
LEAD_CYCLES = 200_000


def time_loop(step, K, world, stream, finish=None):
    """Mean ms per step over exactly K steps, CUDA events on `stream`,
    barrier + synchronize on both sides.  `finish` joins any side streams
    into `stream` before the end event."""
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(LEAD_CYCLES)
    start.record(stream)
    for _ in range(K):
        step()
    if finish is not None:
        finish()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end) / K


class E2ELoop:
    """Double-buffered host<->device traffic around the decode: H2D of the
    next step's inputs on one copy stream, D2H of each output on another, the
    decode on the compute stream, ordered by events."""

    def __init__(self, inputs, out, stream):
        self.compute = stream
        self.h2d_stream = torch.cuda.Stream(device=out.device)
        self.d2h_stream = torch.cuda.Stream(device=out.device)
        self.host_in = [tuple(t.cpu().pin_memory() for t in inputs) for _ in range(2)]
        self.dev_in = [tuple(torch.empty_like(t) for t in inputs) for _ in range(2)]
        self.dev_out = [torch.empty_like(out) for _ in range(2)]
        self.host_out = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
                         for _ in range(2)]
        self.uploaded = [torch.cuda.Event() for _ in range(2)]
        self.decoded = [torch.cuda.Event() for _ in range(2)]
        self.downloaded = [torch.cuda.Event() for _ in range(2)]
        self.i = 0
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.host_in[0])
        self.d2h_bytes = out.numel() * out.element_size()
        self._upload(0)

    def _upload(self, j):
        with torch.cuda.stream(self.h2d_stream):
            # buffer j was last read by the decode two steps ago
            self.h2d_stream.wait_event(self.decoded[j])
            for d, h in zip(self.dev_in[j], self.host_in[j]):
                d.copy_(h, non_blocking=True)
            self.uploaded[j].record(self.h2d_stream)

    def step(self, decode):
        j = self.i % 2
        self._upload(1 - j)  # next step's inputs, overlapping this decode
        self.compute.wait_event(self.uploaded[j])
        self.compute.wait_event(self.downloaded[j])  # out buffer j is free again
        decode(*self.dev_in[j], self.dev_out[j])
        self.decoded[j].record(self.compute)
        with torch.cuda.stream(self.d2h_stream):
            self.d2h_stream.wait_event(self.decoded[j])
            self.host_out[j].copy_(self.dev_out[j], non_blocking=True)
            self.downloaded[j].record(self.d2h_stream)
        self.i += 1

    def drain(self):
        self.compute.wait_stream(self.d2h_stream)
        self.compute.wait_stream(self.h2d_stream)

    def serial_step(self, decode):
        """One step with nothing overlapped: this step's H2D copies, the
        decode and the D2H copy of its output, in that order on the compute
        stream, so the time per step is the host-to-host latency of a step."""
        with torch.cuda.stream(self.compute):
            for d, h in zip(self.dev_in[0], self.host_in[0]):
                d.copy_(h, non_blocking=True)
            decode(*self.dev_in[0], self.dev_out[0])
            self.host_out[0].copy_(self.dev_out[0], non_blocking=True)

    def last_output(self):
        torch.cuda.synchronize()
        return self.host_out[(self.i - 1) % 2].to(self.dev_out[0].device)


def serial_e2e(e2e, decode, steps, world, stream, device):
    """Mean ms per step of E2ELoop.serial_step over min(steps, 200) steps,
    max over ranks (after the pipelined loop has drained)."""
    torch.cuda.synchronize()
    for _ in range(3):
        e2e.serial_step(decode)
    n = max(1, min(steps, 200))
    return max_over_ranks(time_loop(lambda: e2e.serial_step(decode), n, world, stream), world,
                          device)


SERIAL_NOTE = ("serial_*: the same step with nothing overlapped (H2D of the step's inputs, the "
               "decode, D2H of its output, in order on one stream): the per-step host-to-host "
               "latency; value/ms_per_step above are the pipelined serving loop")


def per_step_median_us(step, n, stream):
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
    torch.cuda.synchronize()
    evs[0].record(stream)
    for i in range(n):
        step()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    return statistics.median(evs[i].elapsed_time(evs[i + 1]) * 1e3 for i in range(n))


def cpu_sample_case(n_requests):
    """Requests with the rep shape (S=8192, Hq=32, Hkv=8, bs=16) on CPU."""
    import cases

    return cases.make_case([8192] * n_requests, 32, 8, 16, seed=2, pool_factor=1.0,
                           device="cpu")


def time_oracle(case, reps, nthreads):
    import oracle

    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.attention_ref(*case, SCALE, nthreads=nthreads)
        ts.append(time.perf_counter() - t0)
    return ts


def cpu_baseline(budget_s):
    """The oracle port on the host cores, on a bounded sample of the rep
    workload; returns the cpu_baseline object."""
    import cases
    import oracle

    threads = oracle.default_threads()
    n_req = 4
    case = cpu_sample_case(n_req)
    time_oracle(case, 1, threads)  # warm (page-in, thread start)
    one = time_oracle(case, 1, threads)[0]
    reps = max(2, min(200, int(budget_s / max(one, 1e-6))))
    ts = time_oracle(case, reps, threads)
    mean = statistics.mean(ts)
    kv = cases.kv_bytes([8192] * n_req, 8)
    return {"value": round(kv / mean / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{n_req} of the 32 requests of config 2 (S=8192, Hq=32, Hkv=8, bs=16), "
                      f"{reps} runs, mean {mean * 1e3:.2f} ms; oracle/gqa_oracle.c "
                      f"(python/reference.py:attention_ref restated in C), {threads} threads",
            "ms_per_full_step_extrapolated": round(mean * 1e3 * 32 / n_req, 3)}


REF_PY = os.path.join(REPO, "baseline", "_ref", "reference.py")


def reference_py_baseline(budget_s):
    """The reference's own CPU oracle, python/reference.py:attention_ref, on a
    bounded sample of rep requests on all host cores (torch CPU threads).

    The reference has no installable package, so __graft_entry__.build()
    stages an unmodified copy of that file in the git-ignored baseline/_ref/
    when a reference checkout is present; None when the copy is absent.
    """
    if not os.path.exists(REF_PY):
        return None
    import importlib.util

    import cases
    import oracle

    spec = importlib.util.spec_from_file_location("reference_py", REF_PY)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    threads = oracle.default_threads()
    saved = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        n_req = 1
        case = cpu_sample_case(n_req)
        mod.attention_ref(*case, SCALE)  # warm (page-in, thread pool)
        t0 = time.perf_counter()
        mod.attention_ref(*case, SCALE)
        one = time.perf_counter() - t0
        reps = max(2, min(50, int(budget_s / max(one, 1e-6))))
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            mod.attention_ref(*case, SCALE)
            ts.append(time.perf_counter() - t0)
    finally:
        torch.set_num_threads(saved)
    mean = statistics.mean(ts)
    kv = cases.kv_bytes([8192] * n_req, 8)
    return {"value": round(kv / mean / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": "reference",
            "sample": f"{n_req} of the 32 requests of config 2 (S=8192, Hq=32, Hkv=8, bs=16), "
                      f"{reps} runs, mean {mean * 1e3:.1f} ms; python/reference.py:attention_ref "
                      f"(the reference's own code, unmodified), torch CPU with {threads} threads",
            "ms_per_full_step_extrapolated": round(mean * 1e3 * 32 / n_req, 1)}


# ---------------------------------------------------------------- arms

def run_reference(args, world, rank):
    """CPU restatement of the reference's oracle (the reference's only CPU
    implementation of the path, python/reference.py) on the host cores."""
    if rank != 0:
        return
    import cases
    import oracle

    threads = oracle.default_threads()
    probe = cpu_sample_case(1)
    time_oracle(probe, 1, threads)
    t_req = statistics.mean(time_oracle(probe, 2, threads))
    per_step_budget = args.ref_seconds / max(1, args.steps + args.warmup)
    n_req = int(max(1, min(32, per_step_budget // max(t_req, 1e-9))))
    case = cpu_sample_case(n_req)
    time_oracle(case, args.warmup, threads)
    ts = time_oracle(case, args.steps, threads)
    mean = statistics.mean(ts)
    kv = cases.kv_bytes([8192] * n_req, 8)
    gbs = kv / mean / 1e9
    full_ms = mean * 1e3 * 32 / n_req
    line = {
        "impl": "reference",
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(full_ms, 4),
        "median_us_per_step": round(statistics.median(ts) * 1e6 * 32 / n_req, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) bf16, cases.py recipe)",
        "config": {"workload": "config2_rep", "B": 32, "seq_len": 8192, "Hq": 32, "Hkv": 8,
                   "block_size": 16, "per_step_sample_requests": n_req,
                   "ms_per_step_basis": "sample time x 32 / sample requests"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{n_req} of 32 requests of config 2 per step; "
                                   "oracle/gqa_oracle.c restating python/reference.py"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        # the reference's own python/reference.py on the same cores, beside the port
        "reference_py": reference_py_baseline(10.0),
    }
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    import binding
    import cases

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import sharding

        sharding.init_process_group("nccl", timeout_s=120)
    case, cfg, kv_local, kind = build_workload(args.workload, rank, world, device, args.batch)
    q, k, v, bt, sl = case
    ns = 0 if args.num_splits == "auto" else int(args.num_splits)

    out = torch.empty_like(q)
    if args.api != "block_table" and (kind != "batch" or args.kernel != "auto"):
        raise SystemExit("--api csr / csr_replan needs a batch workload and --kernel auto")
    if args.api != "block_table":
        page = k.shape[1]
        csr = binding.block_table_to_paged(bt, sl, page)
        wrapper = binding.BatchDecodeWithPagedKVCacheWrapper()

        def plan(indptr, indices, last):
            wrapper.plan(indptr, indices, last, q.shape[1], k.shape[2], 128, page,
                         sm_scale=SCALE, num_blocks=k.shape[0])
        plan(*csr)
        if args.api == "csr":
            def step():
                wrapper.run(q, (k, v), out=out)
            launches_per_step = 2  # scan + cut-row merge
        else:
            def step():
                plan(*csr)
                wrapper.run(q, (k, v), out=out)
            launches_per_step = 3  # plan, scan, cut-row merge
    elif kind == "batch" and args.kernel != "auto":
        if args.kernel == "v2":
            ns2 = 8 if ns == 0 else ns
            fn = lambda *a: binding.gqa_decode_v2(*a, num_splits=ns2)  # noqa: E731
            launches_per_step = 1 if ns2 == 1 else 2
        else:
            fn = binding.KERNELS[args.kernel]
            launches_per_step = 1

        def step():
            out.copy_(fn(q, k, v, bt, sl, SCALE))
        launches_per_step += 1  # the copy into the step's output buffer
    elif kind == "batch":
        def step():
            binding.gqa_decode(q, k, v, bt, sl, SCALE, num_splits=ns, out=out)
        # balanced: scan + cut-row merge; one split: scan; fixed splits: scan + merge
        launches_per_step = 1 if ns == 1 else 2
    else:
        import sharding

        if args.exchange == "p2p":
            dec = sharding.P2PKVRangeDecoder(q.shape[0], q.shape[1], k.shape[2], device)
            launches_per_step = 2  # scan + merge/exchange kernel

            def step():
                dec.decode(q, k, v, bt, sl, SCALE, out=out)
        else:
            dec = sharding.KVRangeDecoder()
            launches_per_step = 4  # scan + cut-row merge (states), state merge after NCCL, copy

            def step():
                out.copy_(dec.decode(q, k, v, bt, sl, SCALE))

    # correctness spot check before timing (bench/common.py:75-89): the first
    # two requests (or the whole shard) against the CPU oracle.
    step()
    torch.cuda.synchronize()
    import oracle

    if kind == "batch":
        reqs = list(range(min(2, q.shape[0])))
        ref = oracle.attention_ref(*cases.subset(case, reqs), SCALE)
        spot_out = out[reqs].float().cpu()
    else:
        spot_out = None
        ref = None
        if world == 1:
            ref = oracle.attention_ref(*cases.subset(case, [0]), SCALE)
            spot_out = out.float().cpu()
    if ref is not None:
        err = (spot_out - ref).abs().max().item()
        if not torch.allclose(spot_out, ref, atol=1e-2, rtol=1e-2):
            raise SystemExit(f"spot check failed: max-abs {err:.3e}")
    status = binding.get_status(True)
    if status:
        raise SystemExit(f"device status {status} after spot check")

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    uuids = [str(torch.cuda.get_device_properties(device).uuid)]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, uuids[0])
        uuids = gathered
    sampler = ClockSampler(uuids) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ms = time_loop(step, args.steps, world, stream)
    clocks = sampler.stop() if sampler else None
    ms_max = max_over_ranks(ms, world, device)
    kv_total = sum_over_ranks(kv_local, world, device)
    median_us = per_step_median_us(step, min(args.steps, 200), stream)
    median_us = max_over_ranks(median_us, world, device)

    # e2e through the public API with host buffers: every step copies its q,
    # block_table and seq_lens H2D from pinned memory and its out back D2H.
    # As in a serving loop, step i+1's inputs are uploaded (copy stream) while
    # step i decodes, and step i's output is downloaded (second copy stream)
    # while step i+1 decodes; buffers are double-buffered.
    e2e = E2ELoop((q, *csr) if args.api != "block_table" else (q, bt, sl), out, stream)
    if args.api != "block_table":
        def decode(q_d, indptr_d, indices_d, last_d, out_d):
            plan(indptr_d, indices_d, last_d)
            wrapper.run(q_d, (k, v), out=out_d)
    elif kind == "batch" and args.kernel != "auto":
        def decode(q_d, bt_d, sl_d, out_d):
            out_d.copy_(fn(q_d, k, v, bt_d, sl_d, SCALE))
    elif kind == "batch":
        def decode(q_d, bt_d, sl_d, out_d):
            binding.gqa_decode(q_d, k, v, bt_d, sl_d, SCALE, num_splits=ns, out=out_d)
    elif args.exchange == "p2p":
        def decode(q_d, bt_d, sl_d, out_d):
            dec.decode(q_d, k, v, bt_d, sl_d, SCALE, out=out_d)
    else:
        def decode(q_d, bt_d, sl_d, out_d):
            out_d.copy_(dec.decode(q_d, k, v, bt_d, sl_d, SCALE))
    for _ in range(max(3, args.warmup // 4)):
        e2e.step(decode)
    e2e.drain()
    h2d, d2h = e2e.h2d_bytes, e2e.d2h_bytes
    ms_e2e = max_over_ranks(time_loop(lambda: e2e.step(decode), args.steps, world, stream,
                                      finish=e2e.drain), world, device)
    if not torch.equal(e2e.last_output(), out):
        raise SystemExit("e2e output differs from the device-resident output")
    ms_serial = serial_e2e(e2e, decode, args.steps, world, stream, device)
    status = binding.get_status(True)
    if status:
        raise SystemExit(f"device status {status} after timing")

    if kind == "kvrange" and hasattr(dec, "close"):
        dec.close()
    if rank != 0:
        return
    peak, peak_src = measured_hbm_peak()
    kernel_name, capture = dominant_kernel(args)
    achieved = kv_local / (ms * 1e-3) / 1e9  # rank 0's kernel, per launch
    value = kv_total / (ms_max * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 5),
        "median_us_per_step": round(median_us, 2),
        "pct_of_sol": round(100.0 * value / (peak * world), 2),
        "higher_is_better": True,
        "scaling": "weak" if args.workload in ("rep", "wide") else "strong",
        "vs_baseline": round(value / BASELINE_GBS, 3),
        "vs_baseline_basis": "reference v2 best (splits=32) at the rep shape on 1 H100: "
                             "1.1426 ms per GiB = 939.7 GB/s",
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 q/K/V, cases.py recipe)",
        "config": dict(cfg, parallelism=f"dp{world}" if kind == "batch" else f"kv{world}",
                       num_splits=args.num_splits, kernel=args.kernel, api=args.api,
                       exchange=args.exchange if kind == "kvrange" else None,
                       l2="inputs > 126 MB L2 (1+ GiB KV per GPU); no flush needed",
                       kv_bytes_per_step=int(kv_total)),
        "e2e": {"value": round(kv_total / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(ms_e2e, 5), "h2d_bytes_per_step": int(h2d * world),
                "d2h_bytes_per_step": int(d2h * world),
                "path": E2E_PATHS[args.api] + "; double-buffered on two copy streams "
                        "overlapping the previous / next decode",
                "serial_ms_per_step": round(ms_serial, 5),
                "serial_value": round(kv_total / (ms_serial * 1e-3) / 1e9, 2),
                "serial_note": SERIAL_NOTE},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": profiled_traffic(capture, kv_local), "peak_source": peak_src,
                     "traffic_source": f"profiles/{capture}.ncu.txt" if capture else None,
                     "kernel": kernel_name,
                     "algorithmic_bytes_per_launch": int(kv_local)},
        "gpu_launches": int(args.steps * launches_per_step),
        "gpu_launches_note": f"{launches_per_step} per step in the timed device-resident loop "
                             "(the e2e loop launches the same per step)",
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
        line["cpu_baseline"]["reference_py"] = reference_py_baseline(min(10.0, args.cpu_seconds))
    else:
        line["cpu_baseline"] = None
    print(json.dumps(line), flush=True)


def mla_seq_lens(B, mean, s_q, seed=0):
    """Ragged cache lengths ~ Normal(mean, mean / 2), at least s_q (the
    distribution of FlashMLA's varlen performance grid, which the reference's
    docs/g0/flashmla_bench_raw.txt logs at b = 128)."""
    g = torch.Generator().manual_seed(seed)
    s = torch.normal(float(mean), float(mean) / 2, (B,), generator=g)
    return s.round().clamp(min=s_q).to(torch.int64).tolist()


def run_mla(args, world, rank, local):
    """MLA latent-cache decode (K2) on the FlashMLA performance grid shape:
    b = 128 requests per GPU, h_q heads, s_q query tokens, 64-token pages."""
    import cases
    import mla_decode

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import sharding

        sharding.init_process_group("nccl", timeout_s=120)
    B = args.batch or 128
    s_q, h_q = args.mla_sq, args.mla_hq
    sl = mla_seq_lens(B, args.mla_sk, s_q, seed=rank)
    case = cases.make_mla_case(sl, s_q, h_q, seed=10 + rank, pool_factor=1.0, poison=False,
                               device=device)
    q, kv, bt, sl_t = case
    scale = 1.0 / math.sqrt(192)
    ns = int(mla_decode._ext.mla_pick_splits(B, s_q, h_q, bt.shape[1],
                                            torch.cuda.get_device_properties(device)
                                            .multi_processor_count))
    holder = {}

    def step():
        holder["o"] = mla_decode.mla_decode(q, kv, bt, sl_t, scale, causal=args.mla_causal,
                                            num_splits=ns)

    step()
    torch.cuda.synchronize()
    import oracle

    reqs = [0, 1]
    ro, rl = oracle.mla_ref(*cases.mla_subset(case, reqs), scale, causal=args.mla_causal)
    out = holder["o"][0][reqs].float().cpu()
    if not torch.allclose(out, ro, atol=1e-2, rtol=1e-2):
        raise SystemExit(f"mla spot check failed: {(out - ro).abs().max().item():.3e}")
    if mla_decode.get_status(True):
        raise SystemExit("mla device status set")
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    uuids = [str(torch.cuda.get_device_properties(device).uuid)]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, uuids[0])
        uuids = gathered
    sampler = ClockSampler(uuids) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ms = time_loop(step, args.steps, world, stream)
    clocks = sampler.stop() if sampler else None
    ms_max = max_over_ranks(ms, world, device)
    median_us = max_over_ranks(per_step_median_us(step, min(args.steps, 200), stream), world,
                               device)
    kv_local = cases.mla_kv_bytes(sl)
    fl_local = cases.mla_flops(sl, s_q, h_q)
    kv_total = sum_over_ranks(kv_local, world, device)
    fl_total = sum_over_ranks(fl_local, world, device)

    # e2e: q and the page table up, out and lse back, every step
    out_buf = torch.empty((B, s_q, h_q, 512), dtype=torch.bfloat16, device=device)
    e2e = E2ELoop((q, bt, sl_t), out_buf, stream)

    def decode(q_d, bt_d, sl_d, out_d):
        o, _ = mla_decode.mla_decode(q_d, kv, bt_d, sl_d, scale, causal=args.mla_causal,
                                     num_splits=ns)
        out_d.copy_(o)
    for _ in range(3):
        e2e.step(decode)
    e2e.drain()
    ms_e2e = max_over_ranks(time_loop(lambda: e2e.step(decode), args.steps, world, stream,
                                      finish=e2e.drain), world, device)
    ms_serial = serial_e2e(e2e, decode, args.steps, world, stream, device)
    if mla_decode.get_status(True):
        raise SystemExit("mla device status set after timing")
    if rank != 0:
        return
    peak, peak_src = measured_hbm_peak()
    tc_peak = 1694.0
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            tc_peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    achieved = kv_local / (ms * 1e-3) / 1e9
    tflops = fl_local / (ms * 1e-3) / 1e12
    value = kv_total / (ms_max * 1e-3) / 1e9
    line = {
        "metric": "MLA decode: latent-cache GB/s and TFLOP/s (FlashMLA accounting)",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max, 5),
        "median_us_per_step": round(median_us, 2),
        "pct_of_sol": round(100.0 * value / (peak * world), 2),
        "tflops": round(fl_total / (ms_max * 1e-3) / 1e12, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "vs_baseline_basis": "FlashMLA on H100 at this grid point: docs/g0/flashmla_bench_raw.txt",
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16, cases.make_mla_case)",
        "config": {"workload": f"mla_b{B}_sq{s_q}_hq{h_q}_sk{args.mla_sk}", "B": B,
                   "s_q": s_q, "h_q": h_q, "mean_seq_len": args.mla_sk,
                   "seq_lens": "Normal(mean, mean/2) >= s_q, seeded", "page": 64,
                   "causal": args.mla_causal, "num_splits": ns, "kernel": "mla",
                   "parallelism": f"dp{world}", "kv_bytes_per_step": int(kv_total),
                   "flops_per_step": int(fl_total),
                   "l2": "inputs > 126 MB L2; no flush needed"},
        "e2e": {"value": round(kv_total / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(ms_e2e, 5),
                "h2d_bytes_per_step": int(e2e.h2d_bytes * world),
                "d2h_bytes_per_step": int(e2e.d2h_bytes * world),
                "path": "mla_decode.mla_decode -> C ABI mla_decode_launch; q, block_table and "
                        "seq_lens H2D, out D2H every step, double-buffered",
                "serial_ms_per_step": round(ms_serial, 5),
                "serial_value": round(kv_total / (ms_serial * 1e-3) / 1e9, 2),
                "serial_note": SERIAL_NOTE,
                "copy_note": "q [B, s_q, h_q, 576] and out [B, s_q, h_q, 512] bf16 cross PCIe "
                             "every step (18.9 + 16.8 MB at b=128, h_q=128): at ~50 GB/s that "
                             "is ~0.7 ms of copies against a ~0.5 ms decode, so the pipelined "
                             "loop is bound by the copies, not the kernel"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": peak_src, "kernel": "mla_decode_kernel",
                     "algorithmic_bytes_per_launch": int(kv_local),
                     "tensor_achieved_tflops": round(tflops, 1), "tensor_peak_tflops": tc_peak,
                     "tensor_frac": round(tflops / tc_peak, 4)},
        # 128-row query groups: the persistent kernel and its combine pass
        "gpu_launches": int(args.steps * (2 if (s_q * h_q) % 128 == 0 or ns > 1 else 1)),
        "clocks": clocks, "cpu_baseline": None,
    }
    print(json.dumps(line), flush=True)


def dsa_launches_per_step(B, s_q, h_q, topk, ns, sms):
    """Kernels one sparse decode step launches: indexer, top-k, then for h_q
    a multiple of 128 the MLA rows kernel over the selection, plus its
    combine pass when it takes the balanced split (the choice
    mla_launch_impl makes in mla_decode.cu: whole units per CTA pair in
    waves, 3.3 us per 64-token tile + 6 us per wave, against 30 us + 3.7 us
    per tile per pair); otherwise the gather and the MLA decode (+ its merge
    for splits)."""
    if h_q % 128 != 0:
        return 4 + (1 if ns > 1 else 0)
    units = B * s_q * h_q // 128
    pairs = max(1, sms // 2)
    nt = (topk + 63) // 64
    waves = (units + pairs - 1) // pairs
    whole = waves * (3.3 * nt + 6.0)
    balanced = 30.0 + 3.7 * units * nt / pairs
    return 3 if whole <= balanced else 4


def run_dsa(args, world, rank, local):
    """DSA-style sparse decode (K3): indexer -> top-k -> gather -> MLA decode
    over the selected tokens, b = 128 requests per GPU at the MLA grid's cache
    lengths, DeepSeek-V3.2's indexer shape (64 index heads of 128 dims) and
    top-k 2048."""
    import numpy as np

    import cases
    import dsa_decode
    import mla_decode
    import oracle

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import sharding

        sharding.init_process_group("nccl", timeout_s=120)
    B = args.batch or 128
    s_q, h_q, topk = args.mla_sq, args.mla_hq, args.dsa_topk
    n_idx = 64 // s_q
    causal = args.mla_causal
    sl = mla_seq_lens(B, args.mla_sk, s_q, seed=rank)
    case = cases.make_dsa_case(sl, s_q, h_q, n_idx_heads=n_idx, seed=20 + rank, pool_factor=1.0,
                               poison=False, device=device)
    q, kv, q_idx, w_idx, k_idx, bt, sl_t = case
    scale = 1.0 / math.sqrt(192)
    kpad = (topk + 63) // 64 * 64
    rows = B * s_q
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    ns = int(mla_decode._ext.mla_pick_splits(rows, 1, h_q, kpad // 64, sms))
    holder = {}

    def step():
        holder["o"] = dsa_decode.sparse_decode(q, kv, q_idx, w_idx, k_idx, bt, sl_t, topk, scale,
                                               causal, ns)

    step()
    torch.cuda.synchronize()
    # spot check: selection bit-exact on the GPU's own scores, attention vs the oracle
    reqs = [0, 1]
    scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl_t, causal)
    sc = scores[reqs].cpu()
    for j, b in enumerate(reqs):
        sc[j, :, sl[b]:] = -math.inf
    out, lse, idx = holder["o"]
    if not np.array_equal(idx[reqs].cpu().numpy(), oracle.dsa_topk(sc, topk)):
        raise SystemExit("dsa top-k spot check failed")
    sub = cases.mla_subset((q, kv, bt, sl_t), reqs)
    ro, _ = oracle.dsa_sparse_ref(sub[0], sub[1], sub[2], idx[reqs].cpu(), scale)
    if not torch.allclose(out[reqs].float().cpu(), ro, atol=1e-2, rtol=1e-2):
        raise SystemExit("dsa attention spot check failed")
    if dsa_decode.get_status(True) or mla_decode.get_status(True):
        raise SystemExit("dsa device status set")
    del scores, sc, out, lse, idx
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    uuids = [str(torch.cuda.get_device_properties(device).uuid)]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, uuids[0])
        uuids = gathered
    sampler = ClockSampler(uuids) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ms = time_loop(step, args.steps, world, stream)
    clocks = sampler.stop() if sampler else None
    ms_max = max_over_ranks(ms, world, device)
    median_us = max_over_ranks(per_step_median_us(step, min(args.steps, 200), stream), world,
                               device)

    # each stage alone, on the same inputs (stage times sum to about the step)
    st_scores = dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl_t, causal)
    fused = h_q % 128 == 0
    stages = {
        "dsa_indexer_kernel": lambda: dsa_decode.dsa_indexer(q_idx, w_idx, k_idx, bt, sl_t,
                                                             causal),
    }
    if fused:
        # top-k also resolves the selected rows; the MLA kernel fetches them
        st_idx, st_counts, st_rows = dsa_decode.dsa_topk_rows(st_scores, sl_t, topk, bt,
                                                              kv.shape[0], causal)
        stages["dsa_topk_kernel"] = lambda: dsa_decode.dsa_topk_rows(
            st_scores, sl_t, topk, bt, kv.shape[0], causal)
        stages["mla_decode_rows_kernel"] = lambda: dsa_decode.sparse_mla_decode_rows(
            q, kv, st_rows, st_counts, scale, ns)
    else:
        st_idx, st_counts = dsa_decode.dsa_topk(st_scores, sl_t, topk, causal)
        stages["dsa_topk_kernel"] = lambda: dsa_decode.dsa_topk(st_scores, sl_t, topk, causal)
        st_pages = dsa_decode.dsa_gather(kv, bt, st_idx)
        table = dsa_decode._identity_table(rows, kpad // 64, device)
        q_rows = q.reshape(rows, 1, h_q, 576)
        cnt_rows = st_counts.reshape(rows)
        stages["dsa_gather_kernel"] = lambda: dsa_decode.dsa_gather(kv, bt, st_idx)
        stages["mla_decode_kernel"] = lambda: mla_decode.mla_decode(q_rows, st_pages, table,
                                                                    cnt_rows, scale,
                                                                    num_splits=ns)
    n_stage = max(3, min(args.steps, 200))
    stage_ms = {}
    for name, fn in stages.items():
        for _ in range(3):
            fn()
        stage_ms[name] = time_loop(fn, n_stage, 1, stream)
    counts = st_counts.cpu().to(torch.int64)
    vis = [[max(0, min(S, S - s_q + 1 + i)) if causal else S for i in range(s_q)] for S in sl]
    tok_sel = int(counts.sum())
    sum_S = sum(sl)
    stage_bytes = {
        "dsa_indexer_kernel": sum_S * 128 * 2 + rows * n_idx * (128 * 2 + 4) + s_q * sum_S * 4,
        # scores read, indices written (and, fused, the selected rows' block
        # ids read and their cache rows written)
        "dsa_topk_kernel": sum(sum(v) for v in vis) * 4 + rows * topk * 4 * (3 if fused else 1),
    }
    if fused:
        stage_bytes["mla_decode_rows_kernel"] = (tok_sel * 1152 + rows * topk * 4 +
                                                 rows * h_q * (576 + 512) * 2)
    else:
        stage_bytes["dsa_gather_kernel"] = tok_sel * 1152 + rows * kpad * 1152 + rows * topk * 4
        stage_bytes["mla_decode_kernel"] = tok_sel * 1152 + rows * h_q * (576 + 512) * 2
    bytes_local = sum(stage_bytes.values())
    bytes_total = sum_over_ranks(bytes_local, world, device)

    # e2e: q, q_idx, w_idx and the page table up, out back, every step
    out_buf = torch.empty((B, s_q, h_q, 512), dtype=torch.bfloat16, device=device)
    e2e = E2ELoop((q, q_idx, w_idx, bt, sl_t), out_buf, stream)

    def decode(q_d, qi_d, w_d, bt_d, sl_d, out_d):
        o, _, _ = dsa_decode.sparse_decode(q_d, kv, qi_d, w_d, k_idx, bt_d, sl_d, topk, scale,
                                           causal, ns)
        out_d.copy_(o)
    for _ in range(3):
        e2e.step(decode)
    e2e.drain()
    ms_e2e = max_over_ranks(time_loop(lambda: e2e.step(decode), args.steps, world, stream,
                                      finish=e2e.drain), world, device)
    ms_serial = serial_e2e(e2e, decode, args.steps, world, stream, device)
    if dsa_decode.get_status(True) or mla_decode.get_status(True):
        raise SystemExit("dsa device status set after timing")
    if rank != 0:
        return
    peak, peak_src = measured_hbm_peak()
    top = max(stage_ms, key=stage_ms.get)
    achieved = stage_bytes[top] / (stage_ms[top] * 1e-3) / 1e9
    value = bytes_total / (ms_max * 1e-3) / 1e9
    line = {
        "metric": "DSA sparse decode step: algorithmic GB/s (indexer + top-k + MLA over the "
                  "selected rows)",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max, 5),
        "median_us_per_step": round(median_us, 2),
        "pct_of_sol": round(100.0 * value / (peak * world), 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16, cases.make_dsa_case)",
        "config": {"workload": f"dsa_b{B}_sq{s_q}_hq{h_q}_sk{args.mla_sk}_topk{topk}", "B": B,
                   "s_q": s_q, "h_q": h_q, "index_heads": n_idx, "topk": topk,
                   "mean_seq_len": args.mla_sk,
                   "seq_lens": "Normal(mean, mean/2) >= s_q, seeded", "page": 64,
                   "causal": causal, "mla_num_splits": ns, "parallelism": f"dp{world}",
                   "bytes_per_step": int(bytes_total),
                   "l2": "index keys + latent cache > 126 MB L2; no flush needed"},
        "stages_us": {k: round(v * 1e3, 2) for k, v in stage_ms.items()},
        "stage_bytes": {k: int(v) for k, v in stage_bytes.items()},
        "e2e": {"value": round(bytes_total / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(ms_e2e, 5),
                "h2d_bytes_per_step": int(e2e.h2d_bytes * world),
                "d2h_bytes_per_step": int(e2e.d2h_bytes * world),
                "path": "dsa_decode.sparse_decode -> C ABI dsa_indexer_launch, dsa_topk_launch, "
                        "mla_decode_sparse_launch (h_q % 128 == 0; else dsa_gather_launch + "
                        "mla_decode_launch); q, q_idx, w_idx, block_table and seq_lens H2D, out "
                        "D2H every step, double-buffered",
                "serial_ms_per_step": round(ms_serial, 5),
                "serial_value": round(bytes_total / (ms_serial * 1e-3) / 1e9, 2),
                "serial_note": SERIAL_NOTE,
                "copy_note": "q [B, s_q, h_q, 576] (18.9 MB at b=128) and the index queries go up "
                             "and out [B, s_q, h_q, 512] (16.8 MB) comes back over PCIe every "
                             "step, more time than the ~0.3 ms decode itself"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": peak_src, "kernel": top,
                     "algorithmic_bytes_per_launch": int(stage_bytes[top])},
        "gpu_launches": int(args.steps * dsa_launches_per_step(B, s_q, h_q, topk, ns, sms)),
        "clocks": clocks, "cpu_baseline": None,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world, rank, local = dist_env()
    if args.gpus != world and world > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    try:
        if args.workload == "mla":
            run_mla(args, world, rank, local)
            return
        if args.workload == "dsa":
            run_dsa(args, world, rank, local)
            return
        run_ours(args, world, rank, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
