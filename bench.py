"""Benchmark of the B200 paged-attention path (one JSON line on rank 0).

Headline (default ``--workload decode_d64``): the large ragged decode sweep -- per
GPU a batch of 256 sequences with context lengths log-normal (median 1024,
sigma 1.0) clipped to [16, 32768], bf16 KV, block size 16, one attention layer,
14 query / 2 kv heads, head_dim 64.  Every rank draws the same 256 lengths
(``default_rng(0)``) over its own pool and random tables (weak scaling: the
per-GPU work of N GPUs is the work of one).  Block tables are random over a pool
sized to 60% of the GPU's memory.  One step = decode append (slot lookup through
the device block tables, write of the step's new K/V token, context lengths) ->
split-K batched decode attention.  `value` is decode algorithmic bytes (K/V of
every context token + q + out + tables + lengths) per second over the whole
step, summed over ranks.  Four batches with disjoint random tables rotate so
consecutive steps read different KV blocks (888 MB per GPU > 126 MB L2).

Timing: after the warm-up, ``--windows`` windows of exactly ``--steps`` steps
each are timed with CUDA events on the launching stream, each bracketed by a
barrier and a device synchronisation; a window's job time is its maximum over
ranks, and the line reports the median window (the spread and every rank's own
step time beside it).

The same line carries, measured in the same process after the headline (``--sub
none`` skips them; ``--sub engine,mixed_d64`` picks some), one sub-object per
other workload of this path:

* ``decode_d128``: the same sweep at 28 query / 4 kv heads, head_dim 128;
* ``prefill_d64``: 8 prompt chunks of 512 tokens after prior paged context
  U[0, 4096] (``default_rng(0)``) -- metadata, slot write, chunked prefill;
  causal attention FLOPs per second, tensor roofline;
* ``mixed_d64``: the mixed step -- the same 8 chunks plus 248 decode rows
  (log-normal, median 768, clipped to [16, 8192]) in one step on one pool:
  metadata -> slot write of every new token -> batched decode -> chunked
  prefill; decode bytes and prefill FLOPs reported against their own rooflines;
* ``engine``: the paged backend on a random-init Qwen2.5-0.5B-shaped replica
  per GPU (the reference load test's shapes: prompts U[4, 2048], max_tokens
  U[32, 512], 256 concurrent, 512-token prefill budget, greedy, closed loop)
  with the NCCL token gather after every step; generated tokens/s summed over
  ranks, each rank's step time and gather wait beside it.

Each workload also runs alone (``--workload``), and ``engine_load`` runs the
open-loop Poisson load (``--rate``, ``--duration``).

``--impl reference`` times the reference's own C++ op (built from its sources
into oracle/_ref) on the host cores on a bounded sample of the same workload;
for ``prefill_d64`` (whose reference is torch code, not a built op) it times
the oracle's C restatement of the reference's attend().
"""

from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    "decode_d64": dict(kind="decode", heads=14, kv_heads=2, head_dim=64),
    "decode_d128": dict(kind="decode", heads=28, kv_heads=4, head_dim=128),
    "prefill_d64": dict(kind="prefill", heads=14, kv_heads=2, head_dim=64),
    "mixed_d64": dict(kind="mixed", heads=14, kv_heads=2, head_dim=64),
    "engine": dict(kind="engine", heads=14, kv_heads=2, head_dim=64),
    # Open-loop Poisson arrivals (--rate requests/s over all GPUs, --duration s):
    # tokens/s over the makespan and TTFT / end-to-end latency percentiles.
    "engine_load": dict(kind="engine_load", heads=14, kv_heads=2, head_dim=64),
}
# Sub-objects of the default line, in the order they run.
SUITE = ("decode_d128", "prefill_d64", "mixed_d64", "engine")
SEQS_PER_GPU = 256
BLOCK = 16
ROTATIONS = 4
POOL_FRACTION = 0.6
PREFILL_CHUNKS = 8
PREFILL_CHUNK = 512
PREFILL_ROTATIONS = 16
MIXED_DECODE_ROWS = 248
MIXED_ROTATIONS = 4
ENGINE_REQUESTS = 1024      # per GPU, all queued at the start
ENGINE_CONCURRENT = 256     # max concurrent sequences per GPU
ENGINE_PREFILL = 512        # prompt tokens per step
ENGINE_PROMPT = (4, 2048)
ENGINE_MAX_TOKENS = (32, 512)
# Default --steps / --warmup per workload kind (engine steps reach steady
# state only after the first admissions' prompts are through).
DEFAULT_STEPS = {"decode": (200, 20), "prefill": (100, 20), "mixed": (100, 20),
                 "engine": (600, 600), "engine_load": (0, 0)}
# Steps of the sub-objects in the default line: (steps, warmup, windows).
SUB_STEPS = {"decode": (50, 10, 20), "prefill": (50, 10, 10), "mixed": (50, 10, 10),
             "engine": (400, 600, 1)}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--warmup", type=int, default=None)
    p.add_argument("--windows", type=int, default=50,
                   help="timed windows of --steps steps each (the median is reported)")
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="decode_d64")
    p.add_argument("--sub", default="all",
                   help="sub-objects of the decode_d64 line: all, none, or a comma list of "
                        + ", ".join(SUITE))
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="CPU work per CPU-baseline measurement")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--rate", default="128",
                   help="engine_load: arrivals per second over all GPUs (a comma list runs "
                        "each rate in turn on the same replicas)")
    p.add_argument("--duration", type=float, default=30.0,
                   help="engine_load: seconds of arrivals")
    p.add_argument("--pool-gb", type=float, default=0.0,
                   help="pool size per GPU in GB (default: 60%% of device memory)")
    args = p.parse_args()
    steps, warmup = DEFAULT_STEPS[WORKLOADS[args.workload]["kind"]]
    args.steps = steps if args.steps is None else args.steps
    args.warmup = warmup if args.warmup is None else args.warmup
    args.windows = max(1, args.windows)
    if args.sub == "all":
        args.sub = list(SUITE)
    elif args.sub == "none":
        args.sub = []
    else:
        args.sub = [s.strip() for s in args.sub.split(",") if s.strip()]
        unknown = [s for s in args.sub if s not in SUITE]
        if unknown:
            p.error(f"unknown sub-objects {unknown}; choose from {list(SUITE)}")
    return args


# ------------------------------------------------------------------ workload


def decode_lengths() -> np.ndarray:
    """The 256 context lengths of one GPU's batch: log-normal (median 1024,
    sigma 1) from default_rng(0), rounded, clipped to [16, 32768].  Every rank
    uses the same draw."""
    rng = np.random.default_rng(0)
    lens = rng.lognormal(math.log(1024.0), 1.0, SEQS_PER_GPU)
    return np.clip(np.rint(lens), 16, 32768).astype(np.int64)


def algorithmic_bytes(lens, heads, kv_heads, head_dim) -> int:
    """K/V of every context token + q + out (bf16) + table entries + lengths."""
    blocks = sum(-(-int(n) // BLOCK) for n in lens)
    kv = 2 * kv_heads * int(np.sum(lens)) * head_dim * 2
    return kv + len(lens) * heads * head_dim * (2 + 2) + blocks * 4 + len(lens) * 4


def prefill_priors(rank: int = 0) -> np.ndarray:
    """Prior context of each rank's chunks: default_rng(0)'s first 8 draws on
    every rank (weak scaling: the same work per GPU), their order rotated by
    the rank."""
    pri = np.random.default_rng(0).integers(0, 4097, PREFILL_CHUNKS)
    return np.roll(pri, rank).astype(np.int64)


def mixed_shapes() -> tuple[np.ndarray, np.ndarray]:
    """The mixed step of one GPU, all from default_rng(0): the 8 chunks' priors
    U[0, 4096] (the prefill workload's), then 248 decode lengths log-normal
    (median 768, sigma 1) rounded and clipped to [16, 8192] (each length counts
    the step's new token)."""
    rng = np.random.default_rng(0)
    priors = rng.integers(0, 4097, PREFILL_CHUNKS).astype(np.int64)
    lens = rng.lognormal(math.log(768.0), 1.0, MIXED_DECODE_ROWS)
    return priors, np.clip(np.rint(lens), 16, 8192).astype(np.int64)


def prefill_flops(priors, heads, head_dim, n=PREFILL_CHUNK) -> int:
    """QK^T + PV over the keys each query sees: 4 H D (n P + n (n + 1) / 2)."""
    return sum(4 * heads * head_dim * (n * int(p) + n * (n + 1) // 2) for p in priors)


# ------------------------------------------------------------------ shared pieces


def setup_process():
    """(world, rank, device); NCCL process group for N > 1 (short timeout)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    return world, rank, dev


def teardown(world):
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def measured_peak(key: str, fallback: float):
    """(peak, note) from MEASURED_PEAKS.json, else the stated fallback."""
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        peaks = {}
    if peaks.get(key):
        return float(peaks[key]), f"measured (MEASURED_PEAKS.json {key})"
    return fallback, f"fallback {fallback:g}"


def release_memory():
    import gc

    import torch

    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def capture_steps(step, rotations, dev):
    """One CUDA graph per rotation holding a whole step (PDL edges between its
    launches are kept inside the graph), captured after one eager run of each
    rotation.  Returns (graphs, capture stream, this package's kernel launches
    per graph)."""
    import torch

    from batchstream_inference_engine_b200 import ops

    stream = torch.cuda.current_stream(dev)
    capture = torch.cuda.Stream(dev)
    capture.wait_stream(stream)
    graphs = []
    with torch.cuda.stream(capture):
        for r in range(rotations):
            step(r)
        torch.cuda.synchronize(dev)
        ops.take_status(dev)
        counts = []
        for r in range(rotations):
            g = torch.cuda.CUDAGraph()
            before = ops.kernel_launches()
            with torch.cuda.graph(g, stream=capture):
                step(r)
            graphs.append(g)
            counts.append(ops.kernel_launches() - before)
    torch.cuda.synchronize(dev)
    return graphs, capture, counts


def take_all_status(capture, dev):
    """Raises if a replayed graph (workspace of the capture stream) or an eager
    call (current stream) recorded a device-side problem."""
    import torch

    from batchstream_inference_engine_b200 import ops

    with torch.cuda.stream(capture):
        ops.take_status(dev)
    ops.take_status(dev)


def timed_windows(replay, steps, warmup, windows, dev, world, clocks=None):
    """`warmup` untimed steps, then `windows` windows of exactly `steps` steps,
    each bracketed by a barrier and a synchronisation and timed with CUDA
    events on the launching stream.  `replay(i)` enqueues step i.  Returns
    this rank's window times (ms)."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.current_stream(dev)
    for i in range(warmup):
        replay(i)
    torch.cuda.synchronize(dev)
    times = []
    with (clocks if clocks is not None else contextlib.nullcontext()):
        for w in range(windows):
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize(dev)
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for i in range(steps):
                replay(warmup + w * steps + i)
            t1.record(stream)
            torch.cuda.synchronize(dev)
            times.append(t0.elapsed_time(t1))
    if world > 1:
        dist.barrier()
    return times


def time_kernel_chain(launch, rotations, repeats, steps, warmup, dev, world, rounds=5,
                      min_launches=400):
    """Mean device time of one launch: a CUDA graph of rotations x repeats
    launches back to back (launch(r) for each rotation r in turn) replayed
    until about max(steps, min_launches) launches were timed, with CUDA events
    around the replays on the launching stream; `rounds` such timings, the
    median kept (a short run's one timing could catch a stall)."""
    import torch
    import torch.distributed as dist

    from batchstream_inference_engine_b200 import ops

    stream = torch.cuda.current_stream(dev)
    capture = torch.cuda.Stream(dev)
    capture.wait_stream(stream)
    with torch.cuda.stream(capture):
        for r in range(rotations):
            launch(r)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=capture):
            for _ in range(repeats):
                for r in range(rotations):
                    launch(r)
    torch.cuda.synchronize(dev)
    per = rotations * repeats
    replays = max(1, -(-max(steps, min_launches) // per))
    for _ in range(max(1, warmup // per)):
        graph.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    times = []
    for _ in range(rounds):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(replays):
            graph.replay()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        times.append(t0.elapsed_time(t1) / (replays * per))
    with torch.cuda.stream(capture):
        ops.take_status(dev)
    del graph
    return sorted(times)[len(times) // 2]


def gather_rows(values, dev, world):
    """Every rank's list of floats (same length on every rank): [world][n]."""
    import torch
    import torch.distributed as dist

    if world == 1:
        return [list(values)]
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    out = torch.empty((world, t.numel()), dtype=torch.float64, device=dev)
    dist.all_gather_into_tensor(out, t)
    return out.tolist()


def max_over_ranks(values, sums, dev, world):
    """Max over ranks of `values`, sum over ranks of `sums` (floats)."""
    import torch
    import torch.distributed as dist

    if world == 1:
        return list(values), list(sums)
    mx = torch.tensor(values, dtype=torch.float64, device=dev)
    sm = torch.tensor(sums, dtype=torch.float64, device=dev)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return mx.tolist(), sm.tolist()


def window_summary(rows, steps):
    """Per-window job time = max over ranks; the median window and the spread
    (ms per step), and each rank's own median ms per step."""
    job = [max(col) for col in zip(*rows)]
    per_step = sorted(t / steps for t in job)
    q = lambda f: per_step[min(len(per_step) - 1, int(f * len(per_step)))]  # noqa: E731
    return statistics.median(job), {
        "windows": len(job),
        "steps_per_window": steps,
        "ms_per_step_min": round(per_step[0], 5),
        "ms_per_step_p10": round(q(0.1), 5),
        "ms_per_step_median": round(statistics.median(per_step), 5),
        "ms_per_step_p90": round(q(0.9), 5),
        "ms_per_step_max": round(per_step[-1], 5),
        "per_rank_ms_per_step": [round(statistics.median(r) / steps, 5) for r in rows],
    }


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every 2 ms while the
    timed loop runs (reading only; no GPU setting is touched)."""

    REASONS = {
        "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
        "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
        "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
        "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
    }

    def __init__(self, device):
        self.device = device
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._handle = None

    def _open(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.device)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        try:
            self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except pynvml.NVMLError:
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)
        self._nvml = pynvml
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)

    def _run(self):
        nv, h = self._nvml, self._handle
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                pass
            self._stop.wait(0.002)

    def __enter__(self):
        try:
            self._open()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
        return False

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        active = set()
        for _, bits in self.samples:
            for name, const in self.REASONS.items():
                if bits & getattr(self._nvml, const):
                    active.add(name)
        return {"sm_mhz": statistics.median(mhz for mhz, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(active),
                "samples": len(self.samples)}


# ------------------------------------------------------------------ CPU baseline


def cpu_sample_inputs(lens, heads, kv_heads, head_dim, count, seed=7):
    """Host copies of a few sequences of the workload (compact pools, own tables)."""
    import torch

    rng = np.random.default_rng(seed)
    pick = rng.choice(len(lens), size=min(count, len(lens)), replace=False)
    cases = []
    g = torch.Generator().manual_seed(seed)
    for i in pick:
        n = int(lens[i])
        nb = -(-n // BLOCK)
        perm = torch.randperm(nb, generator=g).tolist()
        k = torch.randn(kv_heads, nb, BLOCK, head_dim, generator=g).bfloat16()
        v = torch.randn(kv_heads, nb, BLOCK, head_dim, generator=g).bfloat16()
        q = torch.randn(heads, head_dim, generator=g).bfloat16()
        cases.append((q, k, v, perm, n))
    return cases


def time_cpu(lens, heads, kv_heads, head_dim, seconds):
    """Times the reference C++ op (oracle/_ref) or, if absent, the oracle port,
    called per sequence as the reference calls it, on all host cores (the op
    releases the GIL, so a thread per core runs calls in parallel)."""
    import torch

    import oracle

    op = oracle.load_reference_op()
    kind = "reference" if op is not None else "port"
    cores = os.cpu_count() or 1
    torch.set_num_threads(1)  # the parallelism is across calls, one per core
    cases = cpu_sample_inputs(lens, heads, kv_heads, head_dim, count=64)
    groups = heads // kv_heads

    if op is not None:
        def run(case):
            q, k, v, table, n = case
            op(q, k, v, table, n, BLOCK, groups, head_dim ** -0.5)
    else:
        prepared = [(q.view(torch.int16).numpy().view(np.uint16),
                     k.view(torch.int16).numpy().view(np.uint16),
                     v.view(torch.int16).numpy().view(np.uint16), t, n)
                    for q, k, v, t, n in cases]

        def run(case_index):
            q, k, v, t, n = prepared[case_index]
            oracle.decode(q, k, v, t, n, BLOCK, groups, head_dim ** -0.5)

    items = cases if op is not None else list(range(len(cases)))
    nbytes = [algorithmic_bytes([c[4]], heads, kv_heads, head_dim) for c in cases]
    with ThreadPoolExecutor(max_workers=cores) as pool:
        list(pool.map(run, items[: min(len(items), cores)]))  # warm-up
        done_bytes, calls = 0, 0
        start = time.perf_counter()
        while time.perf_counter() - start < seconds:
            list(pool.map(run, items))
            done_bytes += sum(nbytes)
            calls += len(items)
        elapsed = time.perf_counter() - start
    gbs = done_bytes / elapsed / 1e9
    sample = (f"{len(cases)} sequences of the workload (lengths {min(c[4] for c in cases)}-"
              f"{max(c[4] for c in cases)}), {calls} per-sequence op calls over "
              f"{elapsed:.1f} s, {cores} threads")
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": sample}



def time_e2e(copy_in, compute, copy_out, steps, warmup, dev, world):
    """Device time of `steps` end-to-end steps after `warmup` untimed ones.

    A step's inputs come from pinned host memory (`copy_in(b)` into device set
    b), the public API calls run on them (`compute(b)`), and the result goes back
    to pinned host memory (`copy_out(b)`).  As a serving loop would, consecutive
    steps alternate between two device sets and overlap: one CUDA graph per set
    runs, in parallel branches, compute(b), copy_in(1 - b) (the next step's
    inputs) and copy_out(1 - b) (the previous step's result).  Graph replays run
    one after another, so the branches never share a buffer; every timed step
    moves one step's input and output bytes across PCIe."""
    import torch
    import torch.distributed as dist

    from batchstream_inference_engine_b200 import ops

    stream = torch.cuda.current_stream(dev)
    cap = torch.cuda.Stream(dev)
    xin, xout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        for i in range(max(warmup, 2)):
            copy_in(i % 2)
            compute(i % 2)
            copy_out(i % 2)
        ops.take_status(dev)
    torch.cuda.synchronize(dev)
    graphs = []
    for b in range(2):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            xin.wait_stream(cap)
            xout.wait_stream(cap)
            with torch.cuda.stream(xin):
                copy_in(1 - b)
            with torch.cuda.stream(xout):
                copy_out(1 - b)
            compute(b)
            cap.wait_stream(xin)
            cap.wait_stream(xout)
        graphs.append(g)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(cap):
        copy_in(0)  # the first replayed step's inputs
    torch.cuda.synchronize(dev)
    for i in range(warmup):
        graphs[i % 2].replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for i in range(steps):
        graphs[(warmup + i) % 2].replay()
    a1.record(stream)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(cap):
        ops.take_status(dev)  # the captured kernels report through that stream's workspace
    del graphs
    return a0.elapsed_time(a1)



# ------------------------------------------------------------------ GPU arm: decode


def decode_core(args, world, rank, dev, H, Hkv, D, steps, warmup, windows, label,
                clocks=None, extras=True):
    """The ragged decode sweep on this rank; returns the workload's result dict
    on rank 0 (None elsewhere).  Every rank takes the same collective steps."""
    import torch

    from batchstream_inference_engine_b200 import ops

    lens = decode_lengths()
    B = len(lens)
    blocks = [-(-int(n) // BLOCK) for n in lens]
    width = max(blocks)

    free, total = torch.cuda.mem_get_info(dev)
    block_bytes = 2 * Hkv * BLOCK * D * 2
    nb = int(POOL_FRACTION * total // block_bytes)
    if args.pool_gb > 0:
        nb = int(args.pool_gb * 1e9 // block_bytes)
    nb = min(nb, int(0.9 * free // block_bytes), (2**31 - 1) // (Hkv * BLOCK))
    k_pool = torch.empty((Hkv, nb, BLOCK, D), dtype=torch.bfloat16, device=dev)
    v_pool = torch.empty_like(k_pool)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    k_pool.normal_(generator=gen)
    v_pool.normal_(generator=gen)

    # ROTATIONS batches with disjoint random tables over the pool.
    need = sum(blocks)
    perm = torch.randperm(nb, device=dev, generator=gen)[: need * ROTATIONS].to(torch.int32)
    tables = []
    for r in range(ROTATIONS):
        bt = torch.full((B, width), -1, dtype=torch.int32, device=dev)
        cur = r * need
        for i, m in enumerate(blocks):
            bt[i, :m] = perm[cur: cur + m]
            cur += m
        tables.append(bt)
    del perm
    q = torch.randn((ROTATIONS, B, H, D), generator=gen, device=dev).bfloat16()
    k_new = torch.randn((ROTATIONS, B, Hkv, D), generator=gen, device=dev).bfloat16()
    v_new = torch.randn((ROTATIONS, B, Hkv, D), generator=gen, device=dev).bfloat16()
    start_pos = torch.tensor(lens - 1, dtype=torch.int32, device=dev)
    out = torch.empty((B, H, D), dtype=torch.bfloat16, device=dev)
    units = Hkv * sum(blocks)
    scale = D ** -0.5
    step_bytes = algorithmic_bytes(lens, H, Hkv, D)

    # The host knows every context length (start + 1), so the decode kernel
    # partitions its work before waiting on the append (lens_ready), and the
    # append writes only each sequence's last block, so the first loads of the
    # other blocks overlap it too (after_append; programmatic dependent launch).
    lens_d = torch.tensor(lens, dtype=torch.int32, device=dev)

    def append(r, _state=None):
        ops.decode_append(k_new[r], v_new[r], k_pool, v_pool, tables[r], start_pos)
        return lens_d

    def decode(r, ctx):
        ops.paged_attention_batched(q[r], k_pool, v_pool, tables[r], ctx, scale, out=out,
                                    units_hint=units, lens_ready=True, after_append=True)
        return ctx

    # The step (append + decode) is replayed from one CUDA graph per rotation:
    # `value` and ms_per_step.  The decode kernel alone is timed from a second
    # set of graphs that split the step, with events between the two halves.
    step_graphs, step_capture, step_counts = capture_steps(lambda r: decode(r, append(r)),
                                                           ROTATIONS, dev)
    times = timed_windows(lambda i: step_graphs[i % ROTATIONS].replay(), steps, warmup, windows,
                          dev, world, clocks)
    # The decode kernel's own launch time: one graph of decode launches back to
    # back over the rotations (each launch after the previous one, as in the
    # step), timed over whole replays.
    decode_ms = time_kernel_chain(lambda r: decode(r, lens_d), ROTATIONS, 2, steps, warmup,
                                  dev, world)
    take_all_status(step_capture, dev)

    e2e = per_call = None
    if extras:
        e2e_steps = max(steps, 200)
        e2e, per_call = decode_e2e(args, world, dev, q, k_new, v_new, k_pool, v_pool, tables,
                                   start_pos, blocks, width, units, scale, out, e2e_steps,
                                   max(warmup, 5))

    rows = gather_rows(times, dev, world)
    (decode_ms,), _ = max_over_ranks([decode_ms], [], dev, world)
    if e2e is not None:
        (e2e_ms, call_ms), _ = max_over_ranks([e2e[0], per_call[0]], [], dev, world)
    del step_graphs
    result = None
    if rank == 0:
        job_ms, spread = window_summary(rows, steps)
        job_bytes = world * step_bytes
        peak, peak_note = measured_peak("hbm_gbs", 6650.0)
        achieved = step_bytes / (decode_ms / 1e3) / 1e9
        result = {
            "metric": "decode paged-attn HBM GB/s",
            "value": round(job_bytes * steps / (job_ms / 1e3) / 1e9, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": round(job_ms / steps, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded lognormal lengths, N(0,1) K/V/q, random block tables)",
            "config": {
                "workload": f"{label}: ragged decode, {SEQS_PER_GPU} seqs/GPU, lognormal "
                            f"(median 1024, sigma 1) lengths clipped to [16, 32768], "
                            f"{H}q/{Hkv}kv d{D}, block 16, one layer",
                "num_seqs_per_gpu": B,
                "kv_tokens_per_gpu": int(np.sum(lens)),
                "pool_blocks": nb,
                "l2": f"inputs larger than L2: {ROTATIONS} rotating batches with disjoint tables, "
                      f"{ROTATIONS * step_bytes / 1e6:.0f} MB per GPU",
                "step": "decode append (slot lookup + K/V write + lengths) + split-K decode",
                "parallelism": f"dp{world} replicas, the same lengths on every rank, "
                               f"no collective on the path",
            },
            "timing": spread,
            "roofline": {
                "bound": "hbm",
                "kernel": "decode_mma_kernel + decode_merge_kernel (split-K decode, merge pass)",
                "achieved": round(achieved, 1),
                "peak": peak,
                "peak_source": peak_note,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": None,
                "decode_ms": round(decode_ms, 5),
                "decode_ms_how": "mean time of one decode launch (kernel + merge pass) over a "
                                 "graph of back-to-back launches (the rotations in turn), at "
                                 "least 400 launches per timing, median of 5 timings, max over "
                                 "ranks",
                "algorithmic_bytes_per_launch": step_bytes,
            },
            "gpu_launches": sum(step_counts[i % ROTATIONS] for i in range(steps)) * windows,
        }
        if e2e is not None:
            h2d, d2h = e2e[1], e2e[2]
            result["e2e"] = {
                "value": round(job_bytes * e2e_steps / (e2e_ms / 1e3) / 1e9, 1),
                "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / e2e_steps, 5), "steps": e2e_steps,
                "path": "pinned host -> device, decode append + decode, device -> pinned host "
                        "through the public API; two buffer sets in CUDA graphs, the next "
                        "step's copies overlap this step's kernels"}
            result["e2e_per_call"] = {
                "value": round(job_bytes * e2e_steps / (call_ms / 1e3) / 1e9, 1),
                "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(call_ms / e2e_steps, 5), "steps": e2e_steps,
                "path": "every step a plain call of the public API from Python (argument "
                        "checks, ctypes, tensor-map lookup on the host each step), copies in "
                        "and out on the same stream, no CUDA graph"}
    return result


def decode_e2e(args, world, dev, q, k_new, v_new, k_pool, v_pool, tables, start_pos, blocks,
               width, units, scale, out, steps, warmup):
    """End to end through the public API from pinned host buffers: every step
    ships q, the new K/V rows, the start positions and one table entry per
    sequence to the device and reads the attention output back.  Returns
    ((graph ms, h2d bytes, d2h bytes), (per-call ms,)) for `steps` steps."""
    import torch

    from batchstream_inference_engine_b200 import ops

    B = q.shape[1]
    hq = q[0].cpu().pin_memory()
    hk = k_new[0].cpu().pin_memory()
    hv = v_new[0].cpu().pin_memory()
    hstart = start_pos.cpu().pin_memory()
    hdelta = torch.stack([torch.arange(B, dtype=torch.int64) * width,
                          torch.tensor([b - 1 for b in blocks], dtype=torch.int64)]).pin_memory()
    hout = torch.empty(tuple(out.shape), dtype=torch.bfloat16).pin_memory()
    # Two device sets of inputs and outputs: a step computes on one while the
    # next step's inputs arrive in, and the last step's result leaves, the other.
    dq = [torch.empty_like(q[0]) for _ in range(2)]
    dk = [torch.empty_like(k_new[0]) for _ in range(2)]
    dv = [torch.empty_like(v_new[0]) for _ in range(2)]
    dstart = [torch.empty_like(start_pos) for _ in range(2)]
    ddelta = [torch.empty((2, B), dtype=torch.int64, device=dev) for _ in range(2)]
    dout = [torch.empty_like(out) for _ in range(2)]
    e2e_table = tables[0].clone()
    last_col = torch.tensor([b - 1 for b in blocks], device=dev)
    last_entry = e2e_table[torch.arange(B, device=dev), last_col].to(torch.int32)
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hstart, hdelta))
    d2h = hout.numel() * hout.element_size()

    def copy_in(b):
        dq[b].copy_(hq, non_blocking=True)
        dk[b].copy_(hk, non_blocking=True)
        dv[b].copy_(hv, non_blocking=True)
        dstart[b].copy_(hstart, non_blocking=True)
        ddelta[b].copy_(hdelta, non_blocking=True)

    def compute(b):
        flat = e2e_table.view(-1)
        flat.index_copy_(0, ddelta[b][0] + ddelta[b][1], last_entry)
        ctx, _ = ops.decode_append(dk[b], dv[b], k_pool, v_pool, e2e_table, dstart[b])
        ops.paged_attention_batched(dq[b], k_pool, v_pool, e2e_table, ctx, scale, out=dout[b],
                                    units_hint=units)

    def copy_out(b):
        hout.copy_(dout[b], non_blocking=True)

    e2e_ms = time_e2e(copy_in, compute, copy_out, steps, warmup, dev, world)
    call_ms = time_per_call(copy_in, compute, copy_out, steps, warmup, dev, world)
    ops.take_status(dev)
    return (e2e_ms, h2d, d2h), (call_ms,)


def time_per_call(copy_in, compute, copy_out, steps, warmup, dev, world):
    """Device time of `steps` plain steps: copies in, the public API calls and
    the copy out, enqueued from Python every step on one stream (no graph), so
    the host side of every call is inside the timed region."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.current_stream(dev)
    for _ in range(max(warmup, 2)):
        copy_in(0)
        compute(0)
        copy_out(0)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(steps):
        copy_in(0)
        compute(0)
        copy_out(0)
    a1.record(stream)
    torch.cuda.synchronize(dev)
    return a0.elapsed_time(a1)


def run_decode(args):
    """The default line: the d64 (or d128) sweep, then the sub-objects."""
    w = WORKLOADS[args.workload]
    world, rank, dev = setup_process()
    clocks = ClockSampler(dev)
    result = decode_core(args, world, rank, dev, w["heads"], w["kv_heads"], w["head_dim"],
                         args.steps, args.warmup, args.windows, args.workload, clocks=clocks)
    release_memory()
    if rank == 0:
        result["clocks"] = clocks.summary()
        result["windows"] = args.windows
    if args.workload == "decode_d64":
        for name in args.sub:
            sub = run_sub(name, args, world, rank, dev)
            release_memory()
            if rank == 0:
                result[name] = sub
    teardown(world)
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        result["cpu_baseline"] = time_cpu(decode_lengths(), w["heads"], w["kv_heads"],
                                          w["head_dim"], args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_sub(name, args, world, rank, dev):
    """One sub-object of the default line (rank 0 gets the dict)."""
    w = WORKLOADS[name]
    steps, warmup, windows = SUB_STEPS[w["kind"]]
    clocks = ClockSampler(dev)
    if w["kind"] == "decode":
        res = decode_core(args, world, rank, dev, w["heads"], w["kv_heads"], w["head_dim"],
                          steps, warmup, windows, name, clocks=clocks, extras=False)
    elif w["kind"] == "prefill":
        res = prefill_core(args, world, rank, dev, steps, warmup, windows, clocks=clocks,
                           extras=False)
    elif w["kind"] == "mixed":
        res = mixed_core(args, world, rank, dev, steps, warmup, windows, clocks=clocks)
    else:
        res = engine_core(args, world, rank, dev, steps, warmup, clocks=clocks)
    if rank == 0:
        res["clocks"] = clocks.summary()
        for key in ("vs_baseline", "data", "dtype", "n_gpus"):
            res.pop(key, None)
    return res


# ------------------------------------------------------------------ GPU arm: prefill


def prefill_core(args, world, rank, dev, steps, warmup, windows, clocks=None, extras=True):
    import torch

    from batchstream_inference_engine_b200 import ops

    H, Hkv, D = 14, 2, 64
    n = PREFILL_CHUNK
    R = PREFILL_CHUNKS
    priors = prefill_priors(rank)
    totals = priors + n
    blocks = [-(-int(t) // BLOCK) for t in totals]
    width = max(blocks)
    rot = PREFILL_ROTATIONS
    need = sum(blocks)
    nb = need * rot + 64
    gen = torch.Generator(device=dev).manual_seed(4321 + rank)
    k_pool = torch.randn((Hkv, nb, BLOCK, D), generator=gen, device=dev).bfloat16()
    v_pool = torch.randn((Hkv, nb, BLOCK, D), generator=gen, device=dev).bfloat16()
    perm = torch.randperm(nb, device=dev, generator=gen)[: need * rot].to(torch.int32)
    tables = []
    for r in range(rot):
        bt = torch.full((R, width), -1, dtype=torch.int32, device=dev)
        cur = r * need
        for i, m in enumerate(blocks):
            bt[i, :m] = perm[cur: cur + m]
            cur += m
        tables.append(bt)
    T = R * n
    q = torch.randn((rot, T, H, D), generator=gen, device=dev).bfloat16()
    k_new = torch.randn((rot, T, Hkv, D), generator=gen, device=dev).bfloat16()
    v_new = torch.randn((rot, T, Hkv, D), generator=gen, device=dev).bfloat16()
    start_pos = torch.tensor(priors, dtype=torch.int32, device=dev)
    n_new = torch.full((R,), n, dtype=torch.int32, device=dev)
    out = torch.empty((T, H, D), dtype=torch.bfloat16, device=dev)
    scale = D ** -0.5

    def prep(r, _state=None):
        cu, _, slots, ctx = ops.step_metadata(tables[r], start_pos, n_new, T, BLOCK, nb)
        ops.reshape_and_cache(k_new[r], v_new[r], k_pool, v_pool, slots)
        return cu, ctx

    def prefill(r, meta):
        cu, ctx = meta
        ops.prefill_attention(q[r], k_pool, v_pool, tables[r], cu, ctx, scale,
                              max_query_len=n, out=out)
        return meta

    step_graphs, step_capture, step_counts = capture_steps(lambda r: prefill(r, prep(r)), rot,
                                                           dev)
    times = timed_windows(lambda i: step_graphs[i % rot].replay(), steps, warmup, windows, dev,
                          world, clocks)
    # The prefill kernels' own launch time: a graph of prefill launches back to
    # back over the rotations (metadata and slot writes done beforehand).
    metas = [prep(r) for r in range(rot)]
    kernel_ms = time_kernel_chain(lambda r: prefill(r, metas[r]), rot, 1, steps, warmup, dev,
                                  world)
    take_all_status(step_capture, dev)
    step_flops = prefill_flops(priors, H, D)

    e2e = None
    if extras:
        hq = q[0].cpu().pin_memory()
        hk = k_new[0].cpu().pin_memory()
        hv = v_new[0].cpu().pin_memory()
        hstart = start_pos.cpu().pin_memory()
        hout = torch.empty((T, H, D), dtype=torch.bfloat16).pin_memory()
        dq = [torch.empty_like(q[0]) for _ in range(2)]
        dk = [torch.empty_like(k_new[0]) for _ in range(2)]
        dv = [torch.empty_like(v_new[0]) for _ in range(2)]
        dstart = [torch.empty_like(start_pos) for _ in range(2)]
        dout = [torch.empty_like(out) for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hstart))
        d2h = hout.numel() * hout.element_size()

        def copy_in(b):
            dq[b].copy_(hq, non_blocking=True)
            dk[b].copy_(hk, non_blocking=True)
            dv[b].copy_(hv, non_blocking=True)
            dstart[b].copy_(hstart, non_blocking=True)

        def compute(b):
            cu, _, slots, ctx = ops.step_metadata(tables[0], dstart[b], n_new, T, BLOCK, nb)
            ops.reshape_and_cache(dk[b], dv[b], k_pool, v_pool, slots)
            ops.prefill_attention(dq[b], k_pool, v_pool, tables[0], cu, ctx, scale,
                                  max_query_len=n, out=dout[b])

        def copy_out(b):
            hout.copy_(dout[b], non_blocking=True)

        e2e = (time_e2e(copy_in, compute, copy_out, steps, warmup, dev, world), h2d, d2h)
        ops.take_status(dev)

    rows = gather_rows(times, dev, world)
    (kernel_ms,), _ = max_over_ranks([kernel_ms], [], dev, world)
    if e2e is not None:
        (e2e_ms,), _ = max_over_ranks([e2e[0]], [], dev, world)
    del step_graphs
    result = None
    if rank == 0:
        job_ms, spread = window_summary(rows, steps)
        job_flops = world * step_flops
        peak, peak_note = measured_peak("bf16_tflops", 1590.0)
        achieved = step_flops / (kernel_ms / 1e3) / 1e12
        result = {
            "metric": "prefill paged-attn TFLOP/s",
            "value": round(job_flops * steps / (job_ms / 1e3) / 1e12, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": round(job_ms / steps, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded priors, N(0,1) K/V/q, random block tables)",
            "config": {
                "workload": f"prefill_d64: {R} prompt chunks x {n} tokens per GPU after prior "
                            f"paged context U[0, 4096] (the same 8 priors on every rank, order "
                            f"rotated by rank), {H}q/{Hkv}kv d{D}, block 16, one layer",
                "priors_rank0": [int(p) for p in prefill_priors(0)],
                "l2": f"inputs larger than L2: {rot} rotating batches with disjoint tables",
                "step": "step metadata + K/V slot write + chunked-prefill attention",
                "parallelism": f"dp{world} replicas, no collective on the path",
            },
            "timing": spread,
            "roofline": {
                "bound": "tensor",
                "kernel": "prefill_plan_kernel + prefill_kernel (tcgen05 chunked prefill)",
                "achieved": round(achieved, 2),
                "peak": peak,
                "peak_source": peak_note,
                "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4),
                "traffic": None,
                "kernel_ms": round(kernel_ms, 5),
                "algorithmic_flops_per_launch": step_flops,
            },
            "gpu_launches": sum(step_counts[i % rot] for i in range(steps)) * windows,
        }
        if e2e is not None:
            result["e2e"] = {
                "value": round(job_flops * steps / (e2e_ms / 1e3) / 1e12, 2),
                "unit": "TFLOP/s", "h2d_bytes_per_step": e2e[1], "d2h_bytes_per_step": e2e[2],
                "ms_per_step": round(e2e_ms / steps, 5),
                "path": "pinned host -> device, metadata + slot write + prefill, device -> "
                        "pinned host; two buffer sets, the next step's copies overlap this "
                        "step's kernels"}
    return result


def run_prefill(args):
    world, rank, dev = setup_process()
    clocks = ClockSampler(dev)
    result = prefill_core(args, world, rank, dev, args.steps, args.warmup, args.windows,
                          clocks=clocks)
    if rank == 0:
        result["clocks"] = clocks.summary()
    teardown(world)
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        result["cpu_baseline"] = time_cpu_prefill(prefill_priors(0), 14, 2, 64, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)


# ------------------------------------------------------------------ GPU arm: mixed step


def mixed_core(args, world, rank, dev, steps, warmup, windows, clocks=None):
    """The mixed chunked-prefill + decode step on one pool: rows 0..247 decode
    one token each, rows 248..255 are the 8 prompt chunks.  Step = metadata
    (positions, slots, chunk offsets) -> slot write of all 4344 new tokens ->
    batched decode of the 248 rows -> chunked prefill of the 8 chunks, the
    order of the engine's attention step."""
    import torch

    from batchstream_inference_engine_b200 import ops

    H, Hkv, D = 14, 2, 64
    priors, dec_lens = mixed_shapes()
    Bd, P, n = MIXED_DECODE_ROWS, PREFILL_CHUNKS, PREFILL_CHUNK
    R = Bd + P
    # Context lengths after the step (the new tokens included).
    totals = np.concatenate([dec_lens, priors + n])
    starts = np.concatenate([dec_lens - 1, priors])
    counts = np.concatenate([np.ones(Bd, dtype=np.int64), np.full(P, n)])
    blocks = [-(-int(t) // BLOCK) for t in totals]
    width = max(blocks)
    need = sum(blocks)
    rot = MIXED_ROTATIONS
    nb = need * rot + 64
    gen = torch.Generator(device=dev).manual_seed(777 + rank)
    k_pool = torch.randn((Hkv, nb, BLOCK, D), generator=gen, device=dev).bfloat16()
    v_pool = torch.randn((Hkv, nb, BLOCK, D), generator=gen, device=dev).bfloat16()
    perm = torch.randperm(nb, device=dev, generator=gen)[: need * rot].to(torch.int32)
    tables = []
    for r in range(rot):
        bt = torch.full((R, width), -1, dtype=torch.int32, device=dev)
        cur = r * need
        for i, m in enumerate(blocks):
            bt[i, :m] = perm[cur: cur + m]
            cur += m
        tables.append(bt)
    T = int(counts.sum())
    q = torch.randn((rot, T, H, D), generator=gen, device=dev).bfloat16()
    k_new = torch.randn((rot, T, Hkv, D), generator=gen, device=dev).bfloat16()
    v_new = torch.randn((rot, T, Hkv, D), generator=gen, device=dev).bfloat16()
    start_d = torch.tensor(starts, dtype=torch.int32, device=dev)
    n_d = torch.tensor(counts, dtype=torch.int32, device=dev)
    # Host-known context lengths and chunk offsets, as the engine stages them.
    ctx_d = torch.tensor(totals, dtype=torch.int32, device=dev)
    cu_pre = torch.arange(0, P * n + 1, n, dtype=torch.int32, device=dev)
    out = torch.empty((T, H, D), dtype=torch.bfloat16, device=dev)
    scale = D ** -0.5
    dec_units = Hkv * sum(blocks[:Bd])

    def prep(r, _state=None):
        _, _, slots, _ = ops.step_metadata(tables[r], start_d, n_d, T, BLOCK, nb)
        ops.reshape_and_cache(k_new[r], v_new[r], k_pool, v_pool, slots)
        return slots

    def decode(r, state):
        ops.paged_attention_batched(q[r][:Bd], k_pool, v_pool, tables[r], ctx_d[:Bd], scale,
                                    out=out[:Bd], units_hint=dec_units, lens_ready=True,
                                    after_append=True)
        return state

    def prefill(r, state):
        ops.prefill_attention(q[r][Bd:], k_pool, v_pool, tables[r][Bd:], cu_pre, ctx_d[Bd:],
                              scale, max_query_len=n, out=out[Bd:])
        return state

    def step(r):
        prefill(r, decode(r, prep(r)))

    step_graphs, step_capture, step_counts = capture_steps(step, rot, dev)
    times = timed_windows(lambda i: step_graphs[i % rot].replay(), steps, warmup, windows, dev,
                          world, clocks)
    # Each part's own launch time: graphs of that part's launches back to back
    # over the rotations.
    prep_ms = time_kernel_chain(lambda r: prep(r), rot, 1, steps, warmup, dev, world)
    decode_ms = time_kernel_chain(lambda r: decode(r, None), rot, 1, steps, warmup, dev, world)
    prefill_ms = time_kernel_chain(lambda r: prefill(r, None), rot, 1, steps, warmup, dev, world)
    take_all_status(step_capture, dev)
    dec_bytes = algorithmic_bytes(dec_lens, H, Hkv, D)
    pre_flops = prefill_flops(priors, H, D)
    rows = gather_rows(times, dev, world)
    (prep_ms, decode_ms, prefill_ms), _ = max_over_ranks([prep_ms, decode_ms, prefill_ms], [],
                                                          dev, world)
    del step_graphs
    result = None
    if rank == 0:
        job_ms, spread = window_summary(rows, steps)
        hbm, hbm_note = measured_peak("hbm_gbs", 6650.0)
        tc, tc_note = measured_peak("bf16_tflops", 1590.0)
        dec_gbs = dec_bytes / (decode_ms / 1e3) / 1e9
        pre_tf = pre_flops / (prefill_ms / 1e3) / 1e12
        result = {
            "metric": "mixed chunked-prefill + decode step time",
            "value": round(job_ms / steps, 5),
            "unit": "ms",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": round(job_ms / steps, 5),
            "higher_is_better": False,
            "scaling": "weak",
            "config": {
                "workload": f"mixed_d64: {P} prompt chunks x {n} tokens after priors U[0, 4096] "
                            f"+ {Bd} decode rows, lognormal (median 768, sigma 1) lengths "
                            f"clipped to [16, 8192], default_rng(0); {H}q/{Hkv}kv d{D}, "
                            f"block 16, one layer, one pool",
                "priors": [int(p) for p in priors],
                "decode_kv_tokens": int(dec_lens.sum()),
                "l2": f"inputs larger than L2: {rot} rotating batches with disjoint tables",
                "step": "metadata + slot write of every new token + batched decode (248 rows) "
                        "+ chunked prefill (8 chunks), one stream",
            },
            "timing": spread,
            "parts_ms": {"metadata_and_slot_write": round(prep_ms, 5),
                         "decode": round(decode_ms, 5), "prefill": round(prefill_ms, 5),
                         "how": "mean launch time of each part over a graph of its launches "
                                "back to back (median of 5 timings of at least 400 launches)"},
            "decode": {"bound": "hbm", "algorithmic_bytes": dec_bytes,
                       "achieved": round(dec_gbs, 1), "unit": "GB/s", "peak": hbm,
                       "peak_source": hbm_note, "frac": round(dec_gbs / hbm, 4)},
            "prefill": {"bound": "tensor", "algorithmic_flops": pre_flops,
                        "achieved": round(pre_tf, 2), "unit": "TFLOP/s", "peak": tc,
                        "peak_source": tc_note, "frac": round(pre_tf / tc, 4)},
            "gpu_launches": sum(step_counts[i % rot] for i in range(steps)) * windows,
        }
    return result


def run_mixed(args):
    world, rank, dev = setup_process()
    clocks = ClockSampler(dev)
    result = mixed_core(args, world, rank, dev, args.steps, args.warmup, args.windows,
                        clocks=clocks)
    if rank == 0:
        result.update({"vs_baseline": None, "dtype": "bf16",
                       "data": "synthetic (seeded lengths and priors, N(0,1) K/V/q, random "
                               "block tables)",
                       "clocks": clocks.summary()})
    teardown(world)
    if rank == 0:
        print(json.dumps(result), flush=True)


# ------------------------------------------------------------------ GPU arm: engine


def engine_core(args, world, rank, dev, steps, warmup, clocks=None):
    """Closed-loop engine steps on every rank (config: the reference load
    test's shapes, all requests queued at the start) with the NCCL token gather
    after every step.  Returns the rank-0 result dict."""
    import contextlib

    import torch

    from batchstream_inference_engine_b200 import ops
    from batchstream_inference_engine_b200.backend import PagedBackend
    from batchstream_inference_engine_b200.replicas import TokenGather
    from batchstream_inference_engine_b200.serve import BlockBudget, OfflineScheduler
    from batchstream_inference_engine_b200.torch_model import (QWEN25_05B, QWEN25_05B_INTERMEDIATE,
                                                              QWEN25_05B_VOCAB, TorchModel,
                                                              random_weights)

    model = TorchModel(QWEN25_05B, random_weights(), device=dev, dtype=torch.bfloat16)
    blocks = ENGINE_CONCURRENT * -(-(ENGINE_PROMPT[1] + ENGINE_MAX_TOKENS[1]) // BLOCK)
    backend = PagedBackend(model, blocks, BLOCK, ENGINE_PREFILL, max_seqs=ENGINE_CONCURRENT)
    t_graphs = time.perf_counter()
    graphs = model.warm_graphs(backend.pool)
    t_graphs = time.perf_counter() - t_graphs
    # Pipelined: the host composes step t + 1 while step t runs.
    sched = OfflineScheduler(backend, engine_specs(), ENGINE_CONCURRENT,
                             BlockBudget(blocks, BLOCK), pipelined=True)
    gather = TokenGather(ENGINE_CONCURRENT, dev)
    waited = [0.0]

    def tokens_in(result):
        return 0 if result is None else sum(len(d) for d in result[1])

    def engine_step():
        # The step's token gather runs while the next step computes; the count
        # returned is the previous step's (every rank's tokens).
        tokens = sched.step()
        t = time.perf_counter()
        got = tokens_in(gather.submit(not sched.idle, tokens))
        waited[0] += time.perf_counter() - t
        return got

    for _ in range(warmup):
        engine_step()
    gather.collect()
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    before = dict(model.stats)
    generated = 0
    waited[0] = 0.0
    with (clocks if clocks is not None else contextlib.nullcontext()):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        wall = time.perf_counter()
        t0.record(stream)
        for _ in range(steps):
            generated += engine_step()
        t = time.perf_counter()
        generated += tokens_in(gather.collect())
        waited[0] += time.perf_counter() - t
        t1.record(stream)
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - wall
    ops.take_status(dev)
    ms = t0.elapsed_time(t1)
    delta = {k: model.stats[k] - before[k] for k in model.stats}
    flops = model_flops(delta, QWEN25_05B, QWEN25_05B_VOCAB, QWEN25_05B_INTERMEDIATE)
    # The same loop for half as many steps without the token gather: what the
    # gather costs each rank (at one GPU there is no collective either way).
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    quiet = max(1, steps // 2)
    u0 = torch.cuda.Event(enable_timing=True)
    u1 = torch.cuda.Event(enable_timing=True)
    u0.record(stream)
    for _ in range(quiet):
        sched.step()
    u1.record(stream)
    torch.cuda.synchronize(dev)
    ms_quiet = u0.elapsed_time(u1) / quiet
    per_rank = gather_rows([ms, wall * 1e3, waited[0] * 1e3, float(delta["tokens"]),
                            float(delta["rows"]), float(delta["steps"]), ms_quiet], dev, world)
    (ms_max,), (job_flops, job_tokens) = max_over_ranks(
        [ms], [float(flops), float(delta["tokens"])], dev, world)
    if world > 1:
        torch.distributed.barrier()
    del sched, backend, model, gather
    result = None
    if rank == 0:
        peak, peak_note = measured_peak("bf16_tflops_sustained", 1400.0)
        value = generated / (ms_max / 1e3)  # every rank's tokens arrive through the gather
        dev_ms = [r[0] for r in per_rank]
        wall_ms = [r[1] for r in per_rank]
        wait_ms = [r[2] for r in per_rank]
        quiet_ms = [r[6] for r in per_rank]
        result = {
            "metric": "engine tokens/s",
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": round(ms_max / steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded token-id prompts, random-init weights seed 0 N(0,0.02))",
            "config": {
                "workload": f"engine: random-init Qwen2.5-0.5B-shaped replica per GPU, "
                            f"{ENGINE_REQUESTS} requests per GPU queued at start, prompts "
                            f"U{list(ENGINE_PROMPT)}, max_tokens U{list(ENGINE_MAX_TOKENS)}, "
                            f"{ENGINE_CONCURRENT} concurrent, {ENGINE_PREFILL}-token prefill "
                            f"budget per step, greedy, block 16; {graphs} step graphs captured "
                            f"before the run in {t_graphs:.1f} s",
                "step": "one engine step: admit + batched forward (metadata, slot writes, "
                        "decode + chunked-prefill attention, GEMMs) + device argmax + "
                        "token gather",
                "processed_tokens_per_s": round(job_tokens / (ms_max / 1e3), 1),
                "l2": "inputs larger than L2 (weights 1 GB, KV pool per GPU "
                      f"{2 * 24 * 2 * blocks * BLOCK * 64 * 2 / 1e9:.1f} GB)",
                "parallelism": f"dp{world} replicas, the same request list on every rank, "
                               f"NCCL all_gather of each step's sampled tokens (side stream, "
                               f"collected one step later)",
            },
            "per_rank": {
                "ms_per_step": [round(x / steps, 4) for x in dev_ms],
                "host_ms_per_step": [round(x / steps, 4) for x in wall_ms],
                "gather_wait_ms_per_step": [round(x / steps, 4) for x in wait_ms],
                "ms_per_step_without_gather": [round(x, 4) for x in quiet_ms],
                "processed_tokens": [int(r[3]) for r in per_rank],
                "rows": [int(r[4]) for r in per_rank],
            },
            "limiter": engine_limiter([x / steps for x in dev_ms], quiet_ms, world),
            "roofline": {
                "bound": "tensor",
                "kernel": "whole engine step (cuBLAS GEMMs + this package's attention kernels)",
                "achieved": round(job_flops / world / (ms_max / 1e3) / 1e12, 2),
                "peak": peak,
                "peak_source": peak_note,
                "unit": "TFLOP/s",
                "frac": round(job_flops / world / (ms_max / 1e3) / 1e12 / peak, 4),
                "traffic": None,
            },
            "e2e": {"value": round(value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": round(delta["h2d_bytes"] / steps),
                    "d2h_bytes_per_step": round(delta["d2h_bytes"] / steps),
                    "path": "the engine step is the public API: host scheduler -> pinned "
                            "metadata copy -> kernels -> token ids copied back"},
            "gpu_launches": delta["launches"],
        }
    return result


def engine_limiter(step_ms, quiet_ms, world):
    """Names what bounds the multi-GPU engine from per-rank step times: a
    straggler (the slowest rank over the median), or the token gather (a rank's
    step with the gather over the same loop without it), or neither."""
    med = statistics.median(step_ms)
    straggler = max(step_ms) / med - 1.0
    gather = max(s / q - 1.0 for s, q in zip(step_ms, quiet_ms))
    notes = {"straggler_over_median": round(straggler, 4),
             "gather_cost_over_step": round(gather, 4)}
    if world == 1:
        notes["named"] = "single GPU (no gather)"
    elif straggler > 0.03:
        notes["named"] = "straggler rank"
    elif gather > 0.03:
        notes["named"] = "token gather"
    else:
        notes["named"] = "none above 3%: every rank steps at its rate without the gather"
    return notes


def run_engine(args):
    world, rank, dev = setup_process()
    clocks = ClockSampler(dev)
    result = engine_core(args, world, rank, dev, args.steps, args.warmup, clocks=clocks)
    if rank == 0:
        result["clocks"] = clocks.summary()
    teardown(world)
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        result["cpu_baseline"] = time_cpu_engine(args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)


def time_cpu_prefill(priors, heads, kv_heads, head_dim, seconds):
    """Times the oracle's C restatement of the reference's prefill attend()
    (bf16 rounding points) on the host cores, one chunk per thread (ctypes
    releases the GIL), over rounds of the workload's chunks until `seconds`."""
    import torch

    import oracle

    n = PREFILL_CHUNK
    cores = os.cpu_count() or 1
    g = torch.Generator().manual_seed(11)
    cases = []
    for p in priors:
        total = int(p) + n
        nb = -(-total // BLOCK)
        table = torch.randperm(nb, generator=g).tolist()
        bits = lambda t: t.bfloat16().view(torch.int16).numpy().view(np.uint16)
        cases.append((bits(torch.randn(n, heads, head_dim, generator=g)),
                      bits(torch.randn(kv_heads, nb, BLOCK, head_dim, generator=g)),
                      bits(torch.randn(kv_heads, nb, BLOCK, head_dim, generator=g)),
                      table, int(p)))
    groups = heads // kv_heads

    def run(case):
        q, k, v, table, past = case
        oracle.prefill(q, k, v, table, past, BLOCK, groups, head_dim ** -0.5)

    flops = prefill_flops(priors, heads, head_dim)
    with ThreadPoolExecutor(max_workers=min(cores, len(cases))) as pool:
        done, rounds = 0, 0
        start = time.perf_counter()
        while rounds == 0 or time.perf_counter() - start < seconds:
            list(pool.map(run, cases))
            done += flops
            rounds += 1
        elapsed = time.perf_counter() - start
    sample = (f"{rounds} round(s) of the workload's {len(cases)} chunks ({n} tokens after priors "
              f"{min(priors)}-{max(priors)}) through the oracle's C attend(), {elapsed:.1f} s, "
              f"{min(cores, len(cases))} threads")
    return {"value": round(done / elapsed / 1e12, 6), "unit": "TFLOP/s",
            "cores": min(cores, len(cases)), "kind": "port", "sample": sample}


def engine_specs():
    """The requests of one GPU: ENGINE_REQUESTS token-id prompts from seed 1000.
    Every rank serves the same list (weak scaling: the per-GPU work of N GPUs
    is the work of one)."""
    from batchstream_inference_engine_b200.serve import engine_workload

    return engine_workload(ENGINE_REQUESTS, seed=1000, prompt_range=ENGINE_PROMPT,
                           max_tokens_range=ENGINE_MAX_TOKENS)


def model_flops(stats: dict, config, vocab: int, intermediate: int) -> int:
    """GEMM FLOPs of the processed tokens (projections, MLP) + the output
    projection of the rows + the attention over visible keys."""
    hd = config.hidden_size
    kv = config.num_kv_heads * config.head_dim
    per_token = config.num_layers * 2 * (hd * (hd + 2 * kv) + hd * hd + 3 * hd * intermediate)
    return per_token * stats["tokens"] + 2 * hd * vocab * stats["rows"] + stats["attn_flops"]


ENGINE_MAX_QUEUE = 1024  # waiting requests per GPU before arrivals are rejected


def run_engine_load(args):
    """The reference load test's shape (config: open-loop Poisson arrivals,
    prompts U[4, 2048], max_tokens U[32, 512], 256 concurrent and a queue of 1024
    per GPU, 512-token prefill budget, greedy): the global arrival stream is
    dealt round-robin to the GPUs, each serving its share in real time; latency
    is measured on the host clock from each request's scheduled arrival.  Each
    rate of --rate runs in turn on the same replicas (step graphs captured once,
    before the first)."""
    import torch
    import torch.distributed as dist

    from batchstream_inference_engine_b200.backend import PagedBackend
    from batchstream_inference_engine_b200.serve import (BlockBudget, Request, load_summary,
                                                          poisson_arrivals, run_open_loop)
    from batchstream_inference_engine_b200.torch_model import (QWEN25_05B, TorchModel,
                                                              random_weights)

    rates = [float(r) for r in str(args.rate).split(",") if r.strip()]
    world, rank, dev = setup_process()
    model = TorchModel(QWEN25_05B, random_weights(), device=dev, dtype=torch.bfloat16)
    blocks = ENGINE_CONCURRENT * -(-(ENGINE_PROMPT[1] + ENGINE_MAX_TOKENS[1]) // BLOCK)
    backend = PagedBackend(model, blocks, BLOCK, ENGINE_PREFILL, max_seqs=ENGINE_CONCURRENT)
    graphs = model.warm_graphs(backend.pool)
    rnd = lambda x: None if x is None else round(x, 4)  # noqa: E731
    results, launches, clock_list, last = [], 0, [], None
    for rate in rates:
        arrivals = poisson_arrivals(rate, args.duration, seed=2000, prompt_range=ENGINE_PROMPT,
                                    max_tokens_range=ENGINE_MAX_TOKENS)
        mine = [a for i, a in enumerate(arrivals) if i % world == rank]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        before = dict(model.stats)
        with ClockSampler(dev) as clocks:
            requests = run_open_loop(backend, mine, ENGINE_CONCURRENT, ENGINE_MAX_QUEUE,
                                     BlockBudget(blocks, BLOCK), pipelined=True)
        delta = {k: model.stats[k] - before[k] for k in model.stats}
        rows = [(r.arrival, r.first_token_at, r.finished_at, r.status, len(r.tokens))
                for r in requests]
        if world > 1:
            gathered = [None] * world
            dist.all_gather_object(gathered, rows)
            rows = [row for part in gathered for row in part]
            steps = [None] * world
            dist.all_gather_object(steps, delta)
        else:
            steps = [delta]
        if rank == 0:
            merged = []
            for arrival, first, finish, status, n in rows:
                r = Request([], 0, arrival=arrival, first_token_at=first, finished_at=finish,
                            status=status)
                r.tokens = [0] * n
                merged.append(r)
            summ = load_summary(merged)
            total_steps = sum(d["steps"] for d in steps)
            launches += sum(d["launches"] for d in steps)
            clock_list.append(clocks.summary())
            last = (summ, total_steps, delta)
            results.append({
                "rate": rate, "duration_s": args.duration,
                "tokens_per_s": round(summ["tokens_per_s"], 1),
                "makespan_s": round(summ["makespan_s"], 3), "steps": total_steps,
                "ttft_p50_s": rnd(summ["ttft_p50_s"]), "ttft_p99_s": rnd(summ["ttft_p99_s"]),
                "end_to_end_p50_s": rnd(summ["end_to_end_p50_s"]),
                "end_to_end_p99_s": rnd(summ["end_to_end_p99_s"]),
                "requests": {k: summ[k] for k in ("requests", "completed", "tokens",
                                                  "rejected_queue_full", "rejected_too_large",
                                                  "failed")},
                "clocks": clocks.summary()})
    if rank == 0:
        summ, total_steps, delta = last
        print(json.dumps({
            "metric": "engine tokens/s under open-loop Poisson load",
            "value": round(summ["tokens_per_s"], 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": total_steps,
            "warmup": 0,
            "ms_per_step": round(summ["makespan_s"] * 1e3 * world / max(total_steps, 1), 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded Poisson arrivals of token-id prompts, random-init weights)",
            "config": {
                "workload": f"engine_load: open-loop Poisson arrivals over all GPUs at "
                            f"{', '.join(f'{r:g}' for r in rates)} requests/s, {args.duration:g} s "
                            f"each, prompts U{list(ENGINE_PROMPT)}, max_tokens "
                            f"U{list(ENGINE_MAX_TOKENS)}, {ENGINE_CONCURRENT} concurrent and a queue "
                            f"of {ENGINE_MAX_QUEUE} per GPU, {ENGINE_PREFILL}-token prefill budget, "
                            f"greedy, block 16; {graphs} step graphs captured before the run",
                "rates": rates, "duration_s": args.duration,
                "parallelism": f"dp{world} replicas, arrivals dealt round-robin",
                "value_is": "the last rate's tokens/s",
            },
            "by_rate": results,
            "e2e": {"value": round(summ["tokens_per_s"], 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": round(delta["h2d_bytes"] / max(delta["steps"], 1)),
                    "d2h_bytes_per_step": round(delta["d2h_bytes"] / max(delta["steps"], 1)),
                    "path": "the serving loop is the public API"},
            "gpu_launches": launches,
            "clocks": clock_list[-1],
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def time_cpu_engine(seconds, concurrent=16):
    """The reference's paged backend and scheduler loop as the oracle restates
    them (oracle/engine.py: model step, batch composition, allocator,
    admission), bf16 on all host threads for torch, on the engine workload with
    `concurrent` sequences, stepped until `seconds` have passed; generated
    tokens per second."""
    import torch

    from batchstream_inference_engine_b200.torch_model import QWEN25_05B, random_weights
    from oracle.engine import cpu_backend, run_for

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    blocks = concurrent * -(-(ENGINE_PROMPT[1] + ENGINE_MAX_TOKENS[1]) // BLOCK)
    backend = cpu_backend(random_weights(), torch.bfloat16, QWEN25_05B, blocks, BLOCK,
                          ENGINE_PREFILL)
    generated, steps, elapsed = run_for(backend, engine_specs(), concurrent, blocks, BLOCK,
                                        seconds)
    return {"value": round(generated / elapsed, 3), "unit": "tokens/s", "cores": cores,
            "kind": "port",
            "sample": f"{steps} engine steps of the workload with {concurrent} concurrent "
                      f"sequences through the oracle's restatement of the reference model "
                      f"step, paged backend and scheduler loop (bf16), {elapsed:.1f} s, "
                      f"{generated} tokens generated"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    H, Hkv, D = w["heads"], w["kv_heads"], w["head_dim"]
    if w["kind"] in ("engine", "engine_load"):
        return run_reference_engine(args)
    if w["kind"] == "mixed":
        return run_reference_mixed(args)
    prefill = w["kind"] == "prefill"
    # Each step is a bounded sample of the workload (decode: 64 of its sequences,
    # about a quarter of its KV bytes; prefill: the rank's 8 chunks), so the
    # whole run stays within minutes.
    per_step = max(1.0, min(args.cpu_seconds, 6.0) / 2)
    vals = []
    base = None
    for i in range(args.warmup + args.steps):
        seconds = per_step if i >= args.warmup else 0.2
        if prefill:
            res = time_cpu_prefill(prefill_priors(0), H, Hkv, D, seconds)
        else:
            res = time_cpu(decode_lengths(), H, Hkv, D, seconds)
        if i >= args.warmup:
            vals.append(res["value"])
            base = res
    value = statistics.median(vals)
    base["value"] = value
    unit = base["unit"]
    print(json.dumps({
        "metric": "prefill paged-attn TFLOP/s" if prefill else "decode paged-attn HBM GB/s",
        "impl": "reference",
        "value": value,
        "unit": unit,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded priors, N(0,1) K/V/q)" if prefill
        else "synthetic (seeded lognormal lengths, N(0,1) K/V/q)",
        "config": {"workload": f"{args.workload}: " + (
            "oracle C restatement of the reference attend() per chunk on host cores" if prefill
            else "reference C++ op per sequence on host cores")},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference_mixed(args):
    """Mixed step on the host cores: the reference C++ op over a bounded sample
    of the step's decode rows and the oracle's attend() over its 8 chunks, each
    timed as for its own workload; one step's time is the decode rows' bytes at
    the decode rate plus the chunks' FLOPs at the prefill rate."""
    priors, dec_lens = mixed_shapes()
    per_part = max(1.0, min(args.cpu_seconds, 6.0) / 4)
    vals, dec, pre = [], None, None
    for i in range(args.warmup + args.steps):
        seconds = per_part if i >= args.warmup else 0.2
        dec = time_cpu(dec_lens, 14, 2, 64, seconds)
        pre = time_cpu_prefill(priors, 14, 2, 64, seconds)
        if i >= args.warmup:
            ms = (algorithmic_bytes(dec_lens, 14, 2, 64) / (dec["value"] * 1e9)
                  + prefill_flops(priors, 14, 64) / (pre["value"] * 1e12)) * 1e3
            vals.append(ms)
    value = statistics.median(vals)
    print(json.dumps({
        "metric": "mixed chunked-prefill + decode step time", "impl": "reference",
        "value": round(value, 3), "unit": "ms", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded lengths and priors, N(0,1) K/V/q)",
        "config": {"workload": "mixed_d64: reference C++ op per decode row + the oracle's C "
                               "attend() per chunk, on host cores"},
        "cpu_baseline": {"value": round(value, 3), "unit": "ms", "cores": dec["cores"],
                         "kind": dec["kind"],
                         "sample": f"decode: {dec['sample']}; prefill: {pre['sample']}"},
        "e2e": {"value": round(value, 3), "unit": "ms", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference_engine(args):
    """Engine workload on the host cores through the oracle's restatement of the
    reference model step: each step a bounded sample (a few seconds of CPU
    engine steps at 16 concurrent sequences)."""
    per_step = max(2.0, min(args.cpu_seconds, 10.0))
    vals, base = [], None
    for _ in range(max(1, min(args.steps, 3))):
        base = time_cpu_engine(per_step)
        vals.append(base["value"])
    value = statistics.median(vals)
    base["value"] = value
    print(json.dumps({
        "metric": "engine tokens/s", "impl": "reference", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded token-id prompts, random-init weights seed 0 N(0,0.02))",
        "config": {"workload": "engine: the oracle's restatement of the reference model step, "
                               "paged backend and scheduler loop, 16 concurrent sequences, on "
                               "host cores"},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse_args()
    kind = WORKLOADS[args.workload]["kind"]
    if args.impl == "reference":
        run_reference(args)
    elif kind == "prefill":
        run_prefill(args)
    elif kind == "mixed":
        run_mixed(args)
    elif kind == "engine":
        run_engine(args)
    elif kind == "engine_load":
        run_engine_load(args)
    else:
        run_decode(args)


if __name__ == "__main__":
    main()
