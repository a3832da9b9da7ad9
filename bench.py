"""Benchmark of the paged-attention decode path (one JSON line on rank 0).

Workload (default ``decode_d64``): the large ragged decode sweep — per GPU a batch
of 256 sequences with context lengths log-normal (median 1024, sigma 1.0)
clipped to [16, 32768], bf16 KV, block size 16, one attention layer, 14 query /
2 kv heads, head_dim 64 (``decode_d128``: 28 / 4 heads, head_dim 128).  Block
tables are random over a pool sized to 60% of the GPU's memory.  With N GPUs,
256 * N sequences are drawn and split across ranks by a greedy
longest-first partition into shards with equal KV tokens (weak scaling: per-GPU
work is fixed).

One step = one decode step of one layer for the whole batch: decode append
(slot lookup through the device block tables, write of the step's new K/V
token, context lengths) -> split-K batched decode attention.  `value` is decode algorithmic bytes
(K/V of every context token + q + out + tables + lengths) per second over the
whole step, max over ranks.  Four batches with disjoint random tables rotate so
consecutive steps read different KV blocks (888 MB footprint > 126 MB L2).

Workload ``prefill_d64``: the prefill part of the mixed chunked-prefill step —
per GPU 8 prompt chunks of 512 tokens after prior paged context drawn uniform
in [0, 4096] (``default_rng(0)``), 14 query / 2 kv heads, head_dim 64, bf16.
One step = device metadata -> slot write of the chunks' K/V -> chunked-prefill
attention (tcgen05).  `value` is causal attention FLOPs
(sum over chunks of 4 * H * D * (512 * prior + 512 * 513 / 2)) per second over
the whole step; the roofline is the tensor pipe.  Sixteen batches with disjoint
tables rotate (inputs larger than L2).

``--impl reference`` times the reference's own C++ op (built from its sources
into oracle/_ref) on the host cores on a bounded sample of the same workload;
for ``prefill_d64`` (whose reference is torch code, not a built op) it times
the oracle's C restatement of the reference's attend().
"""

from __future__ import annotations

import argparse
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
    "engine": dict(kind="engine", heads=14, kv_heads=2, head_dim=64),
    # Open-loop Poisson arrivals (--rate requests/s over all GPUs, --duration s):
    # tokens/s over the makespan and TTFT / end-to-end latency percentiles.
    "engine_load": dict(kind="engine_load", heads=14, kv_heads=2, head_dim=64),
}
SEQS_PER_GPU = 256
BLOCK = 16
ROTATIONS = 4
POOL_FRACTION = 0.6
PREFILL_CHUNKS = 8
PREFILL_CHUNK = 512
PREFILL_ROTATIONS = 16
ENGINE_REQUESTS = 1024      # per GPU, all queued at the start
ENGINE_CONCURRENT = 256     # max concurrent sequences per GPU
ENGINE_PREFILL = 512        # prompt tokens per step
ENGINE_PROMPT = (4, 2048)
ENGINE_MAX_TOKENS = (32, 512)
# Default --steps / --warmup per workload kind (engine steps reach steady
# state only after the first admissions' prompts are through).
DEFAULT_STEPS = {"decode": (1000, 20), "prefill": (1000, 20), "engine": (600, 600),
                 "engine_load": (0, 0)}  # engine_load runs for --duration instead


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--warmup", type=int, default=None)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="decode_d64")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="CPU work per CPU-baseline measurement")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--rate", type=float, default=128.0,
                   help="engine_load: arrivals per second over all GPUs")
    p.add_argument("--duration", type=float, default=30.0,
                   help="engine_load: seconds of arrivals")
    p.add_argument("--pool-gb", type=float, default=0.0,
                   help="pool size per GPU in GB (default: 60%% of device memory)")
    args = p.parse_args()
    steps, warmup = DEFAULT_STEPS[WORKLOADS[args.workload]["kind"]]
    args.steps = steps if args.steps is None else args.steps
    args.warmup = warmup if args.warmup is None else args.warmup
    return args


# ------------------------------------------------------------------ workload


def lengths_all(n_gpus: int) -> np.ndarray:
    rng = np.random.default_rng(0)
    lens = rng.lognormal(math.log(1024.0), 1.0, SEQS_PER_GPU * n_gpus)
    return np.clip(np.rint(lens), 16, 32768).astype(np.int64)


def shard(lens: np.ndarray, n: int, rank: int) -> np.ndarray:
    """Longest-first greedy partition into n shards with equal KV tokens."""
    order = np.argsort(-lens, kind="stable")
    loads = np.zeros(n, dtype=np.int64)
    counts = np.zeros(n, dtype=np.int64)
    owner = np.empty(len(lens), dtype=np.int64)
    cap = math.ceil(len(lens) / n)
    for i in order:
        cand = [r for r in range(n) if counts[r] < cap]
        r = min(cand, key=lambda x: (loads[x], x))
        owner[i] = r
        loads[r] += lens[i]
        counts[r] += 1
    return lens[owner == rank]


def algorithmic_bytes(lens, heads, kv_heads, head_dim) -> int:
    """K/V of every context token + q + out (bf16) + table entries + lengths."""
    blocks = sum(-(-int(n) // BLOCK) for n in lens)
    kv = 2 * kv_heads * int(np.sum(lens)) * head_dim * 2
    return kv + len(lens) * heads * head_dim * (2 + 2) + blocks * 4 + len(lens) * 4


def prefill_priors(n_gpus: int, rank: int) -> np.ndarray:
    """Prior context of each rank's chunks: default_rng(0)'s first 8 draws on
    every rank (weak scaling: the same work per GPU), their order rotated by
    the rank."""
    pri = np.random.default_rng(0).integers(0, 4097, PREFILL_CHUNKS)
    return np.roll(pri, rank).astype(np.int64)


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


def measured_peak(key: str, fallback: float):
    """(peak, note) from MEASURED_PEAKS.json, else the stated fallback."""
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        peaks = {}
    if peaks.get(key):
        return float(peaks[key]), f"measured (MEASURED_PEAKS.json {key})"
    return fallback, f"fallback {fallback:g}"


def capture_graphs(prep, kernel, rotations, warmup, dev):
    """Two CUDA graphs per rotation (prep: metadata + slot write; kernel: the
    attention launch), captured on a side stream after eager warm-up.  Returns
    (graphs, capture stream); each entry keeps the metadata tensors its graphs
    write and read alive."""
    import torch

    from batchstream_inference_engine_b200 import ops

    stream = torch.cuda.current_stream(dev)
    capture = torch.cuda.Stream(dev)
    capture.wait_stream(stream)
    with torch.cuda.stream(capture):
        for i in range(warmup):
            kernel(i % rotations, prep(i % rotations))
        ops.take_status(dev)
        graphs = []
        for r in range(rotations):
            ga, gb = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            before = ops.kernel_launches()
            with torch.cuda.graph(ga, stream=capture):
                meta = prep(r)
            with torch.cuda.graph(gb, stream=capture):
                kernel(r, meta)
            # This package's kernels in the pair: each replay launches them again.
            graphs.append((ga, gb, meta, ops.kernel_launches() - before))
        ops.take_status(dev)
    torch.cuda.synchronize(dev)
    return graphs, capture


def take_all_status(capture, dev):
    """Raises if a replayed graph (workspace of the capture stream) or an eager
    call (current stream) recorded a device-side problem."""
    import torch

    from batchstream_inference_engine_b200 import ops

    with torch.cuda.stream(capture):
        ops.take_status(dev)
    ops.take_status(dev)


def timed_replays(graphs, steps, warmup, dev, world):
    """Replays the graphs; returns (total ms, mean attention-kernel ms, clocks).
    Events around the attention graph time the kernel on the launching stream."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.current_stream(dev)
    for i in range(warmup):
        ga, gb, *_ = graphs[i % len(graphs)]
        ga.replay()
        gb.replay()
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev) as clocks:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        torch.cuda.nvtx.range_push("timed")
        for i in range(steps):
            ga, gb, *_ = graphs[i % len(graphs)]
            ga.replay()
            mids[i].record(stream)
            gb.replay()
            ends[i].record(stream)
        torch.cuda.nvtx.range_pop()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    kernel_ms = statistics.mean(m.elapsed_time(e) for m, e in zip(mids, ends))
    return t0.elapsed_time(t1), kernel_ms, clocks.summary()


def capture_steps(step, rotations, dev):
    """One CUDA graph per rotation holding a whole step (PDL edges between its
    launches are kept inside the graph).  Returns (graphs, capture stream,
    this package's kernel launches per graph)."""
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


def replayed_launches(counts, steps):
    """Kernel launches of `steps` replays cycling through graphs with `counts`."""
    return sum(counts[i % len(counts)] for i in range(steps))


def timed_graph_steps(graphs, steps, warmup, dev, world):
    """Replays whole-step graphs; returns (total ms of `steps` steps, clocks)."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.current_stream(dev)
    for i in range(warmup):
        graphs[i % len(graphs)].replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev) as clocks:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        torch.cuda.nvtx.range_push("timed")
        for i in range(steps):
            graphs[i % len(graphs)].replay()
        torch.cuda.nvtx.range_pop()
        t1.record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    return t0.elapsed_time(t1), clocks.summary()


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


# ------------------------------------------------------------------ GPU arm


def run_decode(args):
    import torch
    import torch.distributed as dist

    from batchstream_inference_engine_b200 import ops

    world, rank, dev = setup_process()
    w = WORKLOADS[args.workload]
    H, Hkv, D = w["heads"], w["kv_heads"], w["head_dim"]
    all_lens = lengths_all(world)
    lens = shard(all_lens, world, rank)
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
    q = torch.randn((ROTATIONS, B, H, D), generator=gen, device=dev).bfloat16()
    k_new = torch.randn((ROTATIONS, B, Hkv, D), generator=gen, device=dev).bfloat16()
    v_new = torch.randn((ROTATIONS, B, Hkv, D), generator=gen, device=dev).bfloat16()
    start_pos = torch.tensor(lens - 1, dtype=torch.int32, device=dev)
    out = torch.empty((B, H, D), dtype=torch.bfloat16, device=dev)
    units = Hkv * sum(blocks)
    scale = D ** -0.5

    # The host knows every context length (start + 1), so the decode kernel
    # partitions its work before waiting on the append (lens_ready), and the
    # append writes only each sequence's last block, so the first loads of the
    # other blocks overlap it too (after_append; programmatic dependent launch).
    lens_d = torch.tensor(lens, dtype=torch.int32, device=dev)

    def prep(r):
        ops.decode_append(k_new[r], v_new[r], k_pool, v_pool, tables[r], start_pos)
        return lens_d

    def decode(r, ctx):
        ops.paged_attention_batched(q[r], k_pool, v_pool, tables[r], ctx, scale, out=out,
                                    units_hint=units, lens_ready=True, after_append=True)

    # The step (append + decode) is replayed from one CUDA graph per rotation:
    # `value` and ms_per_step.  The decode kernel alone is timed from a second
    # set of graphs that split the step, with events between the two halves.
    step_graphs, step_capture, step_counts = capture_steps(lambda r: decode(r, prep(r)),
                                                            ROTATIONS, dev)
    total_ms, clock = timed_graph_steps(step_graphs, args.steps, args.warmup, dev, world)
    graphs, capture = capture_graphs(prep, decode, ROTATIONS, args.warmup, dev)
    _, decode_ms, _ = timed_replays(graphs, args.steps, args.warmup, dev, world)
    take_all_status(capture, dev)
    take_all_status(step_capture, dev)
    step_bytes = algorithmic_bytes(lens, H, Hkv, D)

    # End to end through the public API from pinned host buffers: every step
    # ships q, the new K/V rows, the lengths and one table entry per sequence
    # to the device and reads the attention output back.
    stream = torch.cuda.current_stream(dev)
    hq = q[0].cpu().pin_memory()
    hk = k_new[0].cpu().pin_memory()
    hv = v_new[0].cpu().pin_memory()
    hstart = start_pos.cpu().pin_memory()
    hdelta = torch.stack([torch.arange(B, dtype=torch.int64) * width,
                          torch.tensor([b - 1 for b in blocks], dtype=torch.int64)]).pin_memory()
    hout = torch.empty((B, H, D), dtype=torch.bfloat16).pin_memory()
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
    last_entry = e2e_table[torch.arange(B, device=dev), last_col].to(torch.int64)
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
        flat.index_copy_(0, ddelta[b][0] + ddelta[b][1], last_entry.to(torch.int32))
        ctx, _ = ops.decode_append(dk[b], dv[b], k_pool, v_pool, e2e_table, dstart[b])
        ops.paged_attention_batched(dq[b], k_pool, v_pool, e2e_table, ctx, scale, out=dout[b],
                                    units_hint=units)

    def copy_out(b):
        hout.copy_(dout[b], non_blocking=True)

    e2e_ms = time_e2e(copy_in, compute, copy_out, args, dev, world)
    ops.take_status(dev)

    (total_ms, e2e_ms, decode_ms), (job_bytes,) = max_over_ranks(
        [total_ms, e2e_ms, decode_ms], [float(step_bytes)], dev, world)
    result = None
    if rank == 0:
        peak, peak_note = measured_peak("hbm_gbs", 6650.0)
        achieved = step_bytes / (decode_ms / 1e3) / 1e9
        result = {
            "metric": "decode paged-attn HBM GB/s",
            "value": round(job_bytes * args.steps / (total_ms / 1e3) / 1e9, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded lognormal lengths, N(0,1) K/V/q, random block tables)",
            "config": {
                "workload": f"{args.workload}: ragged decode, {SEQS_PER_GPU} seqs/GPU, lognormal "
                            f"(median 1024, sigma 1) lengths clipped to [16, 32768], "
                            f"{H}q/{Hkv}kv d{D}, block 16, one layer",
                "num_seqs_per_gpu": B,
                "kv_tokens_rank0": int(np.sum(lens)),
                "pool_blocks": nb,
                "l2": f"inputs larger than L2: {ROTATIONS} rotating batches with disjoint tables, "
                      f"{ROTATIONS * step_bytes / 1e6:.0f} MB per GPU",
                "step": "decode append (slot lookup + K/V write + lengths) + split-K decode",
                "parallelism": f"dp{world} replicas, no collective on the path",
            },
            "roofline": {
                "bound": "hbm",
                "kernel": "decode_mma_kernel (split-K decode)",
                "achieved": round(achieved, 1),
                "peak": peak,
                "peak_source": peak_note,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": profiled_traffic(args.workload),
                "decode_ms": round(decode_ms, 4),
                "algorithmic_bytes_per_launch": step_bytes,
            },
            "e2e": {"value": round(job_bytes * args.steps / (e2e_ms / 1e3) / 1e9, 1),
                    "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms / args.steps, 4),
                    "path": "pinned host -> device, decode append + decode, device -> pinned host; "
                            "two buffer sets, the next step's copies overlap this step's kernels"},
            "gpu_launches": replayed_launches(step_counts, args.steps),
            "clocks": clock,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        result["cpu_baseline"] = time_cpu(all_lens, H, Hkv, D, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)


def time_e2e(copy_in, compute, copy_out, args, dev, world):
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
        for i in range(max(args.warmup, 2)):
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
    for i in range(args.warmup):
        graphs[i % 2].replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for i in range(args.steps):
        graphs[(args.warmup + i) % 2].replay()
    a1.record(stream)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(cap):
        ops.take_status(dev)  # the captured kernels report through that stream's workspace
    del graphs
    return a0.elapsed_time(a1)


def profiled_traffic(workload: str):
    """DRAM bytes per launch of the attention kernel from the committed ncu
    summary of this workload (profiles/<kernel>_<workload>.md, line
    `traffic_bytes_per_launch: N`), or None when there is none."""
    for path in sorted((ROOT / "profiles").glob(f"*_{workload}.md")):
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return int(line.split(":", 1)[1].strip())
                except ValueError:
                    return None
    return None


def run_prefill(args):
    import torch
    import torch.distributed as dist

    from batchstream_inference_engine_b200 import ops

    world, rank, dev = setup_process()
    w = WORKLOADS[args.workload]
    H, Hkv, D = w["heads"], w["kv_heads"], w["head_dim"]
    n = PREFILL_CHUNK
    R = PREFILL_CHUNKS
    priors = prefill_priors(world, rank)
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

    def prep(r):
        cu, _, slots, ctx = ops.step_metadata(tables[r], start_pos, n_new, T, BLOCK, nb)
        ops.reshape_and_cache(k_new[r], v_new[r], k_pool, v_pool, slots)
        return cu, ctx

    def prefill(r, meta):
        cu, ctx = meta
        ops.prefill_attention(q[r], k_pool, v_pool, tables[r], cu, ctx, scale,
                              max_query_len=n, out=out)

    graphs, capture = capture_graphs(prep, prefill, rot, args.warmup, dev)
    total_ms, kernel_ms, clock = timed_replays(graphs, args.steps, args.warmup, dev, world)
    take_all_status(capture, dev)
    step_flops = prefill_flops(priors, H, D)

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
        ops.prefill_attention(dq[b], k_pool, v_pool, tables[0], cu, ctx, scale, max_query_len=n,
                              out=dout[b])

    def copy_out(b):
        hout.copy_(dout[b], non_blocking=True)

    e2e_ms = time_e2e(copy_in, compute, copy_out, args, dev, world)
    ops.take_status(dev)

    (total_ms, e2e_ms, kernel_ms), (job_flops,) = max_over_ranks(
        [total_ms, e2e_ms, kernel_ms], [float(step_flops)], dev, world)
    result = None
    if rank == 0:
        peak, peak_note = measured_peak("bf16_tflops", 1590.0)
        achieved = step_flops / (kernel_ms / 1e3) / 1e12
        result = {
            "metric": "prefill paged-attn TFLOP/s",
            "value": round(job_flops * args.steps / (total_ms / 1e3) / 1e12, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded priors, N(0,1) K/V/q, random block tables)",
            "config": {
                "workload": f"{args.workload}: {R} prompt chunks x {n} tokens per GPU after prior "
                            f"paged context U[0, 4096] (the same 8 priors on every rank, order "
                            f"rotated by rank), {H}q/{Hkv}kv d{D}, block 16, one layer",
                "priors_rank0": [int(p) for p in prefill_priors(world, 0)],
                "l2": f"inputs larger than L2: {rot} rotating batches with disjoint tables",
                "step": "step metadata + K/V slot write + chunked-prefill attention",
                "parallelism": f"dp{world} replicas, no collective on the path",
            },
            "roofline": {
                "bound": "tensor",
                "kernel": "prefill_kernel (tcgen05 chunked prefill)",
                "achieved": round(achieved, 2),
                "peak": peak,
                "peak_source": peak_note,
                "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4),
                "traffic": profiled_traffic(args.workload),
                "kernel_ms": round(kernel_ms, 4),
                "algorithmic_flops_per_launch": step_flops,
            },
            "e2e": {"value": round(job_flops * args.steps / (e2e_ms / 1e3) / 1e12, 2),
                    "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms / args.steps, 4),
                    "path": "pinned host -> device, metadata + slot write + prefill, device -> "
                            "pinned host; two buffer sets, the next step's copies overlap this step's kernels"},
            "gpu_launches": replayed_launches([g[3] for g in graphs], args.steps),
            "clocks": clock,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        result["cpu_baseline"] = time_cpu_prefill(priors, H, Hkv, D, args.cpu_seconds)
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


def engine_specs(world: int, rank: int):
    """This rank's round-robin share of one global request list
    (ENGINE_REQUESTS per GPU)."""
    from batchstream_inference_engine_b200.replicas import shard_requests
    from batchstream_inference_engine_b200.serve import engine_workload

    specs = engine_workload(ENGINE_REQUESTS * world, seed=1000, prompt_range=ENGINE_PROMPT,
                            max_tokens_range=ENGINE_MAX_TOKENS)
    return shard_requests(specs, world, rank)


def model_flops(stats: dict, config, vocab: int, intermediate: int) -> int:
    """GEMM FLOPs of the processed tokens (projections, MLP) + the output
    projection of the rows + the attention over visible keys."""
    hd = config.hidden_size
    kv = config.num_kv_heads * config.head_dim
    per_token = config.num_layers * 2 * (hd * (hd + 2 * kv) + hd * hd + 3 * hd * intermediate)
    return per_token * stats["tokens"] + 2 * hd * vocab * stats["rows"] + stats["attn_flops"]


def run_engine(args):
    import torch
    import torch.distributed as dist

    from batchstream_inference_engine_b200 import ops
    from batchstream_inference_engine_b200.backend import PagedBackend
    from batchstream_inference_engine_b200.replicas import TokenGather
    from batchstream_inference_engine_b200.serve import BlockBudget, OfflineScheduler
    from batchstream_inference_engine_b200.torch_model import (QWEN25_05B, QWEN25_05B_INTERMEDIATE,
                                                              QWEN25_05B_VOCAB, TorchModel,
                                                              random_weights)

    world, rank, dev = setup_process()
    model = TorchModel(QWEN25_05B, random_weights(), device=dev, dtype=torch.bfloat16)
    blocks = ENGINE_CONCURRENT * -(-(ENGINE_PROMPT[1] + ENGINE_MAX_TOKENS[1]) // BLOCK)
    backend = PagedBackend(model, blocks, BLOCK, ENGINE_PREFILL, max_seqs=ENGINE_CONCURRENT)
    # Pipelined: the host composes step t + 1 while step t runs.
    sched = OfflineScheduler(backend, engine_specs(world, rank), ENGINE_CONCURRENT,
                             BlockBudget(blocks, BLOCK), pipelined=True)
    gather = TokenGather(ENGINE_CONCURRENT, dev)

    def tokens_in(result):
        return 0 if result is None else sum(len(d) for d in result[1])

    def engine_step():
        # The step's token gather runs while the next step computes; the count
        # returned is the previous step's (every rank's tokens).
        return tokens_in(gather.submit(not sched.idle, sched.step()))

    for _ in range(args.warmup):
        engine_step()
    gather.collect()
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    before = dict(model.stats)
    generated = 0
    with ClockSampler(dev) as clocks:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            generated += engine_step()
        generated += tokens_in(gather.collect())
        t1.record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ops.take_status(dev)
    ms = t0.elapsed_time(t1)
    delta = {k: model.stats[k] - before[k] for k in model.stats}
    flops = model_flops(delta, QWEN25_05B, QWEN25_05B_VOCAB, QWEN25_05B_INTERMEDIATE)
    (ms,), (job_flops, job_tokens) = max_over_ranks([ms], [float(flops), float(delta["tokens"])],
                                                     dev, world)
    result = None
    if rank == 0:
        peak, peak_note = measured_peak("bf16_tflops_sustained", 1400.0)
        value = generated / (ms / 1e3)  # every rank's tokens arrive through the gather
        result = {
            "metric": "engine tokens/s",
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
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
                            f"budget per step, greedy, block 16",
                "step": "one engine step: admit + batched forward (metadata, slot writes, "
                        "decode + chunked-prefill attention, GEMMs) + device argmax + "
                        "token gather",
                "processed_tokens_per_s": round(job_tokens / (ms / 1e3), 1),
                "l2": "inputs larger than L2 (weights 1 GB, KV pool per GPU "
                      f"{2 * 24 * 2 * blocks * BLOCK * 64 * 2 / 1e9:.1f} GB)",
                "parallelism": f"dp{world} replicas, round-robin request shards, NCCL "
                               f"all_gather of each step's sampled tokens (side stream, "
                               f"collected one step later)",
            },
            "roofline": {
                "bound": "tensor",
                "kernel": "whole engine step (cuBLAS GEMMs + this package's attention kernels)",
                "achieved": round(job_flops / world / (ms / 1e3) / 1e12, 2),
                "peak": peak,
                "peak_source": peak_note,
                "unit": "TFLOP/s",
                "frac": round(job_flops / world / (ms / 1e3) / 1e12 / peak, 4),
                "traffic": None,
            },
            "e2e": {"value": round(value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": round(delta["h2d_bytes"] / args.steps),
                    "d2h_bytes_per_step": round(delta["d2h_bytes"] / args.steps),
                    "path": "the engine step is the public API: host scheduler -> pinned "
                            "metadata copy -> kernels -> token ids copied back"},
            "gpu_launches": delta["launches"],
            "clocks": clocks.summary(),
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        result["cpu_baseline"] = time_cpu_engine(args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)


ENGINE_MAX_QUEUE = 1024  # waiting requests per GPU before arrivals are rejected


def run_engine_load(args):
    """The reference load test's shape (config: open-loop Poisson arrivals,
    prompts U[4, 2048], max_tokens U[32, 512], 256 concurrent and a queue of 1024
    per GPU, 512-token prefill budget, greedy): the global arrival stream is
    dealt round-robin to the GPUs, each serving its share in real time; latency
    is measured on the host clock from each request's scheduled arrival."""
    import torch
    import torch.distributed as dist

    from batchstream_inference_engine_b200.backend import PagedBackend
    from batchstream_inference_engine_b200.serve import (BlockBudget, load_summary,
                                                          poisson_arrivals, run_open_loop)
    from batchstream_inference_engine_b200.torch_model import (QWEN25_05B, TorchModel,
                                                              random_weights)

    world, rank, dev = setup_process()
    model = TorchModel(QWEN25_05B, random_weights(), device=dev, dtype=torch.bfloat16)
    blocks = ENGINE_CONCURRENT * -(-(ENGINE_PROMPT[1] + ENGINE_MAX_TOKENS[1]) // BLOCK)
    backend = PagedBackend(model, blocks, BLOCK, ENGINE_PREFILL, max_seqs=ENGINE_CONCURRENT)
    graphs = model.warm_graphs(backend.pool)
    arrivals = poisson_arrivals(args.rate, args.duration, seed=2000, prompt_range=ENGINE_PROMPT,
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
    rows = [(r.arrival, r.first_token_at, r.finished_at, r.status, len(r.tokens)) for r in requests]
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, rows)
        rows = [row for part in gathered for row in part]
        steps = [None] * world
        dist.all_gather_object(steps, delta)
    else:
        steps = [delta]
    if rank == 0:
        from batchstream_inference_engine_b200.serve import Request

        merged = []
        for arrival, first, finish, status, n in rows:
            r = Request([], 0, arrival=arrival, first_token_at=first, finished_at=finish,
                        status=status)
            r.tokens = [0] * n
            merged.append(r)
        summ = load_summary(merged)
        total_steps = sum(d["steps"] for d in steps)
        rnd = lambda x: None if x is None else round(x, 4)  # noqa: E731
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
                "workload": f"engine_load: open-loop Poisson {args.rate:g} requests/s over all GPUs "
                            f"for {args.duration:g} s, prompts U{list(ENGINE_PROMPT)}, max_tokens "
                            f"U{list(ENGINE_MAX_TOKENS)}, {ENGINE_CONCURRENT} concurrent and a queue "
                            f"of {ENGINE_MAX_QUEUE} per GPU, {ENGINE_PREFILL}-token prefill budget, "
                            f"greedy, block 16; {graphs} step graphs captured before the run",
                "rate": args.rate, "duration_s": args.duration,
                "parallelism": f"dp{world} replicas, arrivals dealt round-robin",
            },
            "latency": {"ttft_p50_s": rnd(summ["ttft_p50_s"]), "ttft_p99_s": rnd(summ["ttft_p99_s"]),
                        "end_to_end_p50_s": rnd(summ["end_to_end_p50_s"]),
                        "end_to_end_p99_s": rnd(summ["end_to_end_p99_s"]),
                        "clock": "host wall clock from each request's scheduled arrival"},
            "requests": {k: summ[k] for k in ("requests", "completed", "tokens",
                                              "rejected_queue_full", "rejected_too_large",
                                              "failed")},
            "makespan_s": round(summ["makespan_s"], 3),
            "e2e": {"value": round(summ["tokens_per_s"], 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": round(delta["h2d_bytes"] / max(delta["steps"], 1)),
                    "d2h_bytes_per_step": round(delta["d2h_bytes"] / max(delta["steps"], 1)),
                    "path": "the serving loop is the public API"},
            "gpu_launches": sum(d["launches"] for d in steps),
            "clocks": clocks.summary(),
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def time_cpu_engine(seconds, concurrent=16):
    """The oracle's CPU restatement of the reference model step (bf16, all host
    threads for torch) on the engine workload with `concurrent` sequences,
    stepped until `seconds` have passed; generated tokens per second."""
    import torch

    from batchstream_inference_engine_b200.serve import BlockBudget, OfflineScheduler
    from batchstream_inference_engine_b200.torch_model import QWEN25_05B, random_weights
    from oracle.engine import cpu_backend

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    blocks = concurrent * -(-(ENGINE_PROMPT[1] + ENGINE_MAX_TOKENS[1]) // BLOCK)
    backend = cpu_backend(random_weights(), torch.bfloat16, QWEN25_05B, blocks, BLOCK,
                          ENGINE_PREFILL, max_seqs=concurrent)
    sched = OfflineScheduler(backend, engine_specs(1, 0), concurrent, BlockBudget(blocks, BLOCK))
    sched.step()  # warm-up
    generated, steps = 0, 0
    start = time.perf_counter()
    while time.perf_counter() - start < seconds:
        generated += len(sched.step())
        steps += 1
    elapsed = time.perf_counter() - start
    return {"value": round(generated / elapsed, 3), "unit": "tokens/s", "cores": cores,
            "kind": "port",
            "sample": f"{steps} engine steps of the workload with {concurrent} concurrent "
                      f"sequences through the oracle's CPU restatement of the reference "
                      f"model step (bf16), {elapsed:.1f} s, {generated} tokens generated"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    H, Hkv, D = w["heads"], w["kv_heads"], w["head_dim"]
    if w["kind"] in ("engine", "engine_load"):
        return run_reference_engine(args)
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
            res = time_cpu_prefill(prefill_priors(1, 0), H, Hkv, D, seconds)
        else:
            res = time_cpu(lengths_all(1), H, Hkv, D, seconds)
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
        "config": {"workload": "engine: oracle CPU restatement of the reference model step, "
                               "16 concurrent sequences, on host cores"},
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
    elif kind == "engine":
        run_engine(args)
    elif kind == "engine_load":
        run_engine_load(args)
    else:
        run_decode(args)


if __name__ == "__main__":
    main()
