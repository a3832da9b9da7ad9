"""Continuous batching over a backend: the reference BatchingScheduler's
admission and completion rules (src/server/scheduler.py:112-163) with the
BlockBudget (src/server/kv_budget.py:19-36), run synchronously — for a fixed set
of requests all queued at the start (``serve``), or under open-loop Poisson
arrivals with a bounded queue (``run_open_loop``, the reference load generator's
workload and latency report: bench/loadgen.py:57-67, 100-114, bench/report.py:
28-71).

Per loop turn: admit waiting requests from the head of the queue while fewer
than ``max_concurrent`` are active and the budget reserves the head's
ceil((prompt + max_tokens) / block_size) blocks; run one backend step; record
each output token; a request completes on an end-of-generation token or at
``max_tokens`` tokens, releasing its sequence and its reservation.  A
RuntimeError from the step fails every active request, as the reference does.
"""

from __future__ import annotations

import math
import time
from collections import deque
from dataclasses import dataclass, field


class BlockBudget:
    """src/server/kv_budget.py:1-36: capacity in blocks, requests reserve their
    worst case rounded up to whole blocks."""

    def __init__(self, num_blocks: int, block_size: int):
        self._capacity = num_blocks
        self.available = num_blocks
        self._block_size = block_size

    def _blocks(self, tokens: int) -> int:
        return -(-tokens // self._block_size)

    def fits_ever(self, tokens: int) -> bool:
        return self._blocks(tokens) <= self._capacity

    def try_reserve(self, tokens: int) -> bool:
        blocks = self._blocks(tokens)
        if blocks > self.available:
            return False
        self.available -= blocks
        return True

    def release(self, tokens: int) -> None:
        self.available += self._blocks(tokens)


@dataclass(eq=False)
class Request:
    prompt_tokens: list[int]
    max_tokens: int
    tokens: list[int] = field(default_factory=list)
    failed: bool = False
    done: bool = False
    issued: int = 0  # tokens launched (pipelined loop)
    retired: bool = False  # its sequence was released with its last tokens in flight
    # Open-loop load: scheduled arrival, first token and finish (seconds from the
    # start of the run), and the outcome ("ok", "failed", "rejected_*").
    arrival: float = 0.0
    first_token_at: float | None = None
    finished_at: float | None = None
    status: str = ""

    @property
    def kv_tokens(self) -> int:
        return len(self.prompt_tokens) + self.max_tokens


class OfflineScheduler:
    """One turn of the loop per ``step()``: admit, run one backend step, record
    and complete.  ``idle`` once every request is done.

    ``pipelined``: each turn launches the next step before it reads the
    previous one, so the host composes step t + 1 while step t runs (the
    backend feeds each generating sequence's last token by reference on the
    device).  Same tokens as the plain loop: a request that reaches max_tokens
    is not launched again, and the one extra row of a sequence that ended on an
    end-of-generation token is dropped."""

    def __init__(self, backend, specs, max_concurrent: int, budget: BlockBudget,
                 pipelined: bool = False, clock=None):
        self.backend = backend
        self.pipelined = pipelined
        self.clock = clock  # when set, token and finish times are recorded
        self._inflight = None
        self.max_concurrent = max_concurrent
        self.budget = budget
        self.requests = [Request(list(p), int(m)) for p, m in specs]
        for r in self.requests:
            if not budget.fits_ever(r.kv_tokens):
                raise RuntimeError("request can never fit in the KV budget")
        self.waiting = deque(self.requests)
        self.active: dict[int, Request] = {}

    @property
    def idle(self) -> bool:
        return not self.waiting and not self.active and self._inflight is None

    def _complete(self, seq_id: int, request: Request) -> None:
        del self.active[seq_id]
        self.budget.release(request.kv_tokens)
        if not request.retired:
            self.backend.release_sequence(seq_id)
        request.done = True
        request.status = "failed" if request.failed else "ok"
        if self.clock is not None:
            request.finished_at = self.clock()

    def _record(self, request: Request, token: int) -> None:
        request.tokens.append(token)
        if self.clock is not None and request.first_token_at is None:
            request.first_token_at = self.clock()

    def _fail_all(self) -> dict[int, int]:
        self._inflight = None
        for seq_id, request in list(self.active.items()):
            request.failed = True
            self._complete(seq_id, request)
        return {}

    def step(self) -> dict[int, int]:
        """Returns {seq_id: token} of the step (empty when idle)."""
        while (self.waiting and len(self.active) < self.max_concurrent
               and self.budget.try_reserve(self.waiting[0].kv_tokens)):
            request = self.waiting.popleft()
            self.active[self.backend.start_sequence(request.prompt_tokens)] = request
        if not self.active:
            if self.waiting:
                raise RuntimeError("the budget cannot admit the next request")
            return {}
        if self.pipelined:
            return self._step_pipelined()
        try:
            outputs = self.backend.step()
        except RuntimeError:
            return self._fail_all()
        for seq_id, output in outputs.items():
            request = self.active[seq_id]
            self._record(request, output.token)
            if output.finished or len(request.tokens) >= request.max_tokens:
                self._complete(seq_id, request)
        return {seq_id: output.token for seq_id, output in outputs.items()}

    def _step_pipelined(self) -> dict[int, int]:
        try:
            launched = self.backend.launch()
            outputs = self.backend.finish(self._inflight) if self._inflight is not None else {}
        except RuntimeError:
            return self._fail_all()
        self._inflight = launched
        if launched is not None:
            for seq_id, _, row in launched.rows:
                request = self.active.get(seq_id)
                if row is None or request is None or request.retired:
                    continue
                request.issued += 1
                if request.issued >= request.max_tokens:
                    # Its last token is in flight: no further rows.  The blocks
                    # may be reused by later steps, which run after this one.
                    self.backend.release_sequence(seq_id)
                    request.retired = True
        recorded = {}
        for seq_id, output in outputs.items():
            request = self.active.get(seq_id)
            if request is None:
                continue  # ended on an end-of-generation token one step earlier
            self._record(request, output.token)
            recorded[seq_id] = output.token
            if output.finished or len(request.tokens) >= request.max_tokens:
                self._complete(seq_id, request)
        return recorded


def serve(backend, specs, max_concurrent: int, budget: BlockBudget, on_step=None,
          pipelined: bool = False) -> list[Request]:
    """Runs every (prompt_tokens, max_tokens) in ``specs`` to completion and
    returns the requests in submission order.  ``on_step(tokens)`` is called
    after each backend step with its {seq_id: token}."""
    scheduler = OfflineScheduler(backend, specs, max_concurrent, budget, pipelined=pipelined)
    while not scheduler.idle:
        tokens = scheduler.step()
        if on_step is not None:
            on_step(tokens)
    return scheduler.requests


@dataclass(frozen=True)
class Arrival:
    time: float  # seconds after the start of the run
    prompt_tokens: list
    max_tokens: int


def poisson_arrivals(rate: float, duration: float, seed: int = 0, vocab_size: int = 151936,
                     prompt_range=(4, 2048), max_tokens_range=(32, 512)) -> list[Arrival]:
    """Open-loop Poisson arrivals at `rate` per second for `duration` seconds:
    exponential gaps from one generator and the requests (token-id prompts of
    uniform length, ids uniform over the vocabulary, max_tokens uniform) from a
    second, so the request sequence is the same at every rate (the reference
    load generator's scheme, bench/loadgen.py:57-67)."""
    import numpy as np

    timing = np.random.default_rng(seed)
    requests = np.random.default_rng(seed + 1)
    arrivals = []
    now = timing.exponential(1.0 / rate)
    while now < duration:
        n = int(requests.integers(prompt_range[0], prompt_range[1] + 1))
        prompt = requests.integers(0, vocab_size, n).tolist()
        max_tokens = int(requests.integers(max_tokens_range[0], max_tokens_range[1] + 1))
        arrivals.append(Arrival(float(now), prompt, max_tokens))
        now += timing.exponential(1.0 / rate)
    return arrivals


def run_open_loop(backend, arrivals: list[Arrival], max_concurrent: int, max_queue: int,
                  budget: BlockBudget, pipelined: bool = True, clock=time.perf_counter,
                  sleep=time.sleep) -> list[Request]:
    """Serves `arrivals` as they come: a request joins the waiting queue at its
    scheduled time, or is rejected when the queue holds `max_queue` requests
    (status "rejected_queue_full") or it can never fit the budget
    ("rejected_too_large"), as the reference scheduler's submit does
    (src/server/scheduler.py:50-58).  Returns every request with its times."""
    start = clock()
    elapsed = lambda: clock() - start  # noqa: E731
    scheduler = OfflineScheduler(backend, [], max_concurrent, budget, pipelined=pipelined,
                                 clock=elapsed)
    queue = deque(arrivals)
    requests = []
    while queue or not scheduler.idle:
        now = elapsed()
        while queue and queue[0].time <= now:
            a = queue.popleft()
            request = Request(list(a.prompt_tokens), a.max_tokens, arrival=a.time)
            requests.append(request)
            if not budget.fits_ever(request.kv_tokens):
                request.status, request.done = "rejected_too_large", True
            elif len(scheduler.waiting) >= max_queue:
                request.status, request.done = "rejected_queue_full", True
            else:
                scheduler.waiting.append(request)
        if scheduler.idle:
            if queue:
                sleep(max(0.0, queue[0].time - elapsed()))
            continue
        scheduler.step()
    return requests


def nearest_rank(values: list[float], percent: float) -> float | None:
    """Nearest-rank percentile (bench/report.py:28-30)."""
    if not values:
        return None
    ordered = sorted(values)
    return ordered[math.ceil(percent / 100 * len(ordered)) - 1]


def load_summary(requests: list[Request]) -> dict:
    """Tokens per second over the makespan (first scheduled arrival to the last
    completion) and TTFT / end-to-end latency percentiles, all measured from the
    scheduled arrival so queueing delay counts (bench/report.py:33-71)."""
    ok = [r for r in requests if r.status == "ok"]
    ttft = [r.first_token_at - r.arrival for r in ok if r.first_token_at is not None]
    e2e = [r.finished_at - r.arrival for r in ok]
    first = min((r.arrival for r in requests), default=0.0)
    makespan = max((r.finished_at for r in ok), default=first) - first
    tokens = sum(len(r.tokens) for r in ok)
    counts = {s: sum(r.status == s for r in requests)
              for s in ("rejected_queue_full", "rejected_too_large", "failed")}
    return {
        "requests": len(requests), "completed": len(ok), "tokens": tokens,
        "makespan_s": makespan,
        "tokens_per_s": tokens / makespan if makespan > 0 else 0.0,
        "ttft_p50_s": nearest_rank(ttft, 50), "ttft_p99_s": nearest_rank(ttft, 99),
        "end_to_end_p50_s": nearest_rank(e2e, 50), "end_to_end_p99_s": nearest_rank(e2e, 99),
        **counts,
    }


def engine_workload(num_requests: int = 24, seed: int = 0, vocab_size: int = 151936,
                    prompt_range=(4, 277), max_tokens_range=(16, 128)):
    """Seeded token-id prompts: lengths uniform in prompt_range, ids uniform over
    the vocabulary, max_tokens uniform in max_tokens_range (inclusive)."""
    import numpy as np

    rng = np.random.default_rng(seed)
    lengths = rng.integers(prompt_range[0], prompt_range[1] + 1, num_requests)
    prompts = [rng.integers(0, vocab_size, int(n)).tolist() for n in lengths]
    max_tokens = rng.integers(max_tokens_range[0], max_tokens_range[1] + 1, num_requests).tolist()
    return list(zip(prompts, max_tokens))
