"""Offline continuous batching over a backend: the reference BatchingScheduler's
admission and completion rules (src/server/scheduler.py:112-163) with the
BlockBudget (src/server/kv_budget.py:19-36), run synchronously for a fixed set
of requests that are all queued at the start.

Per loop turn: admit waiting requests from the head of the queue while fewer
than ``max_concurrent`` are active and the budget reserves the head's
ceil((prompt + max_tokens) / block_size) blocks; run one backend step; record
each output token; a request completes on an end-of-generation token or at
``max_tokens`` tokens, releasing its sequence and its reservation.  A
RuntimeError from the step fails every active request, as the reference does.
"""

from __future__ import annotations

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

    @property
    def kv_tokens(self) -> int:
        return len(self.prompt_tokens) + self.max_tokens


class OfflineScheduler:
    """One turn of the loop per ``step()``: admit, run one backend step, record
    and complete.  ``idle`` once every request is done."""

    def __init__(self, backend, specs, max_concurrent: int, budget: BlockBudget):
        self.backend = backend
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
        return not self.waiting and not self.active

    def _complete(self, seq_id: int, request: Request) -> None:
        del self.active[seq_id]
        self.budget.release(request.kv_tokens)
        self.backend.release_sequence(seq_id)
        request.done = True

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
        try:
            outputs = self.backend.step()
        except RuntimeError:
            for seq_id, request in list(self.active.items()):
                request.failed = True
                self._complete(seq_id, request)
            return {}
        for seq_id, output in outputs.items():
            request = self.active[seq_id]
            request.tokens.append(output.token)
            if output.finished or len(request.tokens) >= request.max_tokens:
                self._complete(seq_id, request)
        return {seq_id: output.token for seq_id, output in outputs.items()}


def serve(backend, specs, max_concurrent: int, budget: BlockBudget, on_step=None) -> list[Request]:
    """Runs every (prompt_tokens, max_tokens) in ``specs`` to completion and
    returns the requests in submission order.  ``on_step(tokens)`` is called
    after each backend step with its {seq_id: token}."""
    scheduler = OfflineScheduler(backend, specs, max_concurrent, budget)
    while not scheduler.idle:
        tokens = scheduler.step()
        if on_step is not None:
            on_step(tokens)
    return scheduler.requests


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
