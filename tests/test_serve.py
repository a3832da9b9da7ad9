"""Host logic of the GPU backend and the offline scheduler, on the CPU with a
fake model (no kernels): batch composition (backend/paged.py:60-99), admission
and completion (scheduler.py:112-163), block budgets (kv_budget.py:19-36)."""

import pytest
import torch

from batchstream_inference_engine_b200.backend import PagedBackend, QwenIds, StepOutput
from batchstream_inference_engine_b200.serve import BlockBudget, Request, engine_workload, serve
from batchstream_inference_engine_b200.torch_model import ModelConfig

TINY = ModelConfig(num_layers=1, hidden_size=8, num_heads=2, num_kv_heads=1, rope_theta=1e4,
                   rms_norm_eps=1e-6)


class FakeModel:
    """Records each step's (seq_id, tokens) rows; the next token of a row is
    1000 + its sequence's cache length after the step (deterministic)."""

    def __init__(self, eog_at=None):
        self.config = TINY
        self.device = torch.device("cpu")
        self.dtype = torch.float32
        self.max_position = 4096
        self.steps = []
        self.eog_at = eog_at or {}
        self.last = []  # ids of the last step, by row (what token references name)

    def next_tokens(self, groups):
        return self.launch_tokens(groups).result()

    def launch_tokens(self, groups):
        resolved = [[self.last[-1 - t] if t < 0 else t for t in tokens] for tokens, _ in groups]
        self.steps.append([(cache.seq_id, toks) for toks, (_, cache) in zip(resolved, groups)])
        out = []
        for tokens, cache in groups:
            cache.reserve(len(tokens))
            cache.advance(len(tokens))
            out.append(self.eog_at.get((cache.seq_id, cache.length), 1000 + cache.length))
        self.last = out
        return FakePending(out)


class FakePending:
    def __init__(self, values):
        self.values = values

    def ref(self, i):
        return -1 - i

    def result(self):
        return self.values


def make_backend(model=None, num_blocks=64, prefill_chunk=8):
    return PagedBackend(model or FakeModel(), num_blocks, 16, prefill_chunk)


def test_generating_rows_come_first_then_chunks_under_the_budget():
    model = FakeModel()
    b = make_backend(model, prefill_chunk=8)
    a = b.start_sequence(list(range(5)))
    c = b.start_sequence(list(range(10, 22)))
    out = b.step()
    # Budget 8: all 5 of a, 3 of c; only a is done with its prompt.
    assert model.steps[-1] == [(a, [0, 1, 2, 3, 4]), (c, [10, 11, 12])]
    assert out == {a: StepOutput(1005, False)}
    out = b.step()
    # a generates first, then c's next 8 prompt tokens.
    assert model.steps[-1] == [(a, [1005]), (c, [13, 14, 15, 16, 17, 18, 19, 20])]
    assert out == {a: StepOutput(1006, False)}
    out = b.step()
    assert model.steps[-1] == [(a, [1006]), (c, [21])]
    assert out == {a: StepOutput(1007, False), c: StepOutput(1012, False)}


def test_end_of_generation_stops_a_sequence():
    model = FakeModel(eog_at={(0, 4): 151645})
    b = make_backend(model)
    s = b.start_sequence([1, 2, 3])
    assert b.step() == {s: StepOutput(1003, False)}
    assert b.step() == {s: StepOutput(151645, True)}
    assert b.step() == {}
    b.release_sequence(s)
    assert b.blocks_in_use == 0


def test_blocks_follow_the_reference_allocator():
    b = make_backend()
    s = b.start_sequence(list(range(40)))
    for _ in range(5):
        b.step()
    # 40 prompt tokens + 1 generated (the last step's token is not cached yet).
    assert b.pool.block_table(s) == [63, 62, 61]
    b.release_sequence(s)
    assert b.pool.allocator._free[-3:] == [63, 62, 61]


def test_serve_admits_in_order_up_to_the_limit_and_completes_at_max_tokens():
    model = FakeModel()
    b = make_backend(model, num_blocks=64, prefill_chunk=64)
    specs = [([1] * 5, 3), ([2] * 5, 2), ([3] * 5, 4)]
    requests = serve(b, specs, max_concurrent=2, budget=BlockBudget(64, 16))
    assert [len(r.tokens) for r in requests] == [3, 2, 4]
    assert all(r.done and not r.failed for r in requests)
    # The third request waits until one of the first two completes.
    first_rows = [sid for sid, _ in model.steps[0]]
    assert first_rows == [0, 1]
    assert b.blocks_in_use == 0


def test_serve_holds_the_head_until_the_budget_fits():
    model = FakeModel()
    b = make_backend(model, num_blocks=4, prefill_chunk=64)
    # Each request reserves ceil((prompt + max_tokens) / 16) blocks: 3, then 2.
    specs = [([1] * 30, 10), ([2] * 10, 10)]
    requests = serve(b, specs, max_concurrent=8, budget=BlockBudget(4, 16))
    assert all(r.done for r in requests)
    # Never both active: the second only starts after the first completed.
    assert all(len(step) == 1 for step in model.steps)


@pytest.mark.parametrize("num_blocks", [64, 6])
def test_pipelined_loop_gives_the_same_tokens(num_blocks):
    # Ends by end-of-generation tokens and by max_tokens, admissions gated by
    # the concurrency limit and (with 6 blocks) by the budget.
    specs = [([1] * 5, 6), ([2] * 20, 3), ([3] * 2, 8), ([4] * 9, 5), ([5] * 3, 7), ([6], 4)]
    eog = {(0, 8): 151645, (2, 4): 151643, (4, 5): 151645}
    runs = []
    for pipelined in (False, True):
        model = FakeModel(eog_at=eog)
        b = make_backend(model, num_blocks=num_blocks, prefill_chunk=8)
        requests = serve(b, specs, max_concurrent=3, budget=BlockBudget(num_blocks, 16),
                         pipelined=pipelined)
        assert all(r.done and not r.failed for r in requests)
        assert b.blocks_in_use == 0
        runs.append([r.tokens for r in requests])
    assert runs[0] == runs[1]
    assert runs[0][0][-1] == 151645 and len(runs[0][0]) < 6  # stopped early
    assert [len(t) for t in runs[0]][1] == 3  # stopped at max_tokens


class BrokenAtLaunch(FakeModel):
    def launch_tokens(self, groups):
        raise RuntimeError("launch failed")


class BrokenAtResult(FakeModel):
    """Fails when a step's ids are read (a device-side status bit)."""

    def launch_tokens(self, groups):
        pending = super().launch_tokens(groups)

        def result():
            raise RuntimeError("device-side status")
        pending.result = result
        return pending


@pytest.mark.parametrize("model", [BrokenAtLaunch, BrokenAtResult])
@pytest.mark.parametrize("pipelined", [False, True])
def test_serve_fails_every_active_request_on_a_step_error(model, pipelined):
    b = make_backend(model())
    requests = serve(b, [([1, 2], 4), ([3], 4)], max_concurrent=8, budget=BlockBudget(64, 16),
                     pipelined=pipelined)
    assert all(r.failed and r.done for r in requests)
    assert b.blocks_in_use == 0


def test_budget_rounds_to_blocks():
    budget = BlockBudget(10, 16)
    assert budget.fits_ever(160) and not budget.fits_ever(161)
    assert budget.try_reserve(17) and budget.available == 8
    budget.release(17)
    assert budget.available == 10


def test_request_too_large_is_rejected():
    with pytest.raises(RuntimeError):
        serve(make_backend(), [([1] * 100, 100)], 8, BlockBudget(4, 16))


def test_engine_workload_shape():
    specs = engine_workload()
    assert len(specs) == 24
    assert all(4 <= len(p) <= 277 and 16 <= m <= 128 for p, m in specs)
    assert all(0 <= t < 151936 for p, _ in specs for t in p)
    assert engine_workload() == specs


def test_qwen_ids_vocabulary():
    v = QwenIds()
    assert v.is_end_of_generation(151643) and v.is_end_of_generation(151645)
    assert not v.is_end_of_generation(0)
    with pytest.raises(RuntimeError):
        v.tokenize("text")


def test_request_kv_tokens():
    assert Request([1, 2, 3], 5).kv_tokens == 8


class FakeClock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t

    def sleep(self, dt):
        self.t += dt


class TimedModel(FakeModel):
    """Every step takes `dt` seconds of the fake clock."""

    def __init__(self, clock, dt=0.01, **kw):
        super().__init__(**kw)
        self.clock, self.dt = clock, dt

    def launch_tokens(self, groups):
        self.clock.t += self.dt
        return super().launch_tokens(groups)


@pytest.mark.parametrize("pipelined", [False, True])
def test_open_loop_latencies_are_measured_from_the_scheduled_arrival(pipelined):
    from batchstream_inference_engine_b200.serve import Arrival, load_summary, run_open_loop

    clock = FakeClock()
    b = make_backend(TimedModel(clock, dt=0.01), num_blocks=64, prefill_chunk=64)
    arrivals = [Arrival(0.0, [1] * 4, 3), Arrival(0.5, [2] * 4, 2), Arrival(0.505, [3] * 4, 2)]
    reqs = run_open_loop(b, arrivals, max_concurrent=8, max_queue=8, budget=BlockBudget(64, 16),
                         pipelined=pipelined, clock=clock, sleep=clock.sleep)
    assert [r.status for r in reqs] == ["ok"] * 3
    assert [len(r.tokens) for r in reqs] == [3, 2, 2]
    # The first request's first token comes with its prefill step (one step,
    # or two when its result is read one turn later).
    steps = 2 if pipelined else 1
    assert reqs[0].first_token_at == pytest.approx(0.01 * steps)
    # The idle loop slept until the second arrival: no queueing delay counted.
    assert reqs[1].first_token_at - reqs[1].arrival == pytest.approx(0.01 * steps)
    s = load_summary(reqs)
    assert s["completed"] == 3 and s["tokens"] == 7
    assert s["makespan_s"] == pytest.approx(max(r.finished_at for r in reqs))
    assert s["ttft_p99_s"] >= s["ttft_p50_s"] > 0


def test_open_loop_rejects_when_the_queue_is_full_or_a_request_never_fits():
    from batchstream_inference_engine_b200.serve import Arrival, load_summary, run_open_loop

    clock = FakeClock()
    b = make_backend(TimedModel(clock, dt=1.0), num_blocks=8, prefill_chunk=64)
    # One active at a time, a queue of one, steps of one second: the second
    # arrival finds the first still queued; the third comes after the first was
    # admitted (the queue is empty again), the fourth while the third waits; a
    # fifth can never fit 8 blocks.
    arrivals = [Arrival(0.0, [1] * 4, 2), Arrival(0.0, [2] * 4, 2), Arrival(0.5, [3] * 4, 2),
                Arrival(0.6, [4] * 4, 2), Arrival(0.7, [9] * 200, 1)]
    reqs = run_open_loop(b, arrivals, max_concurrent=1, max_queue=1, budget=BlockBudget(8, 16),
                         pipelined=True, clock=clock, sleep=clock.sleep)
    assert [r.status for r in reqs] == ["ok", "rejected_queue_full", "ok", "rejected_queue_full",
                                        "rejected_too_large"]
    s = load_summary(reqs)
    assert s["rejected_queue_full"] == 2 and s["rejected_too_large"] == 1 and s["completed"] == 2
    # The third waited for the first to finish: its latency includes the queueing.
    assert reqs[2].first_token_at - reqs[2].arrival > 1.0


def test_nearest_rank_percentile_and_poisson_arrivals():
    from batchstream_inference_engine_b200.serve import nearest_rank, poisson_arrivals

    assert nearest_rank([5.0, 1.0, 3.0, 2.0, 4.0], 50) == 3.0
    assert nearest_rank(list(range(1, 101)), 99) == 99
    assert nearest_rank([], 50) is None
    slow = poisson_arrivals(8, 30.0, seed=3)
    fast = poisson_arrivals(128, 30.0, seed=3)
    assert 160 <= len(slow) <= 320 and 3500 <= len(fast) <= 4200  # ~rate x duration
    assert all(0 < a.time < 30 for a in fast)
    assert all(b.time > a.time for a, b in zip(fast, fast[1:]))
    # The same requests in the same order at every rate.
    assert [(a.prompt_tokens, a.max_tokens) for a in slow] == \
        [(a.prompt_tokens, a.max_tokens) for a in fast[: len(slow)]]
    assert all(4 <= len(a.prompt_tokens) <= 2048 and 32 <= a.max_tokens <= 512 for a in fast)
