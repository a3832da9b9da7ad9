"""Replica token gather with world_size 2 over gloo on the CPU: every rank takes
the same collective steps, ranks that finish early keep joining until all are
idle, and each rank sees every rank's tokens."""

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from batchstream_inference_engine_b200.replicas import TokenGather, shard_requests


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, steps_per_rank, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gather = TokenGather(capacity=4, device="cpu")
        seen, step, rounds = [], 0, 0
        while True:
            active = step < steps_per_rank[rank]
            outputs = {100 * rank + step: 1000 * rank + step} if active else {}
            step += active
            any_active, per_rank = gather.exchange(active, outputs)
            rounds += 1
            seen.append(per_rank)
            if not any_active:
                break
        queue.put((rank, rounds, seen))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_ranks_gather_every_step_until_all_are_idle():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    steps = [3, 5]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, steps, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, rounds, seen = queue.get(timeout=100)
        results[rank] = (rounds, seen)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    # Both ranks joined the same number of gathers: 5 active rounds + 1 idle.
    assert results[0][0] == results[1][0] == 6
    # Both saw the same stream; rank 1's tokens continue after rank 0 is done.
    assert results[0][1] == results[1][1]
    stream = results[0][1]
    assert stream[0] == [{0: 0}, {100: 1000}]
    assert stream[4] == [{}, {104: 1004}]
    assert stream[5] == [{}, {}]


def _lagged_worker(rank, world, port, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gather = TokenGather(capacity=2, device="cpu")
        results = []
        for step in range(4):
            prev = gather.submit(True, {rank: 10 * step + rank})
            results.append(prev)
        results.append(gather.collect())
        queue.put((rank, results))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_submitted_gathers_return_one_step_later():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lagged_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(queue.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    for rank in range(2):
        res = got[rank]
        assert res[0] is None
        for step in range(4):
            assert res[step + 1] == (True, [{0: 10 * step}, {1: 10 * step + 1}])


def test_single_process_gather_without_a_process_group():
    g = TokenGather(capacity=3, device="cpu")
    active, per_rank = g.exchange(True, {7: 11, 9: 13})
    assert active and per_rank == [{7: 11, 9: 13}]
    with pytest.raises(RuntimeError):
        g.exchange(True, {1: 1, 2: 2, 3: 3, 4: 4})


def test_shard_requests_round_robin():
    specs = list(range(10))
    shards = [shard_requests(specs, 3, r) for r in range(3)]
    assert shards == [[0, 3, 6, 9], [1, 4, 7], [2, 5, 8]]
    assert sorted(sum(shards, [])) == specs


def test_gather_record_layout():
    g = TokenGather(capacity=2, device="cpu")
    g.exchange(False, {5: 6})
    assert g._host[0].tolist() == [0, 1, 5, 6, 0, 0]
    # Turns alternate between the two buffers.
    g.exchange(True, {})
    assert g._host[1].tolist() == [1, 0, 0, 0, 0, 0]


def test_exchange_refuses_to_overtake_a_pending_submit():
    g = TokenGather(capacity=2, device="cpu")
    assert g.submit(True, {1: 2}) is None
    with pytest.raises(RuntimeError):
        g.exchange(True, {})
    assert g.collect() == (True, [{1: 2}])
