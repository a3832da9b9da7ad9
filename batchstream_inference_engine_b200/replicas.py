"""Data-parallel replicas: one process per GPU, each with its own model replica,
pool, block tables and scheduler; sequences never cross GPUs, so the attention
path has no collective.  The one exchange is the per-step token stream: after
every engine step each rank contributes the tokens it sampled, and one
``all_gather`` (NCCL over NVLink on GPUs, gloo on the CPU) gives every rank the
whole step's tokens — the serving front end's view of all replicas.

The gather of step i runs on its own stream while step i + 1 computes, and is
collected one step later, so a rank that is briefly faster does not stall on
the others every step.  Every rank takes the same collective steps in the same
order: a rank with no work left still joins each gather (with its ``active``
flag cleared) until all ranks report idle.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class TokenGather:
    """Fixed-size per-step record [active, count, (seq_id, token) * capacity]
    (int32) gathered from every rank."""

    def __init__(self, capacity: int, device: torch.device | str, group=None):
        self.capacity = capacity
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.width = 2 + 2 * capacity
        cuda = self.device.type == "cuda"
        # Two of each buffer: step i's gather may still be in flight while step
        # i + 1's record is staged; a buffer is reused only after the gather
        # that read it was waited for.
        self._host = [torch.zeros(self.width, dtype=torch.int32, pin_memory=cuda)
                      for _ in range(2)]
        self._send = [torch.zeros(self.width, dtype=torch.int32, device=self.device)
                      for _ in range(2)]
        self._recv = [torch.zeros(self.world * self.width, dtype=torch.int32, device=self.device)
                      for _ in range(2)]
        self._recv_host = [torch.zeros(self.world * self.width, dtype=torch.int32, pin_memory=cuda)
                           for _ in range(2)]
        self._stream = torch.cuda.Stream(self.device) if cuda else None
        self._pending = None  # (work handle or None, buffer index) of the last submit
        self._turn = 0

    def _stage(self, i: int, active: bool, outputs: dict[int, int]) -> torch.Tensor:
        if len(outputs) > self.capacity:
            raise RuntimeError(f"{len(outputs)} tokens in one step, capacity {self.capacity}")
        rec = self._host[i]
        rec.zero_()
        rec[0] = int(active)
        rec[1] = len(outputs)
        if outputs:
            pairs = torch.tensor([v for kv in outputs.items() for v in kv], dtype=torch.int32)
            rec[2: 2 + pairs.numel()] = pairs
        return rec

    def _decode(self, rows: torch.Tensor) -> tuple[bool, list[dict[int, int]]]:
        per_rank = []
        for r in range(self.world):
            n = int(rows[r, 1])
            flat = rows[r, 2: 2 + 2 * n].tolist()
            per_rank.append(dict(zip(flat[0::2], flat[1::2])))
        return bool(rows[:, 0].any()), per_rank

    def _start(self, i: int, active: bool, outputs: dict[int, int]):
        rec = self._stage(i, active, outputs)
        if self.world == 1:
            return None
        send, recv = self._send[i], self._recv[i]
        if self._stream is None:
            send.copy_(rec)
            return dist.all_gather_into_tensor(recv, send, group=self.group, async_op=True)
        # The record is host data: its copy and the gather wait for nothing on
        # the compute stream, which may already hold the next steps.
        with torch.cuda.stream(self._stream):
            send.copy_(rec, non_blocking=True)
            return dist.all_gather_into_tensor(recv, send, group=self.group, async_op=True)

    def _finish(self, work, i: int) -> tuple[bool, list[dict[int, int]]]:
        if self.world == 1:
            return self._decode(self._host[i][None])
        if self._stream is None:
            work.wait()
            return self._decode(self._recv[i].view(self.world, -1))
        # Wait and read back on the gather's stream: the compute stream, which
        # may hold the next steps already, takes no dependency on the gather.
        with torch.cuda.stream(self._stream):
            work.wait()
            self._recv_host[i].copy_(self._recv[i], non_blocking=True)
        self._stream.synchronize()
        return self._decode(self._recv_host[i].view(self.world, -1))

    def exchange(self, active: bool, outputs: dict[int, int]) -> tuple[bool, list[dict[int, int]]]:
        """Contributes this rank's {seq_id: token} of one step and returns, for
        that same step, (any rank still active, every rank's {seq_id: token})."""
        if self._pending is not None:
            raise RuntimeError("exchange() while a submitted gather is still pending")
        i = self._turn
        self._turn ^= 1
        return self._finish(self._start(i, active, outputs), i)

    def submit(self, active: bool, outputs: dict[int, int]):
        """Starts the gather of one step without waiting for it and returns the
        previous submitted step's result (None for the first)."""
        i = self._turn
        self._turn ^= 1
        work = self._start(i, active, outputs)
        previous = self.collect()
        self._pending = (work, i)
        return previous

    def collect(self):
        """Waits for the last submitted gather: (any rank active, per-rank
        tokens), or None when nothing is pending."""
        if self._pending is None:
            return None
        work, i = self._pending
        self._pending = None
        return self._finish(work, i)


def shard_requests(specs: list, world: int, rank: int) -> list:
    """Round-robin assignment of requests to replicas (request i -> rank i % world)."""
    return [s for i, s in enumerate(specs) if i % world == rank]
