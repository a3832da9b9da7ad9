"""Data-parallel replicas: one process per GPU, each with its own model replica,
pool, block tables and scheduler; sequences never cross GPUs, so the attention
path has no collective.  The one exchange is the per-step token stream: after
every engine step each rank contributes the tokens it sampled, and one
``all_gather`` (NCCL over NVLink on GPUs, gloo on the CPU) gives every rank the
whole step's tokens — the serving front end's view of all replicas.

Every rank takes the same collective steps in the same order: a rank with no
work left still joins each gather (with its ``active`` flag cleared) until all
ranks report idle.
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
        width = 2 + 2 * capacity
        self._send = torch.zeros(width, dtype=torch.int32, device=self.device)
        self._recv = torch.zeros(self.world * width, dtype=torch.int32, device=self.device)
        self._host = torch.zeros(width, dtype=torch.int32,
                                 pin_memory=self.device.type == "cuda")

    def exchange(self, active: bool, outputs: dict[int, int]) -> tuple[bool, list[dict[int, int]]]:
        """Contributes this rank's {seq_id: token} of one step; returns (any
        rank still active, every rank's {seq_id: token})."""
        if len(outputs) > self.capacity:
            raise RuntimeError(f"{len(outputs)} tokens in one step, capacity {self.capacity}")
        rec = self._host
        rec.zero_()
        rec[0] = int(active)
        rec[1] = len(outputs)
        if outputs:
            pairs = torch.tensor([v for kv in outputs.items() for v in kv], dtype=torch.int32)
            rec[2: 2 + pairs.numel()] = pairs
        self._send.copy_(rec, non_blocking=True)
        if self.world > 1:
            dist.all_gather_into_tensor(self._recv, self._send, group=self.group)
            rows = self._recv.view(self.world, -1).cpu()
        else:
            rows = self._send.cpu()[None]
        per_rank = []
        for r in range(self.world):
            n = int(rows[r, 1])
            flat = rows[r, 2: 2 + 2 * n].tolist()
            per_rank.append(dict(zip(flat[0::2], flat[1::2])))
        return bool(rows[:, 0].any()), per_rank


def shard_requests(specs: list, world: int, rank: int) -> list:
    """Round-robin assignment of requests to replicas (request i -> rank i % world)."""
    return [s for i, s in enumerate(specs) if i % world == rank]
