"""Block allocator with device-resident block tables.

``BlockAllocator`` keeps the reference's semantics exactly
(src/server/block_allocator.py:5-33): a LIFO free list that starts as
``range(num_blocks)``, per-sequence tables that grow to ceil(tokens / block_size)
blocks, all-or-nothing allocation raising ``OutOfBlocks`` (a RuntimeError), and
``free`` returning a table's blocks in table order.  On top of that it mirrors
every table into an int32 tensor ``[max_seqs, max_blocks_per_seq]`` on the GPU
(one row per live sequence), so kernels read block tables and context lengths
from device memory; only new table entries cross PCIe, batched into one copy per
``sync_device()``.
"""

from __future__ import annotations

import torch


class OutOfBlocks(RuntimeError):
    """The pool (or the device table) cannot hold a sequence's next blocks;
    nothing was taken.  A RuntimeError, as the reference raises it."""


class BlockAllocator:
    def __init__(self, num_blocks: int, block_size: int, max_seqs: int = 0,
                 max_blocks_per_seq: int = 0, device: torch.device | str | None = None):
        self._block_size = block_size
        self._free = list(range(num_blocks))
        self._tables: dict[int, list[int]] = {}
        self.num_blocks = num_blocks
        # Device mirror (optional).
        self._device = torch.device(device) if device is not None else None
        self.max_seqs = max_seqs
        self.max_blocks_per_seq = max_blocks_per_seq
        self._rows: dict[int, int] = {}
        self._free_rows = list(range(max_seqs - 1, -1, -1))
        self._synced: dict[int, int] = {}  # entries of each table already on the device
        self.device_tables: torch.Tensor | None = None
        if self._device is not None:
            if max_seqs <= 0 or max_blocks_per_seq <= 0:
                raise ValueError("a device mirror needs max_seqs and max_blocks_per_seq")
            self.device_tables = torch.full((max_seqs, max_blocks_per_seq), -1,
                                            dtype=torch.int32, device=self._device)

    # ---------------------------------------------------------------- reference API

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    @property
    def block_size(self) -> int:
        return self._block_size

    def allocate(self, seq_id: int, total_tokens: int) -> None:
        """Extends seq_id's table (creating it if new) to ceil(total_tokens /
        block_size) blocks, taking each from the end of the free list; takes
        none and raises OutOfBlocks when the free list is too short."""
        table = self._tables.get(seq_id, [])
        missing = -(-total_tokens // self._block_size) - len(table)
        if missing > len(self._free):
            raise OutOfBlocks(f"sequence {seq_id} needs {missing} more blocks but only "
                              f"{len(self._free)} are free")
        needed = missing
        if self.device_tables is not None:
            if len(table) + max(needed, 0) > self.max_blocks_per_seq:
                raise OutOfBlocks(
                    f"sequence needs {len(table) + needed} blocks, the device table row holds "
                    f"{self.max_blocks_per_seq}")
            if seq_id not in self._rows:
                if not self._free_rows:
                    raise OutOfBlocks(f"all {self.max_seqs} device table rows are in use")
                self._rows[seq_id] = self._free_rows.pop()
                self._synced[seq_id] = 0
        for _ in range(needed):
            table.append(self._free.pop())
        self._tables[seq_id] = table

    def block_table(self, seq_id: int) -> list[int]:
        return self._tables[seq_id]

    def locate(self, seq_id: int, position: int) -> tuple[int, int]:
        block_index, offset = divmod(position, self._block_size)
        return self._tables[seq_id][block_index], offset

    def free(self, seq_id: int) -> None:
        self._free.extend(self._tables.pop(seq_id))
        row = self._rows.pop(seq_id, None)
        if row is not None:
            self._synced.pop(seq_id, None)
            self._free_rows.append(row)

    # ---------------------------------------------------------------- device mirror

    def row(self, seq_id: int) -> int:
        """Row of the sequence in ``device_tables``."""
        return self._rows[seq_id]

    def sync_device(self) -> int:
        """Copy table entries added since the last sync to the device; returns how many.

        Stale entries of freed rows are left in place: kernels only read
        ceil(len / block_size) entries of a row, all of which a live sequence owns.
        """
        if self.device_tables is None:
            return 0
        index, value = [], []
        width = self.max_blocks_per_seq
        for seq_id, row in self._rows.items():
            table = self._tables[seq_id]
            done = self._synced[seq_id]
            if done < len(table):
                base = row * width
                index.extend(range(base + done, base + len(table)))
                value.extend(table[done:])
                self._synced[seq_id] = len(table)
        if index:
            packed = torch.tensor([index, value], dtype=torch.int64).pin_memory()
            packed = packed.to(self._device, non_blocking=True)
            flat = self.device_tables.view(-1)
            flat.index_copy_(0, packed[0], packed[1].to(torch.int32))
        return len(index)
