"""The product allocator keeps the reference BlockAllocator's semantics
(src/server/block_allocator.py; tests modelled on tests/test_block_allocator.py)."""

import random
from pathlib import Path

import numpy as np
import pytest

import oracle
from batchstream_inference_engine_b200.block_allocator import BlockAllocator, OutOfBlocks


def test_allocate_covers_requested_tokens_in_whole_blocks():
    a = BlockAllocator(num_blocks=4, block_size=16)
    a.allocate(seq_id=0, total_tokens=17)
    assert len(a.block_table(0)) == 2 and a.free_blocks == 2


def test_grows_only_at_block_boundaries():
    a = BlockAllocator(num_blocks=4, block_size=16)
    a.allocate(0, 1)
    first = a.block_table(0)[0]
    a.allocate(0, 16)
    assert a.block_table(0) == [first]
    a.allocate(0, 17)
    assert a.block_table(0)[0] == first and len(a.block_table(0)) == 2


def test_locate_maps_position_to_block_and_offset():
    a = BlockAllocator(num_blocks=4, block_size=16)
    a.allocate(0, 40)
    t = a.block_table(0)
    assert a.locate(0, 0) == (t[0], 0)
    assert a.locate(0, 15) == (t[0], 15)
    assert a.locate(0, 16) == (t[1], 0)
    assert a.locate(0, 39) == (t[2], 7)


def test_out_of_blocks_is_a_runtime_error_and_changes_nothing():
    a = BlockAllocator(num_blocks=3, block_size=16)
    a.allocate(0, 16)
    table = list(a.block_table(0))
    with pytest.raises(OutOfBlocks):
        a.allocate(0, 64)
    assert issubclass(OutOfBlocks, RuntimeError)
    assert a.block_table(0) == table and a.free_blocks == 2


def test_free_unknown_and_freed_tables_raise_key_error():
    a = BlockAllocator(num_blocks=4, block_size=16)
    with pytest.raises(KeyError):
        a.free(7)
    a.allocate(0, 1)
    a.free(0)
    with pytest.raises(KeyError):
        a.block_table(0)


def test_replays_reference_trace_bit_exactly():
    gold = np.load(Path(__file__).resolve().parent / "golden" / "allocator.npz")
    a = BlockAllocator(num_blocks=64, block_size=8)
    for kind, seq, want, ok in gold["ops"].tolist():
        if kind == 1:
            a.free(seq)
            continue
        try:
            a.allocate(seq, want)
            assert ok == 1
        except OutOfBlocks:
            assert ok == 0
    offsets = gold["offsets"].tolist()
    for i, seq in enumerate(gold["seqs"].tolist()):
        assert a.block_table(seq) == gold["tables"][offsets[i]:offsets[i + 1]].tolist()
    assert a._free == gold["free"].tolist()


def test_matches_oracle_under_a_long_fuzz():
    rng = random.Random(0)
    mine, ref = BlockAllocator(64, 8), oracle.Allocator(64, 8)
    tokens, next_id = {}, 0
    for _ in range(20_000):
        if tokens and (rng.random() < 0.4 or mine.free_blocks == 0):
            s = rng.choice(list(tokens))
            del tokens[s]
            mine.free(s)
            ref.free(s)
        else:
            if tokens and rng.random() < 0.5:
                s = rng.choice(list(tokens))
                want = tokens[s] + rng.randint(1, 20)
            else:
                s, want = next_id, rng.randint(1, 40)
            outcomes = []
            for alloc, exc in ((mine, OutOfBlocks), (ref, oracle.OutOfBlocks)):
                try:
                    alloc.allocate(s, want)
                    outcomes.append(True)
                except exc:
                    outcomes.append(False)
            assert outcomes[0] == outcomes[1]
            if outcomes[0]:
                tokens[s] = want
                if s == next_id:
                    next_id += 1
        used = [b for s in tokens for b in mine.block_table(s)]
        assert len(used) == len(set(used)) and len(used) + mine.free_blocks == 64
    assert mine._free == ref.free_list
    assert all(mine.block_table(s) == ref.tables[s] for s in tokens)


def test_device_rows_are_recycled_and_bounded_on_host():
    # Host bookkeeping of the device mirror, without a device: rows come and go.
    a = BlockAllocator(num_blocks=16, block_size=4)
    a.allocate(0, 5)
    a.free(0)
    assert a.free_blocks == 16
