"""Pins the oracle (the CPU restatement) to the reference's own outputs.

The golden fixtures were produced by the reference's compiled C++ op, its Python
op, its attend() and its BlockAllocator (tests/golden/make_golden.py).  These
tests run on the CPU only.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tests.golden import inputs

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / name)


def bf16_float(bits: np.ndarray) -> np.ndarray:
    return inputs.from_bits(bits).float().numpy()


@pytest.mark.parametrize("length", inputs.SCATTERED_LENGTHS)
def test_oracle_bf16_decode_matches_reference_cpp_op(length):
    gold = load("decode_scattered.npz")
    q, k, v, table = inputs.scattered_bf16(length, seed=length)
    assert inputs.digest(q, k, v) == str(gold[f"digest_{length}"])
    got = oracle.decode(inputs.bf16_bits(q), inputs.bf16_bits(k), inputs.bf16_bits(v), table,
                        length, 4, 2, 8 ** -0.5)
    # Same rounding points and loop order as the reference op: bit-identical.
    np.testing.assert_array_equal(got, gold[f"cpp_{length}"])
    # And within the reference's own C++-vs-Python tolerance of its Python op.
    assert np.abs(bf16_float(got) - bf16_float(gold[f"py_{length}"])).max() <= 0.01


@pytest.mark.parametrize("length", inputs.F32_LENGTHS)
def test_oracle_f32_decode_matches_reference_python_op(length):
    gold = load("decode_f32.npz")
    q, pk, pv, table, _, _ = inputs.scattered_f32(length)
    assert inputs.digest(q, pk, pv) == str(gold[f"digest_{length}"])
    got = oracle.decode(q.numpy(), pk.numpy(), pv.numpy(), table, length, 4, 2, 0.5)
    assert not np.isnan(got).any()
    np.testing.assert_allclose(got, gold[f"paged_{length}"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(got, gold[f"contiguous_{length}"], rtol=0, atol=1e-6)


def test_oracle_op_level_batch_matches_reference():
    gold = load("decode_op_level.npz")
    lengths, tables, q, k, v = inputs.op_level_batch()
    assert inputs.digest(q, k, v) == str(gold["digest"])
    assert lengths == gold["lengths"].tolist()
    kb, vb, qb = (inputs.bf16_bits(t.bfloat16()) for t in (k, v, q))
    for i, (length, table) in enumerate(zip(lengths, tables)):
        assert table == gold[f"table_{i}"].tolist()
        f32 = oracle.decode(q[i].numpy(), k.numpy(), v.numpy(), table, length, 16, 7, 0.125)
        np.testing.assert_allclose(f32, gold[f"f32_{i}"], rtol=0, atol=1e-5)
        b16 = oracle.decode(qb[i], kb, vb, table, length, 16, 7, 0.125)
        np.testing.assert_array_equal(b16, gold[f"cpp_bf16_{i}"])


@pytest.mark.parametrize("case", inputs.PREFILL_CASES)
def test_oracle_prefill_matches_reference_attend(case):
    n, past, heads, kv_heads = case
    gold = load("prefill.npz")
    q, k, v, table = inputs.prefill_case(n, past, heads, kv_heads)
    assert inputs.digest(q, k, v) == str(gold[f"digest_{n}_{past}"])
    groups = heads // kv_heads
    f32 = oracle.prefill(q.numpy(), k.numpy(), v.numpy(), table, past, 16, groups, 0.125)
    assert not np.isnan(f32).any()
    np.testing.assert_allclose(f32, gold[f"f32_{n}_{past}"], rtol=0, atol=2e-5)
    b16 = oracle.prefill(*(inputs.bf16_bits(t.bfloat16()) for t in (q, k, v)), table, past, 16,
                         groups, 0.125)
    ref = bf16_float(gold[f"bf16_{n}_{past}"])
    # torch's bf16 matmul blocks its fp32 sums differently from the oracle's
    # position-order loop, so a few outputs land one bf16 step apart.
    diff = np.abs(bf16_float(b16) - ref)
    assert diff.max() <= 0.02
    assert (diff == 0).mean() > 0.9


def test_oracle_allocator_replays_reference_trace():
    gold = load("allocator.npz")
    alloc = oracle.Allocator(num_blocks=64, block_size=8)
    for kind, seq, want, ok in gold["ops"].tolist():
        if kind == 1:
            alloc.free(seq)
            continue
        try:
            alloc.allocate(seq, want)
            assert ok == 1
        except oracle.OutOfBlocks:
            assert ok == 0
    offsets = gold["offsets"].tolist()
    for i, seq in enumerate(gold["seqs"].tolist()):
        assert alloc.tables[seq] == gold["tables"][offsets[i]:offsets[i + 1]].tolist()
    assert alloc.free_list == gold["free"].tolist()


def test_oracle_slot_mapping_matches_reference_locate():
    gold = load("allocator.npz")
    offsets = gold["offsets"].tolist()
    tables = [gold["tables"][offsets[i]:offsets[i + 1]].tolist()
              for i in range(len(gold["seqs"]))]
    counts = gold["seq_tokens"].tolist()
    _, slots = oracle.slot_mapping(tables, [0] * len(tables), counts, 8)
    np.testing.assert_array_equal(slots, gold["slots"])


def test_oracle_slot_mapping_of_partial_chunks():
    tables = [[5, 2, 7], [0], [3, 1]]
    start = [17, 0, 16]
    n_new = [3, 2, 1]
    pos, slots = oracle.slot_mapping(tables, start, n_new, 16)
    assert pos.tolist() == [17, 18, 19, 0, 1, 16]
    assert slots.tolist() == [2 * 16 + 1, 2 * 16 + 2, 2 * 16 + 3, 0, 1, 1 * 16 + 0]


def test_oracle_never_reads_past_length():
    q, k, v, table = inputs.scattered_bf16(5, seed=0)
    got = oracle.decode(inputs.bf16_bits(q), inputs.bf16_bits(k), inputs.bf16_bits(v), table, 5,
                        4, 2, 0.5)
    assert not np.isnan(bf16_float(got)).any()


def test_planted_mistake_in_oracle_input_is_detected():
    # A one-position shift of the table must change the answer: the fixtures
    # are sensitive to the indexing the oracle restates.
    gold = load("decode_scattered.npz")
    q, k, v, table = inputs.scattered_bf16(17, seed=17)
    wrong = table[1:] + table[:1]
    got = oracle.decode(inputs.bf16_bits(q), inputs.bf16_bits(k), inputs.bf16_bits(v), wrong, 17,
                        4, 2, 8 ** -0.5)
    assert not np.array_equal(got, gold["cpp_17"])


def test_torch_generator_recipes_are_stable():
    # Regeneration on another machine must give the inputs the fixtures hold.
    lengths, _, q, k, v = inputs.op_level_batch()
    assert lengths == load("decode_op_level.npz")["lengths"].tolist()
    assert q.dtype == torch.float32 and k.shape == (2, 256, 16, 64)


def test_recorded_reference_pool_calls_match_the_oracle_bit_for_bit():
    """The op calls recorded from the reference's own PagedKVPool (fixture
    reference_callers.npz): the C oracle on the recorded blocks reproduces the
    reference op's recorded outputs exactly, and the rebuilt arguments have the
    caller's forms (the query's view of the step's rotated queries, the pool's
    layer view)."""
    from tests.test_reference_callers_gpu import _calls, _events, _rebuild

    calls = _calls()
    assert len(calls) == 30
    for call in calls:
        query, keys, values, table = _rebuild(call)
        assert list(query.stride()) == call["q_stride"].tolist()
        assert query.storage_offset() == int(call["q_offset"])
        assert keys.storage_offset() == int(call["pool_offset"])
        got = oracle.decode(inputs.bf16_bits(query.contiguous()), inputs.bf16_bits(keys),
                            inputs.bf16_bits(values), table, int(call["length"]),
                            int(call["block_size"]), int(call["groups"]), float(call["scaling"]))
        assert np.array_equal(got, call["out"].reshape(got.shape))
    events = _events()
    assert sum(e[0] == "start" for e in events) == 24
    assert sum(e[0] == "release" for e in events) == 24
