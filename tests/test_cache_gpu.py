"""Device block tables, step metadata and the K/V slot write: bit-exact against the
reference allocator's locate() (through the oracle) and torch's indexed stores."""

import numpy as np
import pytest
import torch

import oracle
from batchstream_inference_engine_b200 import ops
from batchstream_inference_engine_b200.block_allocator import BlockAllocator

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def grown_allocator(seed=0, num_blocks=300, block_size=16, seqs=24):
    rng = np.random.default_rng(seed)
    alloc = BlockAllocator(num_blocks, block_size, max_seqs=32, max_blocks_per_seq=40, device=DEV)
    lengths = {}
    for s in range(seqs):
        n = int(rng.integers(1, 200))
        alloc.allocate(s, n)
        lengths[s] = n
        if s % 5 == 4:  # free one to fragment the free list
            victim = s - 2
            alloc.free(victim)
            lengths.pop(victim)
    for s in list(lengths)[:6]:  # grow some
        lengths[s] += int(rng.integers(1, 60))
        alloc.allocate(s, lengths[s])
    alloc.sync_device()
    return alloc, lengths


def test_device_tables_mirror_the_allocator_bit_exactly():
    alloc, lengths = grown_allocator()
    dev = alloc.device_tables.cpu()
    for s in lengths:
        table = alloc.block_table(s)
        assert dev[alloc.row(s), : len(table)].tolist() == table
    # Incremental sync only ships new entries.
    s = next(iter(lengths))
    lengths[s] += 16
    alloc.allocate(s, lengths[s])
    assert alloc.sync_device() == len(alloc.block_table(s)) - (len(alloc.block_table(s)) - 1)
    assert alloc.device_tables[alloc.row(s), : len(alloc.block_table(s))].tolist() == \
        alloc.block_table(s)


def test_step_metadata_matches_locate():
    alloc, lengths = grown_allocator(seed=1)
    seqs = list(lengths)
    rng = np.random.default_rng(2)
    start, n_new = [], []
    for s in seqs:
        n = int(rng.integers(0, 5)) if rng.random() < 0.7 else 1
        n = min(n, lengths[s])
        start.append(lengths[s] - n)
        n_new.append(n)
    T = sum(n_new)
    rows = torch.tensor([alloc.row(s) for s in seqs], dtype=torch.int32, device=DEV)
    cu, pos, slots, ctx = ops.step_metadata(
        alloc.device_tables, torch.tensor(start, dtype=torch.int32, device=DEV),
        torch.tensor(n_new, dtype=torch.int32, device=DEV), T, 16, alloc.num_blocks,
        seq_rows=rows)
    want_pos, want_slots = oracle.slot_mapping([alloc.block_table(s) for s in seqs], start, n_new,
                                               16)
    assert pos.cpu().tolist() == want_pos.tolist()
    assert slots.cpu().tolist() == want_slots.tolist()
    assert cu.cpu().tolist() == np.concatenate([[0], np.cumsum(n_new)]).tolist()
    assert ctx.cpu().tolist() == [a + b for a, b in zip(start, n_new)]
    # Each slot is what the reference's locate() returns for that position.
    t = 0
    for s, st, n in zip(seqs, start, n_new):
        for i in range(n):
            blk, off = alloc.locate(s, st + i)
            assert slots[t].item() == blk * 16 + off
            t += 1
    assert ops.take_status() == 0


def test_step_metadata_padding_rows_and_tokens():
    # A fixed-size step: real rows interleaved with padding rows (start < 0),
    # and more tokens than the rows hold.  Real rows are unaffected; padding
    # tokens get position 0 and slot -1, padding rows context length 0.
    alloc, lengths = grown_allocator(seed=3)
    seqs = list(lengths)[:5]
    start = [lengths[s] - 1 for s in seqs]
    n_new = [1] * len(seqs)
    rows = [alloc.row(s) for s in seqs]
    # Insert padding: one decode-style padding row (1 token) and one empty row.
    start_p = start[:2] + [-1] + start[2:] + [-1]
    n_p = n_new[:2] + [1] + n_new[2:] + [0]
    rows_p = rows[:2] + [0] + rows[2:] + [0]
    T = sum(n_p) + 7
    cu, pos, slots, ctx = ops.step_metadata(
        alloc.device_tables, torch.tensor(start_p, dtype=torch.int32, device=DEV),
        torch.tensor(n_p, dtype=torch.int32, device=DEV), T, 16, alloc.num_blocks,
        seq_rows=torch.tensor(rows_p, dtype=torch.int32, device=DEV))
    assert ops.take_status() == 0
    want_pos, want_slots = oracle.slot_mapping([alloc.block_table(s) for s in seqs], start, n_new,
                                               16)
    pos, slots = pos.cpu().tolist(), slots.cpu().tolist()
    real = [0, 1, 3, 4, 5]  # token index of each real row
    assert [pos[t] for t in real] == want_pos.tolist()
    assert [slots[t] for t in real] == want_slots.tolist()
    assert pos[2] == 0 and slots[2] == -1
    assert pos[6:] == [0] * 7 and slots[6:] == [-1] * 7
    assert ctx.cpu().tolist() == [s + 1 for s in start[:2]] + [0] + [s + 1 for s in start[2:]] + [0]
    assert cu.cpu().tolist() == [0, 1, 2, 3, 4, 5, 6, 6]


@pytest.mark.parametrize("in_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("pool_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 4])
def test_decode_append_equals_metadata_plus_slot_write(in_dtype, pool_dtype, head_dim):
    """One fused launch gives the slots, lengths and pool contents of the
    two-launch path, and the slots are locate()'s."""
    alloc, lengths = grown_allocator(seed=3)
    seqs = list(lengths)
    start = [lengths[s] - 1 for s in seqs]  # every row decodes its last position
    B, Hkv = len(seqs), 2
    rows = torch.tensor([alloc.row(s) for s in seqs], dtype=torch.int32, device=DEV)
    start_d = torch.tensor(start, dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(7)
    k = torch.randn((B, Hkv, head_dim), generator=g, device=DEV).to(in_dtype)
    v = torch.randn((B, Hkv, head_dim), generator=g, device=DEV).to(in_dtype)
    shape = (Hkv, alloc.num_blocks, 16, head_dim)
    pools = [torch.randn(shape, generator=g, device=DEV).to(pool_dtype) for _ in range(2)]
    ref_k, ref_v = pools[0].clone(), pools[1].clone()
    _, _, ref_slots, ref_ctx = ops.step_metadata(alloc.device_tables, start_d,
                                                 torch.ones(B, dtype=torch.int32, device=DEV), B,
                                                 16, alloc.num_blocks, seq_rows=rows)
    ops.reshape_and_cache(k, v, ref_k, ref_v, ref_slots)
    ctx, slots = ops.decode_append(k, v, pools[0], pools[1], alloc.device_tables, start_d,
                                   seq_rows=rows)
    assert ops.take_status() == 0
    assert torch.equal(slots, ref_slots) and torch.equal(ctx, ref_ctx)
    assert torch.equal(pools[0], ref_k) and torch.equal(pools[1], ref_v)
    _, want = oracle.slot_mapping([alloc.block_table(s) for s in seqs], start, [1] * B, 16)
    assert slots.cpu().tolist() == want.tolist()


def test_decode_append_negative_start_is_padding():
    alloc, lengths = grown_allocator(seed=5)
    seqs = list(lengths)[:4]
    start = [lengths[s] - 1 for s in seqs]
    start[1] = -1
    rows = torch.tensor([alloc.row(s) for s in seqs], dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(3)
    k = torch.randn((4, 2, 64), generator=g, device=DEV).bfloat16()
    pool_k = torch.zeros((2, alloc.num_blocks, 16, 64), dtype=torch.bfloat16, device=DEV)
    pool_v = torch.zeros_like(pool_k)
    ctx, slots = ops.decode_append(k, k, pool_k, pool_v, alloc.device_tables,
                                   torch.tensor(start, dtype=torch.int32, device=DEV),
                                   seq_rows=rows)
    assert ops.take_status() == 0
    assert ctx.cpu().tolist()[1] == 0 and slots.cpu().tolist()[1] == -1
    # Exactly the three real rows were written.
    assert int((pool_k.abs().sum(dim=-1) > 0).sum()) == 3 * 2


def test_decode_append_bad_table_entry_sets_status():
    alloc, lengths = grown_allocator(seed=4)
    seqs = list(lengths)[:5]
    start = [lengths[s] - 1 for s in seqs]
    tables = alloc.device_tables.clone()
    tables[alloc.row(seqs[2]), start[2] // 16] = alloc.num_blocks + 5
    rows = torch.tensor([alloc.row(s) for s in seqs], dtype=torch.int32, device=DEV)
    k = torch.zeros((5, 2, 64), dtype=torch.bfloat16, device=DEV)
    pool = torch.zeros((2, alloc.num_blocks, 16, 64), dtype=torch.bfloat16, device=DEV)
    _, slots = ops.decode_append(k, k, pool, pool.clone(), tables,
                                 torch.tensor(start, dtype=torch.int32, device=DEV), seq_rows=rows)
    with pytest.raises(RuntimeError, match="block table"):
        ops.take_status()
    assert slots[2].item() == -1 and slots[0].item() >= 0


@pytest.mark.parametrize("in_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("pool_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128, 4])
def test_slot_write_is_an_exact_indexed_store(in_dtype, pool_dtype, head_dim):
    g = torch.Generator(device=DEV).manual_seed(0)
    Hkv, NB, bs, T = 2, 50, 16, 37
    k_pool = torch.randn((Hkv, NB, bs, head_dim), generator=g, device=DEV).to(pool_dtype)
    v_pool = torch.randn((Hkv, NB, bs, head_dim), generator=g, device=DEV).to(pool_dtype)
    # Fused projection output [T, (H + 2 Hkv) * D]: k and v are strided views.
    H = 14
    qkv = torch.randn((T, (H + 2 * Hkv) * head_dim), generator=g, device=DEV).to(in_dtype)
    k = qkv[:, H * head_dim:(H + Hkv) * head_dim].view(T, Hkv, head_dim)
    v = qkv[:, (H + Hkv) * head_dim:].view(T, Hkv, head_dim)
    slots = torch.randperm(NB * bs, generator=torch.Generator().manual_seed(1))[:T].to(torch.int32)
    slots[5] = -1  # padding token: skipped
    want_k, want_v = k_pool.clone(), v_pool.clone()
    for t in range(T):
        s = slots[t].item()
        if s < 0:
            continue
        want_k[:, s // bs, s % bs] = k[t]  # torch's own cast: round to nearest even
        want_v[:, s // bs, s % bs] = v[t]
    ops.reshape_and_cache(k, v, k_pool, v_pool, slots.to(DEV))
    assert torch.equal(k_pool, want_k)
    assert torch.equal(v_pool, want_v)
    assert ops.take_status() == 0


def test_slot_beyond_pool_sets_status():
    Hkv, NB, bs, D = 2, 4, 16, 64
    k_pool = torch.zeros((Hkv, NB, bs, D), dtype=torch.bfloat16, device=DEV)
    v_pool = torch.zeros_like(k_pool)
    k = torch.ones((2, Hkv, D), dtype=torch.bfloat16, device=DEV)
    slots = torch.tensor([3, NB * bs + 9], dtype=torch.int32, device=DEV)
    ops.reshape_and_cache(k, k, k_pool, v_pool, slots)
    with pytest.raises(RuntimeError, match="slot"):
        ops.take_status()
    assert k_pool[:, 0, 3].eq(1).all() and k_pool.sum().item() == Hkv * D


def test_metadata_then_slot_write_then_decode_round_trip():
    """append (slot write) followed by attend reads back exactly what was written."""
    alloc, lengths = grown_allocator(seed=3)
    seqs = list(lengths)[:8]
    Hkv, D, H = 2, 64, 14
    g = torch.Generator(device=DEV).manual_seed(4)
    k_pool = torch.zeros((Hkv, alloc.num_blocks, 16, D), dtype=torch.bfloat16, device=DEV)
    v_pool = torch.zeros_like(k_pool)
    total = [lengths[s] for s in seqs]
    rows = torch.tensor([alloc.row(s) for s in seqs], dtype=torch.int32, device=DEV)
    start = torch.zeros(len(seqs), dtype=torch.int32, device=DEV)
    n_new = torch.tensor(total, dtype=torch.int32, device=DEV)
    T = sum(total)
    _, _, slots, ctx = ops.step_metadata(alloc.device_tables, start, n_new, T, 16,
                                         alloc.num_blocks, seq_rows=rows)
    k = torch.randn((T, Hkv, D), generator=g, device=DEV).bfloat16()
    v = torch.randn((T, Hkv, D), generator=g, device=DEV).bfloat16()
    ops.reshape_and_cache(k, v, k_pool, v_pool, slots)
    q = torch.randn((len(seqs), H, D), generator=g, device=DEV).bfloat16()
    out = ops.paged_attention_batched(q, k_pool, v_pool, alloc.device_tables, ctx, 0.125,
                                      seq_rows=rows)
    assert ops.take_status() == 0
    offsets = np.concatenate([[0], np.cumsum(total)])
    for i in range(len(seqs)):
        kk = k[offsets[i]:offsets[i + 1]].float().cpu()  # [L, Hkv, D]
        vv = v[offsets[i]:offsets[i + 1]].float().cpu()
        qq = q[i].float().cpu()
        ref = torch.empty(H, D)
        for h in range(H):
            s = (kk[:, h // 7] @ qq[h]) * 0.125
            ref[h] = torch.softmax(s, 0) @ vv[:, h // 7]
        err = (out[i].float().cpu() - ref).abs().max() / ref.abs().max()
        assert err.item() <= 2e-2
