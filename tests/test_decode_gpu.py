"""Decode attention on the GPU against the oracle and the reference's golden outputs.

Tolerances (as stated for this path):
  * fp32 kernels: max |out - ref| <= 1e-4 against the fp32 reference.
  * bf16 kernels: max |out - ref| <= 2e-2 * max |ref| against the fp32 reference
    (or, where the reference's own bf16 op is already further than that from
    fp32, no further than it plus 2**-8: see bf16_bound), and, element by element, |out - cpp| <= 0.01 + 2**-7 * |cpp| against the
    reference's own bf16 C++ op: its CPP_TOLERANCE (0.01,
    tests/test_paged_attention.py:150) plus one bf16 step of the value, because
    the split-K online softmax rounds the not-yet-normalised probabilities to
    bf16 where the reference rounds the normalised weights, which moves
    outputs of magnitude 1-2 by up to two bf16 steps on very short contexts.
"""

import math

import numpy as np
import pytest
import torch

import oracle
from batchstream_inference_engine_b200 import ops
from batchstream_inference_engine_b200.paged_attention_cuda import paged_attention
from tests.golden import inputs
from tests.test_capi import BAD_INPUTS

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_REL = 2e-2
CPP_TOL = 0.01


def cpp_close(out: torch.Tensor, cpp: torch.Tensor) -> bool:
    out, cpp = out.float().cpu(), cpp.float().cpu()
    return bool(((out - cpp).abs() <= CPP_TOL + 2.0 ** -7 * cpp.abs()).all())
DEV = "cuda:0"


def bf16_rel_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    ref = ref.float().cpu()
    return ((out.float().cpu() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


def golden(name):
    from pathlib import Path

    return np.load(Path(__file__).resolve().parent / "golden" / name)


@pytest.mark.parametrize("length", inputs.SCATTERED_LENGTHS)
def test_bf16_op_matches_reference_cpp_on_scattered_blocks(length):
    gold = golden("decode_scattered.npz")
    q, k, v, table = inputs.scattered_bf16(length, seed=length)
    out = paged_attention(q.to(DEV), k.to(DEV), v.to(DEV), table, length, 4, 2, 8 ** -0.5)
    assert out.dtype == torch.bfloat16 and out.shape == (4, 8) and out.is_cuda
    cpp = inputs.from_bits(gold[f"cpp_{length}"]).float()
    assert cpp_close(out, cpp)
    ref = oracle.decode(q.float().numpy(), k.float().numpy(), v.float().numpy(), table, length, 4,
                        2, 8 ** -0.5)
    assert bf16_rel_err(out, torch.from_numpy(ref)) <= BF16_REL


@pytest.mark.parametrize("length", inputs.F32_LENGTHS)
def test_f32_op_matches_reference_python_op(length):
    gold = golden("decode_f32.npz")
    q, pk, pv, table, _, _ = inputs.scattered_f32(length)
    out = paged_attention(q.to(DEV), pk.to(DEV), pv.to(DEV), table, length, 4, 2, 0.5)
    assert out.dtype == torch.float32
    assert np.abs(out.cpu().numpy() - gold[f"paged_{length}"]).max() <= F32_TOL


def test_op_never_reads_past_length():
    q, k, v, table = inputs.scattered_bf16(5)
    out = paged_attention(q.to(DEV), k.to(DEV), v.to(DEV), table, 5, 4, 2, 0.5)
    assert not out.isnan().any()


def test_op_accepts_a_non_contiguous_query():
    q, k, v, table = inputs.scattered_bf16(5)
    strided = torch.zeros(4, 3, 8, dtype=torch.bfloat16, device=DEV)
    strided[:, 1] = q.to(DEV)
    a = paged_attention(strided[:, 1], k.to(DEV), v.to(DEV), table, 5, 4, 2, 0.5)
    b = paged_attention(q.to(DEV), k.to(DEV), v.to(DEV), table, 5, 4, 2, 0.5)
    assert torch.equal(a, b)


@pytest.mark.parametrize("change", BAD_INPUTS)
def test_op_rejects_bad_cuda_input_with_an_error_not_a_crash(change):
    q, k, v, table = inputs.scattered_bf16(5)
    args = dict(query=q, keys=k, values=v, table=table, length=5, block_size=4, groups=2)
    args.update(change)
    moved = {n: (t.to(DEV) if isinstance(t, torch.Tensor) else t) for n, t in args.items()}
    with pytest.raises(RuntimeError):
        paged_attention(moved["query"], moved["keys"], moved["values"], moved["table"],
                        moved["length"], moved["block_size"], moved["groups"], 0.5)
    torch.cuda.synchronize()


def test_op_level_batch_per_sequence_and_batched():
    gold = golden("decode_op_level.npz")
    lengths, tables, q, k, v = inputs.op_level_batch()
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    qb, kb, vb = qd.bfloat16(), kd.bfloat16(), vd.bfloat16()
    for i, (length, table) in enumerate(zip(lengths, tables)):
        f32 = paged_attention(qd[i], kd, vd, table, length, 16, 7, 0.125)
        assert np.abs(f32.cpu().numpy() - gold[f"f32_{i}"]).max() <= F32_TOL
        b16 = paged_attention(qb[i], kb, vb, table, length, 16, 7, 0.125)
        cpp = inputs.from_bits(gold[f"cpp_bf16_{i}"]).float()
        assert cpp_close(b16, cpp)
        assert bf16_rel_err(b16, torch.from_numpy(gold[f"f32_{i}"])) <= BF16_REL
    width = max(len(t) for t in tables)
    bt = torch.full((8, width), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, : len(t)] = torch.tensor(t)
    bt, lens = bt.to(DEV), torch.tensor(lengths, dtype=torch.int32, device=DEV)
    for dtype, (qq, kk, vv) in ((torch.float32, (qd, kd, vd)), (torch.bfloat16, (qb, kb, vb))):
        out = ops.paged_attention_batched(qq, kk, vv, bt, lens, 0.125)
        for i in range(8):
            ref = gold[f"f32_{i}"]
            if dtype == torch.float32:
                assert np.abs(out[i].cpu().numpy() - ref).max() <= F32_TOL
            else:
                cpp = inputs.from_bits(gold[f"cpp_bf16_{i}"]).float()
                assert cpp_close(out[i], cpp)
    assert ops.take_status() == 0


def ragged_batch(num_seqs, heads, kv_heads, head_dim, dtype, median=1024.0, sigma=1.0,
                 lo=16, hi=32768, seed=0, spare_blocks=64):
    """Lognormal ragged batch over a shuffled pool (the large-sweep recipe)."""
    rng = np.random.default_rng(seed)
    lens = np.clip(np.rint(rng.lognormal(math.log(median), sigma, num_seqs)), lo, hi).astype(int)
    need = [-(-int(n) // 16) for n in lens]
    nb = sum(need) + spare_blocks
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed))
    width = max(need)
    bt = torch.full((num_seqs, width), -1, dtype=torch.int32)
    cur = 0
    tables = []
    for i, m in enumerate(need):
        tables.append(perm[cur: cur + m].tolist())
        bt[i, :m] = perm[cur: cur + m].to(torch.int32)
        cur += m
    g = torch.Generator(device=DEV).manual_seed(seed)
    k = torch.randn((kv_heads, nb, 16, head_dim), generator=g, device=DEV).to(dtype)
    v = torch.randn((kv_heads, nb, 16, head_dim), generator=g, device=DEV).to(dtype)
    q = torch.randn((num_seqs, heads, head_dim), generator=g, device=DEV).to(dtype)
    return lens.tolist(), tables, bt.to(DEV), q, k, v


def check_against_oracle(out, lens, tables, q, k, v, groups, scale, sample):
    kc, vc, qc = k.float().cpu().numpy(), v.float().cpu().numpy(), q.float().cpu().numpy()
    kbits = inputs.bf16_bits(k.cpu()) if k.dtype == torch.bfloat16 else None
    vbits = inputs.bf16_bits(v.cpu()) if k.dtype == torch.bfloat16 else None
    qbits = inputs.bf16_bits(q.cpu()) if k.dtype == torch.bfloat16 else None
    for i in sample:
        ref32 = oracle.decode(qc[i], kc, vc, tables[i], lens[i], 16, groups, scale)
        if k.dtype == torch.float32:
            assert np.abs(out[i].cpu().numpy() - ref32).max() <= F32_TOL, i
        else:
            cpp_like = inputs.from_bits(
                oracle.decode(qbits[i], kbits, vbits, tables[i], lens[i], 16, groups, scale))
            assert cpp_close(out[i], cpp_like), i
            ref32 = torch.from_numpy(ref32)
            assert bf16_rel_err(out[i], ref32) <= bf16_bound(cpp_like, ref32), i


def bf16_bound(cpp_like: torch.Tensor, ref32: torch.Tensor) -> float:
    """2e-2 of max |ref| against fp32 -- or, where the reference's own bf16 op
    (its bf16 score and weight roundings) is already further from fp32 than that
    (head_dim 128, a few hundred tokens: up to 2.4e-2 seen), no further than the
    reference op plus one bf16 step (2**-8)."""
    return max(BF16_REL, bf16_rel_err(cpp_like, ref32) + 2.0 ** -8)


@pytest.mark.parametrize("heads,kv_heads,head_dim", [(14, 2, 64), (28, 4, 128)])
def test_large_ragged_batch_against_oracle(heads, kv_heads, head_dim):
    lens, tables, bt, q, k, v = ragged_batch(256, heads, kv_heads, head_dim, torch.bfloat16)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = ops.paged_attention_batched(q, k, v, bt, lens_d, head_dim ** -0.5)
    assert ops.take_status() == 0
    assert not out.isnan().any()
    # Every one of the 256 sequences against the oracle.
    check_against_oracle(out, lens, tables, q, k, v, heads // kv_heads, head_dim ** -0.5,
                         range(256))
    # Same inputs, same bits: counters and records are left clean between calls.
    again = ops.paged_attention_batched(q, k, v, bt, lens_d, head_dim ** -0.5)
    assert torch.equal(out, again)
    # Exact linearity in V: scaling V by 2 scales every output by exactly 2.
    twice = ops.paged_attention_batched(q, k, v * 2, bt, lens_d, head_dim ** -0.5)
    assert torch.equal(twice, out * 2)


@pytest.mark.parametrize("units_hint", [1, 7, 64, 1000, 10 ** 6])
def test_grid_size_moves_split_points_but_not_the_answer(units_hint):
    lens, tables, bt, q, k, v = ragged_batch(40, 14, 2, 64, torch.bfloat16, median=300, seed=3)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    base = ops.paged_attention_batched(q, k, v, bt, lens_d, 0.125)
    out = ops.paged_attention_batched(q, k, v, bt, lens_d, 0.125, units_hint=units_hint)
    assert (out.float() - base.float()).abs().max().item() <= 1e-2
    check_against_oracle(out, lens, tables, q, k, v, 7, 0.125, range(0, 40, 5))


@pytest.mark.parametrize("groups", [1, 2, 4, 7, 8, 9, 16])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_tensor_core_path_over_group_sizes(groups, head_dim):
    kv_heads = 2
    lens, tables, bt, q, k, v = ragged_batch(12, groups * kv_heads, kv_heads, head_dim,
                                             torch.bfloat16, median=200, seed=groups)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = ops.paged_attention_batched(q, k, v, bt, lens_d, head_dim ** -0.5)
    check_against_oracle(out, lens, tables, q, k, v, groups, head_dim ** -0.5, range(12))


@pytest.mark.parametrize("groups", [1, 7, 16])
@pytest.mark.parametrize("head_dim", [32, 64, 96])
def test_simt_path_fp32(groups, head_dim):
    kv_heads = 2
    lens, tables, bt, q, k, v = ragged_batch(10, groups * kv_heads, kv_heads, head_dim,
                                             torch.float32, median=150, seed=groups + head_dim)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = ops.paged_attention_batched(q, k, v, bt, lens_d, head_dim ** -0.5)
    check_against_oracle(out, lens, tables, q, k, v, groups, head_dim ** -0.5, range(10))


def test_short_and_block_boundary_lengths():
    lens = [1, 2, 15, 16, 17, 31, 32, 33, 48, 63, 64, 65]
    need = [-(-n // 16) for n in lens]
    nb = sum(need) + 3
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(5))
    bt = torch.full((len(lens), max(need)), -1, dtype=torch.int32)
    tables, cur = [], 0
    for i, m in enumerate(need):
        tables.append(perm[cur: cur + m].tolist())
        bt[i, :m] = perm[cur: cur + m].to(torch.int32)
        cur += m
    g = torch.Generator(device=DEV).manual_seed(9)
    k = torch.full((2, nb, 16, 64), float("nan"), device=DEV)
    v = torch.full((2, nb, 16, 64), float("nan"), device=DEV)
    for i, n in enumerate(lens):  # only positions < len hold numbers
        for pos in range(n):
            blk = tables[i][pos // 16]
            k[:, blk, pos % 16] = torch.randn((2, 64), generator=g, device=DEV)
            v[:, blk, pos % 16] = torch.randn((2, 64), generator=g, device=DEV)
    q = torch.randn((len(lens), 14, 64), generator=g, device=DEV)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    for dtype in (torch.float32, torch.bfloat16):
        qq, kk, vv = q.to(dtype), k.to(dtype), v.to(dtype)
        out = ops.paged_attention_batched(qq, kk, vv, bt.to(DEV), lens_d, 0.125)
        assert not out.isnan().any()
        check_against_oracle(out, lens, tables, qq, kk, vv, 7, 0.125, range(len(lens)))


@pytest.mark.parametrize("head_dim", [64, 128])
def test_sequences_sharing_a_table_row_with_growing_lengths(head_dim):
    # Lengths 1..300 all read one table row through seq_rows (the tokens of a
    # prefill chunk): every block-count step must read the newly reached block.
    lens = list(range(1, 301))
    need = -(-lens[-1] // 16)
    nb = need + 11
    table = torch.randperm(nb, generator=torch.Generator().manual_seed(2))[:need].tolist()
    bt = torch.full((3, need + 4), -1, dtype=torch.int32)
    bt[1, :need] = torch.tensor(table, dtype=torch.int32)
    g = torch.Generator(device=DEV).manual_seed(12)
    heads, kv_heads = (14, 2) if head_dim == 64 else (28, 4)
    k = torch.randn((kv_heads, nb, 16, head_dim), generator=g, device=DEV).bfloat16()
    v = torch.randn((kv_heads, nb, 16, head_dim), generator=g, device=DEV).bfloat16()
    q = torch.randn((len(lens), heads, head_dim), generator=g, device=DEV).bfloat16()
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    rows = torch.ones(len(lens), dtype=torch.int32, device=DEV)
    scale = head_dim ** -0.5
    for hint in (0, 7, 10 ** 6):
        out = ops.paged_attention_batched(q, k, v, bt.to(DEV), lens_d, scale, seq_rows=rows,
                                          units_hint=hint)
        assert ops.take_status() == 0
        check_against_oracle(out, lens, [table] * len(lens), q, k, v, heads // kv_heads, scale,
                             range(len(lens)))


def test_bad_device_table_sets_status_instead_of_faulting():
    lens, tables, bt, q, k, v = ragged_batch(6, 14, 2, 64, torch.bfloat16, median=100, seed=4)
    bad = bt.clone()
    bad[2, 0] = k.size(1) + 7  # beyond the pool
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    ops.paged_attention_batched(q, k, v, bad, lens_d, 0.125)
    with pytest.raises(RuntimeError, match="block table"):
        ops.take_status()
    # The context is still usable and the status word was cleared.
    out = ops.paged_attention_batched(q, k, v, bt, lens_d, 0.125)
    assert ops.take_status() == 0
    check_against_oracle(out, lens, tables, q, k, v, 7, 0.125, range(6))


def test_bad_device_length_sets_status_instead_of_faulting():
    lens, tables, bt, q, k, v = ragged_batch(6, 14, 2, 64, torch.bfloat16, median=100, seed=6)
    bad = torch.tensor(lens, dtype=torch.int32, device=DEV)
    bad[1] = bt.size(1) * 16 + 1  # longer than the table row
    bad[3] = 0
    ops.paged_attention_batched(q, k, v, bt, bad, 0.125)
    with pytest.raises(RuntimeError, match="context length"):
        ops.take_status()


def test_early_loads_after_an_append_give_the_same_bits():
    # Decode launched right behind the append that writes each sequence's new
    # token, with the first loads of the other blocks issued before it ends.
    lens, tables, bt, q, k, v = ragged_batch(48, 14, 2, 64, torch.bfloat16, median=400, seed=13)
    B = len(lens)
    g = torch.Generator(device=DEV).manual_seed(5)
    k_new = torch.randn((B, 2, 64), generator=g, device=DEV).bfloat16()
    v_new = torch.randn((B, 2, 64), generator=g, device=DEV).bfloat16()
    start = torch.tensor([n - 1 for n in lens], dtype=torch.int32, device=DEV)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    k1, v1 = k.clone(), v.clone()
    ops.decode_append(k_new, v_new, k1, v1, bt, start)
    plain = ops.paged_attention_batched(q, k1, v1, bt, lens_d, 0.125)
    k2, v2 = k.clone(), v.clone()
    for _ in range(3):
        ops.decode_append(k_new, v_new, k2, v2, bt, start)
        early = ops.paged_attention_batched(q, k2, v2, bt, lens_d, 0.125, lens_ready=True,
                                            after_append=True)
        assert torch.equal(early, plain)
    assert ops.take_status() == 0
    with pytest.raises(RuntimeError, match="BS_LENS_READY"):
        ops.paged_attention_batched(q, k2, v2, bt, lens_d, 0.125, after_append=True)


def test_zero_length_rows_are_padding():
    lens, tables, bt, q, k, v = ragged_batch(8, 14, 2, 64, torch.bfloat16, median=150, seed=11)
    padded = torch.tensor(lens, dtype=torch.int32, device=DEV)
    padded[2] = 0
    padded[5] = 0
    out = torch.full_like(q, 7.0)
    ops.paged_attention_batched(q, k, v, bt, padded, 0.125, out=out)
    assert ops.take_status() == 0
    assert bool((out[2] == 7.0).all()) and bool((out[5] == 7.0).all())
    keep = [i for i in range(8) if i not in (2, 5)]
    check_against_oracle(out, lens, tables, q, k, v, 7, 0.125, keep)


def test_one_workspace_serves_calls_of_any_size_in_any_order():
    """Single-sequence and batched calls of different sizes share one workspace;
    none may leave state that disturbs the next (segment counters stay zero)."""
    for B, median, seed in [(64, 1024, 11), (4, 50, 12), (256, 1024, 13), (16, 300, 14)]:
        lens, tables, bt, q, k, v = ragged_batch(B, 14, 2, 64, torch.bfloat16, median=median,
                                                 seed=seed)
        lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
        one = paged_attention(q[0], k, v, tables[0], lens[0], 16, 7, 0.125)
        out = ops.paged_attention_batched(q, k, v, bt, lens_d, 0.125)
        assert ops.take_status() == 0
        assert not out.isnan().any()
        assert (one.float() - out[0].float()).abs().max().item() <= 1e-2
        check_against_oracle(out, lens, tables, q, k, v, 7, 0.125, range(B))


@pytest.mark.parametrize("head_dim", [64, 128])
def test_a_wait_that_runs_out_reports_a_timeout_and_the_next_call_is_correct(head_dim):
    """The bounded-wait error path, made to happen without a fault: through the
    test hook, one warp of the tensor-core kernel waits on stages that nothing
    fills, with a 200 us limit.  The launch must finish, report the timeout bit
    (a RuntimeError on the host), leave no copy in flight, and leave the
    workspace so that the next call -- default limit -- is correct."""
    heads, kv_heads = (14, 2) if head_dim == 64 else (28, 4)
    lens, tables, bt, q, k, v = ragged_batch(64, heads, kv_heads, head_dim, torch.bfloat16,
                                             median=600, seed=21)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=DEV)
    scale = head_dim ** -0.5
    ops.set_wait_probe(True, 200_000)
    try:
        ops.paged_attention_batched(q, k, v, bt, lens_d, scale)
        with pytest.raises(RuntimeError, match="timed out"):
            ops.take_status()
    finally:
        ops.set_wait_probe(False, 0)
    for _ in range(2):
        out = ops.paged_attention_batched(q, k, v, bt, lens_d, scale)
        assert ops.take_status() == 0
        check_against_oracle(out, lens, tables, q, k, v, heads // kv_heads, scale, range(64))
