"""Chunked-prefill attention on the GPU against the reference attend() outputs
(golden fixtures) and the oracle.

Tolerances as for decode: fp32 max-abs 1e-4 against the fp32 reference; bf16
max-abs <= 2e-2 * max|ref| against fp32, and element-wise
|out - ref_bf16| <= 0.01 + 2**-7 |ref_bf16| against the reference's bf16 attend().
Both the tcgen05 path (bf16, head_dim 64) and the per-token path run.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from batchstream_inference_engine_b200 import ops
from tests.golden import inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLDEN = Path(__file__).resolve().parent / "golden"


def close_bf16(out, ref_bf16):
    out, ref = out.float().cpu(), ref_bf16.float().cpu()
    return bool(((out - ref).abs() <= 0.01 + 2.0 ** -7 * ref.abs()).all())


def rel_err(out, ref32):
    ref = torch.as_tensor(ref32).float()
    return ((out.float().cpu() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


def single_chunk(q, k, v, table, past, dtype, per_token):
    n, H, D = q.shape
    qd = q.to(dtype).to(DEV)
    kd, vd = k.to(dtype).to(DEV), v.to(dtype).to(DEV)
    bt = torch.tensor([table], dtype=torch.int32, device=DEV)
    cu = torch.tensor([0, n], dtype=torch.int32, device=DEV)
    ctx = torch.tensor([past + n], dtype=torch.int32, device=DEV)
    Hkv = k.shape[0]
    out = ops.prefill_attention(qd, kd, vd, bt, cu, ctx, D ** -0.5 if D != 64 else 0.125,
                                max_query_len=n, per_token=per_token)
    assert ops.take_status() == 0
    return out


@pytest.mark.parametrize("case", inputs.PREFILL_CASES)
@pytest.mark.parametrize("per_token", [False, True])
def test_prefill_matches_reference_attend(case, per_token):
    n, past, heads, kv_heads = case
    gold = np.load(GOLDEN / "prefill.npz")
    q, k, v, table = inputs.prefill_case(n, past, heads, kv_heads)
    b16 = single_chunk(q, k, v, table, past, torch.bfloat16, per_token)
    assert not b16.isnan().any()
    assert close_bf16(b16, inputs.from_bits(gold[f"bf16_{n}_{past}"]))
    assert rel_err(b16, gold[f"f32_{n}_{past}"]) <= 2e-2
    f32 = single_chunk(q, k, v, table, past, torch.float32, per_token)
    assert np.abs(f32.cpu().numpy() - gold[f"f32_{n}_{past}"]).max() <= 1e-4


def mixed_prefill_batch(chunks, priors, heads=14, kv_heads=2, head_dim=64, seed=0):
    """Chunks of `chunks[r]` tokens after `priors[r]` cached ones, paged over a
    shuffled pool whose unused slots are NaN."""
    g = torch.Generator().manual_seed(seed)
    totals = [p + c for p, c in zip(priors, chunks)]
    need = [-(-t // 16) for t in totals]
    nb = sum(need) + 7
    perm = torch.randperm(nb, generator=g)
    tables, cur = [], 0
    for m in need:
        tables.append(perm[cur: cur + m].tolist())
        cur += m
    k = torch.full((kv_heads, nb, 16, head_dim), float("nan"))
    v = torch.full((kv_heads, nb, 16, head_dim), float("nan"))
    for r, t in enumerate(totals):
        kk = torch.randn(kv_heads, t, head_dim, generator=g)
        vv = torch.randn(kv_heads, t, head_dim, generator=g)
        idx = torch.tensor([tables[r][p // 16] * 16 + p % 16 for p in range(t)])
        k.view(kv_heads, -1, head_dim)[:, idx] = kk
        v.view(kv_heads, -1, head_dim)[:, idx] = vv
    T = sum(chunks)
    q = torch.randn(T, heads, head_dim, generator=g)
    width = max(need)
    bt = torch.full((len(chunks), width), -1, dtype=torch.int32)
    for r, t in enumerate(tables):
        bt[r, : len(t)] = torch.tensor(t, dtype=torch.int32)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(chunks)]), dtype=torch.int32)
    ctx = torch.tensor(totals, dtype=torch.int32)
    return q, k, v, tables, bt, cu, ctx


def fp32_reference(q, k, v, tables, chunks, priors, groups, scale):
    """fp32 attention of every chunk token over its causal length, from the
    bf16-rounded inputs: [T, H, D].  The raw scores q . k are rounded to bf16
    first, as the reference's bf16 matmul leaves them (its largest departure
    from fp32: up to about 2% of the output's range on a token whose top
    scores are large); softmax and P V stay in fp32."""
    kf, vf = k.bfloat16().float(), v.bfloat16().float()
    Hkv, _, bs, D = kf.shape
    outs, start = [], 0
    for r, (c, p) in enumerate(zip(chunks, priors)):
        total = p + c
        slots = (torch.tensor(tables[r])[:, None] * bs + torch.arange(bs)).reshape(-1)[:total]
        ks = kf.view(Hkv, -1, D)[:, slots]  # [Hkv, total, D]
        vs = vf.view(Hkv, -1, D)[:, slots]
        qs = q[start: start + c].bfloat16().float().view(c, Hkv, groups, D)
        scores = torch.einsum("thgd,hkd->hgtk", qs, ks).bfloat16().float() * scale
        visible = torch.arange(total)[None, :] <= (p + torch.arange(c))[:, None]
        scores = scores.masked_fill(~visible, float("-inf"))
        o = torch.einsum("hgtk,hkd->thgd", torch.softmax(scores, dim=-1), vs)
        outs.append(o.reshape(c, Hkv * groups, D))
        start += c
    return torch.cat(outs)


def check_all_rows(out, ref32):
    """Per token: max |out - ref| <= 2e-2 * max |ref| over its heads."""
    err = (out.float().cpu() - ref32).abs().flatten(1).max(1).values
    scale = ref32.abs().flatten(1).max(1).values.clamp_min(1e-6)
    bad = torch.nonzero(err > 2e-2 * scale).flatten().tolist()
    assert not bad, bad[:20]


def check_rows(out, q, k, v, tables, chunks, priors, groups, scale, picks):
    """Each picked query token against the oracle's decode over its causal length."""
    kb, vb = inputs.bf16_bits(k.bfloat16()), inputs.bf16_bits(v.bfloat16())
    kf, vf = k.bfloat16().float().numpy(), v.bfloat16().float().numpy()
    starts = np.concatenate([[0], np.cumsum(chunks)])
    for r, i in picks:
        t = starts[r] + i
        length = priors[r] + i + 1
        qb = q[t].bfloat16()
        ref16 = oracle.decode(inputs.bf16_bits(qb), kb, vb, tables[r], length, 16, groups, scale)
        ref32 = oracle.decode(qb.float().numpy(), kf, vf, tables[r], length, 16, groups, scale)
        assert close_bf16(out[t], inputs.from_bits(ref16)), (r, i)
        assert rel_err(out[t], ref32) <= 2e-2, (r, i)


@pytest.mark.parametrize("per_token", [False, True])
def test_mixed_prefill_step_shape(per_token):
    # The mixed-step prefill shape: 512-token chunks after lengthy cached prefixes.
    rng = np.random.default_rng(0)
    priors = rng.integers(0, 4097, 8).tolist()
    chunks = [512] * 8
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch(chunks, priors)
    out = ops.prefill_attention(q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV),
                                bt.to(DEV), cu.to(DEV), ctx.to(DEV), 0.125, max_query_len=512,
                                per_token=per_token)
    assert ops.take_status() == 0
    assert not out.isnan().any()
    check_all_rows(out, fp32_reference(q, k, v, tables, chunks, priors, 7, 0.125))
    picks = [(r, i) for r in range(8) for i in (0, 1, 15, 16, 17, 127, 128, 300, 511)]
    check_rows(out, q, k, v, tables, chunks, priors, 7, 0.125, picks)


def test_ragged_chunks_edge_cases():
    # Chunks shorter than a tile, not multiples of 16 or 128, with and without a
    # cached prefix, prefixes not aligned to blocks.
    chunks = [1, 5, 16, 17, 127, 128, 129, 300]
    priors = [0, 3, 16, 31, 0, 200, 77, 1000]
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch(chunks, priors, seed=4)
    args = (q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV), bt.to(DEV),
            cu.to(DEV), ctx.to(DEV), 0.125)
    fast = ops.prefill_attention(*args, max_query_len=max(chunks))
    slow = ops.prefill_attention(*args, max_query_len=max(chunks), per_token=True)
    assert ops.take_status() == 0
    assert not fast.isnan().any()
    # Every token of both paths against the oracle (the reference's rounding).
    picks = [(r, i) for r, c in enumerate(chunks) for i in range(c)]
    check_rows(fast, q, k, v, tables, chunks, priors, 7, 0.125, picks)
    check_rows(slow, q, k, v, tables, chunks, priors, 7, 0.125, picks)


@pytest.mark.parametrize("chunks,priors", [
    ([300], [2000]),        # 42 query tiles: key ranges of 36 tiles in 4 CTAs each
    ([70], [5000]),         # one tile, rows past the chunk: 4 ranges of ~20 tiles
    ([512, 9], [900, 40]),  # a short prefix caps the split (at least 4 tiles each)
])
def test_split_key_ranges_match_the_oracle(chunks, priors):
    # Fewer query tiles than SMs: each tile's key range is split over several
    # CTAs and their partial results merged; every token against the oracle.
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch(chunks, priors, seed=11)
    args = (q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV), bt.to(DEV),
            cu.to(DEV), ctx.to(DEV), 0.125)
    out = ops.prefill_attention(*args, max_query_len=max(chunks))
    assert ops.take_status() == 0
    assert not out.isnan().any()
    check_all_rows(out, fp32_reference(q, k, v, tables, chunks, priors, 7, 0.125))
    picks = [(r, i) for r, c in enumerate(chunks) for i in range(c)]
    check_rows(out, q, k, v, tables, chunks, priors, 7, 0.125, picks)
    for _ in range(3):  # the split and its merge are deterministic
        assert torch.equal(ops.prefill_attention(*args, max_query_len=max(chunks)), out)


def test_prefill_repeated_calls_are_identical():
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch([200, 64], [500, 9], seed=8)
    args = (q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV), bt.to(DEV),
            cu.to(DEV), ctx.to(DEV), 0.125)
    a = ops.prefill_attention(*args, max_query_len=200)
    b = ops.prefill_attention(*args, max_query_len=200)
    assert torch.equal(a, b)


def test_mixed_step_is_bitwise_stable_across_launches():
    # No atomics touch the arithmetic, so every launch must give the same bits;
    # a race between the loader, MMA and softmax warps shows up as a difference.
    rng = np.random.default_rng(0)
    priors = rng.integers(0, 4097, 8).tolist()
    chunks = [512] * 8
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch(chunks, priors)
    args = (q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV), bt.to(DEV),
            cu.to(DEV), ctx.to(DEV), 0.125)
    first = ops.prefill_attention(*args, max_query_len=512)
    check_all_rows(first, fp32_reference(q, k, v, tables, chunks, priors, 7, 0.125))
    for _ in range(8):
        assert torch.equal(ops.prefill_attention(*args, max_query_len=512), first)
    assert ops.take_status() == 0


def test_prefill_bad_table_sets_status():
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch([40], [100], seed=9)
    bad = bt.clone()
    bad[0, 2] = k.size(1) + 3
    ops.prefill_attention(q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV),
                          bad.to(DEV), cu.to(DEV), ctx.to(DEV), 0.125, max_query_len=40)
    with pytest.raises(RuntimeError, match="block table"):
        ops.take_status()


def _prefill_launches(chunks, priors, max_query_len=None, seed=3):
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch(chunks, priors, seed=seed)
    args = (q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV), bt.to(DEV),
            cu.to(DEV), ctx.to(DEV), 0.125)
    mq = max_query_len or max(chunks)
    ops.prefill_attention(*args, max_query_len=mq)  # workspace sized outside the count
    torch.cuda.synchronize(DEV)
    before = ops.kernel_launches()
    out = ops.prefill_attention(*args, max_query_len=mq)
    torch.cuda.synchronize(DEV)
    assert ops.take_status() == 0
    check_all_rows(out, fp32_reference(q, k, v, tables, chunks, priors, 7, 0.125))
    return ops.kernel_launches() - before


def test_prefill_launch_policy():
    # Query tiles (chunks x heads x 128-token tiles) below the SM count: key
    # ranges split, merged by a second kernel.  Up to one wave of resident CTAs
    # (two per SM): the prefill kernel alone.  More than a wave: the tiles are
    # ranked by key tiles first, inside every CTA for up to 192 (chunk, query
    # tile) pairs, by a planning kernel launched ahead for more.
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    small = ([300], [2000])                   # 14 x 3 = 42 tiles
    one_wave = ([200] * 8, [64 * i for i in range(8)])   # 8 x 14 x 2 = 224 tiles
    large = ([512] * 8, [3485, 2609, 2094, 1105, 1261, 167, 308, 67])  # 32 pairs, 448 tiles
    many = ([200] * 100, [37 * (i % 11) for i in range(100)])  # 200 pairs, 2800 tiles
    assert 42 < sms <= 224 <= 2 * sms < 448
    base = _prefill_launches(*one_wave)
    assert _prefill_launches(*small) == base + 1
    assert _prefill_launches(*large) == base
    assert _prefill_launches(*many) == base + 1
    # A padded launch (a CUDA-graph bucket of 512 query tokens holding four
    # 128-token chunks): 224 query tiles launched, at most 8 x 14 hold tokens,
    # so the key ranges are split and merged.
    padded = ([128] * 4, [2000, 500, 100, 1200])
    assert _prefill_launches(*padded, max_query_len=512) == base + 1


@pytest.mark.parametrize("rows,plan_launches", [(96, 0), (97, 1)])
def test_work_ranked_in_the_ctas_up_to_192_pairs(rows, plan_launches):
    # Every chunk holds 129..256 tokens, two query tiles: 96 chunks are the
    # largest batch the CTAs rank themselves (192 pairs), 97 take the planning
    # kernel.  Both exceed a wave of CTAs; every token is checked against fp32
    # and sampled tokens against the oracle.
    chunks = [129 + (37 * i) % 128 for i in range(rows)]
    priors = [(53 * i) % 700 for i in range(rows)]
    base = _prefill_launches([200] * 8, [64 * i for i in range(8)])
    assert _prefill_launches(chunks, priors, max_query_len=256, seed=17) == base + plan_launches
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch(chunks, priors, seed=17)
    out = ops.prefill_attention(q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV),
                                bt.to(DEV), cu.to(DEV), ctx.to(DEV), 0.125, max_query_len=256)
    assert ops.take_status() == 0
    picks = [(r, i) for r in (0, rows // 2, rows - 1) for i in (0, 128, chunks[r] - 1)]
    check_rows(out, q, k, v, tables, chunks, priors, 7, 0.125, picks)


def test_planned_prefill_bad_table_sets_status():
    # The planned path reads each row from its plan entry; a bad block-table
    # entry is still reported, not read.
    chunks, priors = [512] * 8, [700, 9, 1500, 300, 64, 2048, 5, 900]
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch(chunks, priors, seed=12)
    bad = bt.clone()
    bad[5, 7] = k.size(1) + 11
    ops.prefill_attention(q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV),
                          bad.to(DEV), cu.to(DEV), ctx.to(DEV), 0.125, max_query_len=512)
    with pytest.raises(RuntimeError, match="block table"):
        ops.take_status()


def test_planned_prefill_chunk_longer_than_max_query_len_sets_status():
    # 12 chunks x 14 heads x 2 tiles: a planned launch; chunk 3 holds more
    # tokens than max_query_len allows.
    chunks = [256] * 12
    chunks[3] = 300
    priors = [37 * i for i in range(12)]
    q, k, v, tables, bt, cu, ctx = mixed_prefill_batch(chunks, priors, seed=13)
    ops.prefill_attention(q.bfloat16().to(DEV), k.bfloat16().to(DEV), v.bfloat16().to(DEV),
                          bt.to(DEV), cu.to(DEV), ctx.to(DEV), 0.125, max_query_len=256)
    with pytest.raises(RuntimeError, match="context length"):
        ops.take_status()
