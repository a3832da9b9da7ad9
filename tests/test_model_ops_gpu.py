"""The fused model-step kernels (residual add + RMSNorm, rotary embedding + K/V
append, SwiGLU gating) against the reference TorchModel's own torch formulas
(src/server/torch_model.py:190-192, 262-264, 278-287) run as separate ops on
the same device: the rounding points are the same, so rotary, gating and the
residual sums match bit for bit; RMSNorm differs only through the order of
its fp32 sum of squares."""

import pytest
import torch
import torch.nn.functional as F

from batchstream_inference_engine_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
EPS = 1e-6


def ref_rms_norm(s: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    wide = s.to(torch.float32)
    variance = wide.pow(2).mean(-1, keepdim=True)
    normalized = wide * torch.rsqrt(variance + EPS)
    return weight * normalized.to(s.dtype)


def ref_rotate_half(x: torch.Tensor) -> torch.Tensor:
    first, second = x.chunk(2, dim=-1)
    return torch.cat((-second, first), dim=-1)


def rotary_tables(positions: int, D: int, dtype, theta=1_000_000.0):
    steps = torch.arange(0, D, 2, dtype=torch.float)
    inv = 1.0 / (theta ** (steps / D))
    freqs = torch.arange(positions)[:, None].float() * inv
    angles = torch.cat((freqs, freqs), dim=-1)
    return (angles.cos().to(torch.bfloat16).to(DEV, dtype),
            angles.sin().to(torch.bfloat16).to(DEV, dtype))


def norm_bound(out, ref, dtype):
    # One rounding of the normalised value (before x weight) and of the product
    # may flip with the last bit of the fp32 statistics.
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -20
    return (out.float() - ref.float()).abs().max().item(), 2 * ulp * ref.float().abs().max().item()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("hidden", [896, 2048, 100], ids=["vector", "vector_long", "scalar"])
def test_rms_norm_with_residual_add_in_place(dtype, hidden):
    g = torch.Generator(device=DEV).manual_seed(0)
    T = 37
    x = torch.randn(T, hidden, generator=g, device=DEV).to(dtype)
    add = torch.randn(T, hidden, generator=g, device=DEV).to(dtype) * 3
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device=DEV)).to(dtype)
    s_ref = x + add
    ref = ref_rms_norm(s_ref, w)
    hidden_stream = x.clone()
    out = ops.rms_norm(hidden_stream, w, EPS, add=add, sum_out=hidden_stream)
    assert torch.equal(hidden_stream, s_ref)  # the residual stream, bit for bit
    err, bound = norm_bound(out, ref, dtype)
    assert err <= bound, (err, bound)
    # Without an add it is the plain norm and leaves x alone.
    plain = ops.rms_norm(x, w, EPS)
    err, bound = norm_bound(plain, ref_rms_norm(x, w), dtype)
    assert err <= bound
    ops.take_status(torch.device(DEV))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rms_norm_gathers_rows(dtype):
    g = torch.Generator(device=DEV).manual_seed(1)
    vocab, hidden = 1000, 256
    table = torch.randn(vocab, hidden, generator=g, device=DEV).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device=DEV)).to(dtype)
    idx = torch.tensor([5, 999, 0, 5, 731], dtype=torch.int32, device=DEV)
    gathered = torch.empty(idx.numel(), hidden, dtype=dtype, device=DEV)
    out = ops.rms_norm(table, w, EPS, row_index=idx, sum_out=gathered)
    assert torch.equal(gathered, table[idx.long()])
    err, bound = norm_bound(out, ref_rms_norm(table[idx.long()], w), dtype)
    assert err <= bound
    # Gather with an add: the last-token rows of a residual stream.
    add = torch.randn(vocab, hidden, generator=g, device=DEV).to(dtype)
    out2 = ops.rms_norm(table, w, EPS, add=add, row_index=idx)
    err, bound = norm_bound(out2, ref_rms_norm((table + add)[idx.long()], w), dtype)
    assert err <= bound
    ops.take_status(torch.device(DEV))


def test_rms_norm_bad_index_sets_status():
    x = torch.randn(8, 64, device=DEV)
    w = torch.ones(64, device=DEV)
    idx = torch.tensor([0, 8], dtype=torch.int32, device=DEV)
    ops.rms_norm(x, w, EPS, row_index=idx)
    with pytest.raises(RuntimeError, match="gathered row index"):
        ops.take_status(torch.device(DEV))


def make_rope_case(dtype, pool_dtype, T=29, H=14, Hkv=2, D=64, NB=40, bs=16, seed=2):
    g = torch.Generator(device=DEV).manual_seed(seed)
    qkv = torch.randn(T, (H + 2 * Hkv) * D, generator=g, device=DEV).to(dtype)
    cos, sin = rotary_tables(4096, D, dtype)
    positions = torch.randint(0, 4096, (T,), generator=g, device=DEV, dtype=torch.int32)
    slots = torch.randperm(NB * bs, generator=g, device=DEV)[:T].to(torch.int32)
    slots[3] = -1  # a padding row: no pool write
    kp = torch.randn(Hkv, NB, bs, D, generator=g, device=DEV).to(pool_dtype)
    vp = torch.randn(Hkv, NB, bs, D, generator=g, device=DEV).to(pool_dtype)
    return qkv, cos, sin, positions, slots, kp, vp, (T, H, Hkv, D)


@pytest.mark.parametrize("dtype,pool_dtype", [(torch.float32, torch.float32),
                                              (torch.bfloat16, torch.bfloat16),
                                              (torch.float32, torch.bfloat16)])
def test_rope_append_matches_the_torch_ops_bit_for_bit(dtype, pool_dtype):
    qkv, cos, sin, positions, slots, kp, vp, (T, H, Hkv, D) = make_rope_case(dtype, pool_dtype)
    kp_ref, vp_ref = kp.clone(), vp.clone()
    c = cos.index_select(0, positions.long())[:, None]
    s = sin.index_select(0, positions.long())[:, None]
    q = qkv[:, : H * D].view(T, H, D)
    k = qkv[:, H * D: (H + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (H + Hkv) * D:].view(T, Hkv, D)
    q_ref = q * c + ref_rotate_half(q) * s
    k_ref = k * c + ref_rotate_half(k) * s
    live = slots >= 0
    sl = slots[live].long()
    bs = kp.shape[2]
    kp_ref[:, sl // bs, sl % bs] = k_ref[live].transpose(0, 1).to(pool_dtype)
    vp_ref[:, sl // bs, sl % bs] = v[live].transpose(0, 1).to(pool_dtype)

    q_out = ops.rope_append(qkv, cos, sin, positions, slots, kp, vp, H)
    ops.take_status(torch.device(DEV))
    assert torch.equal(q_out, q_ref)
    assert torch.equal(kp, kp_ref)
    assert torch.equal(vp, vp_ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["vector", "scalar"])
def test_rope_append_reports_bad_positions_and_slots(dtype):
    qkv, cos, sin, positions, slots, kp, vp, (T, H, Hkv, D) = make_rope_case(
        dtype, torch.bfloat16)
    before_k, before_v = kp.clone(), vp.clone()
    bad_pos = positions.clone()
    bad_pos[0] = cos.shape[0]
    ops.rope_append(qkv[:1], cos, sin, bad_pos[:1], torch.full_like(slots[:1], -1), kp, vp, H)
    with pytest.raises(RuntimeError, match="rotary tables"):
        ops.take_status(torch.device(DEV))
    bad_slot = slots.clone()
    bad_slot[0] = kp.shape[1] * kp.shape[2]
    ops.rope_append(qkv[:1], cos, sin, positions[:1], bad_slot[:1], kp, vp, H)
    with pytest.raises(RuntimeError, match="slot outside the pool"):
        ops.take_status(torch.device(DEV))
    assert torch.equal(kp, before_k) and torch.equal(vp, before_v)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("inter", [4864, 37], ids=["vector", "scalar"])
def test_silu_mul_matches_the_torch_ops(dtype, inter):
    g = torch.Generator(device=DEV).manual_seed(3)
    T = 53
    gate_up = (torch.randn(T, 2 * inter, generator=g, device=DEV) * 4).to(dtype)
    gate, up = gate_up.split(inter, dim=-1)
    ref = F.silu(gate) * up
    out = ops.silu_mul(gate_up)
    # Same expression and roundings as torch's SiLU kernel; allow one ulp for
    # the exponential, whose implementation could differ between the builds.
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -22
    diff = (out.float() - ref.float()).abs()
    assert (diff <= ulp * ref.float().abs() + 1e-30).all(), diff.max().item()


def test_locate_only_decode_append_matches_the_full_append():
    torch.manual_seed(4)
    Hkv, NB, bs, D = 2, 64, 16, 64
    kp = torch.randn(Hkv, NB, bs, D, device=DEV).bfloat16()
    vp = torch.randn(Hkv, NB, bs, D, device=DEV).bfloat16()
    tables = torch.randperm(NB, device=DEV)[:48].view(6, 8).to(torch.int32)
    start = torch.tensor([0, 17, 127, -1, 64, 5], dtype=torch.int32, device=DEV)
    k = torch.randn(6, Hkv, D, device=DEV).bfloat16()
    v = torch.randn(6, Hkv, D, device=DEV).bfloat16()
    before_k, before_v = kp.clone(), vp.clone()
    ctx0, slots0 = ops.decode_append(None, None, kp, vp, tables, start)
    assert torch.equal(kp, before_k) and torch.equal(vp, before_v)
    ctx1, slots1 = ops.decode_append(k, v, kp, vp, tables, start)
    ops.take_status(torch.device(DEV))
    assert torch.equal(ctx0, ctx1) and torch.equal(slots0, slots1)
    assert slots0[3].item() == -1 and ctx0[3].item() == 0


def test_kernel_launch_counter_counts_each_kernel():
    x = torch.randn(4, 64, device=DEV)
    w = torch.ones(64, device=DEV)
    before = ops.kernel_launches()
    ops.rms_norm(x, w, EPS)
    ops.silu_mul(torch.randn(4, 128, device=DEV))
    assert ops.kernel_launches() - before == 2
    # A tensor-core decode is the split-K kernel plus its merge pass.
    Hkv, G, D, NB, bs = 2, 7, 64, 8, 16
    kp = torch.randn(Hkv, NB, bs, D, device=DEV).bfloat16()
    vp = torch.randn(Hkv, NB, bs, D, device=DEV).bfloat16()
    q = torch.randn(2, Hkv * G, D, device=DEV).bfloat16()
    tables = torch.arange(NB, device=DEV, dtype=torch.int32).view(2, 4)
    ctx = torch.tensor([40, 64], dtype=torch.int32, device=DEV)
    before = ops.kernel_launches()
    ops.paged_attention_batched(q, kp, vp, tables, ctx, D ** -0.5)
    ops.take_status(torch.device(DEV))
    assert ops.kernel_launches() - before == 2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("vocab", [151936, 1001], ids=["vector", "scalar"])
def test_argmax_rows_matches_torch(dtype, vocab):
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(37, vocab, generator=g, device=DEV).to(dtype)
    x[3, 10] = x[3, 500] = x[3].max() + 1  # a tie: the first index wins
    x[4] = -float("inf")                   # all -inf: index 0
    x[5, 77] = float("nan")                # NaN counts as the maximum
    x[6, 900] = x[6, 100] = float("nan")   # the first NaN
    if vocab > 6 * 4096:
        # Ties among one thread's elements (every 4096th column, 8 per chunk),
        # loaded in the same round and in different rounds.
        x[7, 8 + 2 * 4096] = x[7, 8] = x[7].max() + 1
        x[8, 9 + 5 * 4096] = x[8, 9 + 4096] = x[8].max() + 1
    got = ops.argmax_rows(x)
    assert torch.equal(got.long(), x.float().argmax(dim=-1))
    assert got[3].item() == 10 and got[4].item() == 0 and got[5].item() == 77
    assert got[6].item() == 100
