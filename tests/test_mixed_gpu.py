"""The mixed chunked-prefill + decode step on one pool, as the engine runs it:
8 prompt chunks of 512 tokens after priors U[0, 4096] plus 248 decode rows
(log-normal lengths, median 768, clipped to [16, 8192]) in one step --
step_metadata -> slot write of every new token -> batched decode of the 248
rows -> chunked prefill of the 8 chunks.  The reference composes the same step
as decode rows first, then prompt chunks (src/server/backend/paged.py:60-70),
attending each sequence in turn (src/server/torch_model.py:155-167).

Bounds as for the decode and prefill tests: bit-exact metadata and slot writes;
bf16 outputs element-wise within 0.01 + 2**-7 |ref| of the oracle's reference
rounding and within 2e-2 x max |ref| of fp32.
"""

import numpy as np
import pytest
import torch

import oracle
from batchstream_inference_engine_b200 import ops
from tests.golden import inputs
from tests.test_decode_gpu import check_against_oracle
from tests.test_prefill_gpu import check_rows

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
H, HKV, D, BS = 14, 2, 64, 16
CHUNK = 512


def build_step(seed=0):
    """One pool holding every sequence's cached context (N(0,1) bf16, NaN in
    unused slots), the step's new q/K/V rows and the device metadata inputs."""
    priors, dec_lens = inputs.mixed_step_shapes()
    Bd, P = len(dec_lens), len(priors)
    totals = np.concatenate([dec_lens, priors + CHUNK])
    starts = np.concatenate([dec_lens - 1, priors])
    counts = np.concatenate([np.ones(Bd, dtype=np.int64), np.full(P, CHUNK)])
    need = [-(-int(t) // BS) for t in totals]
    nb = sum(need) + 9
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(nb, generator=g)
    tables, cur = [], 0
    for m in need:
        tables.append(perm[cur: cur + m].tolist())
        cur += m
    bt = torch.full((len(totals), max(need)), -1, dtype=torch.int32)
    for r, t in enumerate(tables):
        bt[r, : len(t)] = torch.tensor(t, dtype=torch.int32)
    gd = torch.Generator(device=DEV).manual_seed(seed)
    k = torch.full((HKV, nb, BS, D), float("nan"), device=DEV)
    v = torch.full((HKV, nb, BS, D), float("nan"), device=DEV)
    # Cached context: positions 0 .. start - 1 of every row.
    slots = np.concatenate([np.array(tables[r])[np.arange(int(s)) // BS] * BS + np.arange(int(s)) % BS
                            for r, s in enumerate(starts)])
    idx = torch.from_numpy(slots).to(DEV)
    k.view(HKV, -1, D)[:, idx] = torch.randn((HKV, len(slots), D), generator=gd, device=DEV)
    v.view(HKV, -1, D)[:, idx] = torch.randn((HKV, len(slots), D), generator=gd, device=DEV)
    T = int(counts.sum())
    q = torch.randn((T, H, D), generator=gd, device=DEV).bfloat16()
    k_new = torch.randn((T, HKV, D), generator=gd, device=DEV).bfloat16()
    v_new = torch.randn((T, HKV, D), generator=gd, device=DEV).bfloat16()
    return dict(priors=priors, dec_lens=dec_lens, totals=totals, starts=starts, counts=counts,
                tables=tables, bt=bt.to(DEV), nb=nb, k=k.bfloat16(), v=v.bfloat16(), q=q,
                k_new=k_new, v_new=v_new, T=T)


def run_step(s, k_pool, v_pool):
    """The engine's order on one stream: metadata, slot write, decode, prefill."""
    Bd = len(s["dec_lens"])
    start_d = torch.tensor(s["starts"], dtype=torch.int32, device=DEV)
    n_d = torch.tensor(s["counts"], dtype=torch.int32, device=DEV)
    cu, pos, slots, ctx = ops.step_metadata(s["bt"], start_d, n_d, s["T"], BS, s["nb"])
    ops.reshape_and_cache(s["k_new"], s["v_new"], k_pool, v_pool, slots)
    ctx_host = torch.tensor(s["totals"], dtype=torch.int32, device=DEV)
    out = torch.full_like(s["q"], float("nan"))
    ops.paged_attention_batched(s["q"][:Bd], k_pool, v_pool, s["bt"], ctx_host[:Bd], D ** -0.5,
                                out=out[:Bd], lens_ready=True, after_append=True)
    ops.prefill_attention(s["q"][Bd:], k_pool, v_pool, s["bt"][Bd:], cu[Bd:] - Bd, ctx[Bd:],
                          D ** -0.5, max_query_len=CHUNK, out=out[Bd:])
    assert ops.take_status() == 0
    return out, (cu, pos, slots, ctx)


@pytest.fixture(scope="module")
def step():
    s = build_step()
    k_pool, v_pool = s["k"].clone(), s["v"].clone()
    out, meta = run_step(s, k_pool, v_pool)
    return s, k_pool, v_pool, out, meta


def test_mixed_step_metadata_and_slot_writes_are_exact(step):
    s, k_pool, v_pool, _, (cu, pos, slots, ctx) = step
    exp_pos, exp_slots = oracle.slot_mapping(s["tables"], s["starts"].tolist(),
                                             s["counts"].tolist(), BS)
    assert np.array_equal(slots.cpu().numpy(), exp_slots)
    assert np.array_equal(pos.cpu().numpy(), exp_pos)
    assert np.array_equal(ctx.cpu().numpy(), s["totals"])
    assert np.array_equal(cu.cpu().numpy(), np.concatenate([[0], np.cumsum(s["counts"])]))
    # Every new row sits at its slot, bit for bit; nothing else changed.
    idx = torch.from_numpy(exp_slots).to(DEV)
    assert torch.equal(k_pool.view(HKV, -1, D)[:, idx], s["k_new"].transpose(0, 1))
    assert torch.equal(v_pool.view(HKV, -1, D)[:, idx], s["v_new"].transpose(0, 1))
    mask = torch.ones(k_pool.view(HKV, -1, D).shape[1], dtype=torch.bool, device=DEV)
    mask[idx] = False
    for pool, orig in ((k_pool, s["k"]), (v_pool, s["v"])):
        kept = pool.view(HKV, -1, D)[:, mask].nan_to_num(7.0)
        assert torch.equal(kept, orig.view(HKV, -1, D)[:, mask].nan_to_num(7.0))


def test_every_decode_row_of_the_mixed_step_matches_the_oracle(step):
    s, k_pool, v_pool, out, _ = step
    Bd = len(s["dec_lens"])
    check_against_oracle(out[:Bd], s["dec_lens"].tolist(), s["tables"][:Bd], s["q"][:Bd],
                         k_pool, v_pool, H // HKV, D ** -0.5, range(Bd))


def test_mixed_step_prefill_tokens_match_the_oracle(step):
    s, k_pool, v_pool, out, _ = step
    Bd = len(s["dec_lens"])
    P = len(s["priors"])
    picks = [(r, i) for r in range(P) for i in (0, 1, 15, 16, 17, 127, 128, 255, 300, 511)]
    # check_rows reads the pool through the fp32 and bf16 views of k / v.
    check_rows(out[Bd:], s["q"][Bd:].float().cpu(), k_pool.float().cpu(), v_pool.float().cpu(),
               s["tables"][Bd:], [CHUNK] * P, s["priors"].tolist(), H // HKV, D ** -0.5, picks)


def test_mixed_step_prefill_every_token_against_fp32(step):
    """Every token of the 8 chunks against a plain torch fp32 attention of the
    same (bf16) inputs over its causal length."""
    s, k_pool, v_pool, out, _ = step
    Bd = len(s["dec_lens"])
    kf, vf = k_pool.float(), v_pool.float()
    start = Bd
    for r, p in enumerate(s["priors"].tolist()):
        total = p + CHUNK
        table = torch.tensor(s["tables"][Bd + r], device=DEV)
        sl = (table[:, None] * BS + torch.arange(BS, device=DEV)).reshape(-1)[:total]
        ks, vs = kf.view(HKV, -1, D)[:, sl], vf.view(HKV, -1, D)[:, sl]
        qs = s["q"][start: start + CHUNK].float().view(CHUNK, HKV, H // HKV, D)
        scores = torch.einsum("thgd,hkd->hgtk", qs, ks) * D ** -0.5
        vis = torch.arange(total, device=DEV)[None, :] <= (p + torch.arange(CHUNK, device=DEV))[:, None]
        scores = scores.masked_fill(~vis, float("-inf"))
        ref = torch.einsum("hgtk,hkd->thgd", torch.softmax(scores, -1), vs).reshape(CHUNK, H, D)
        got = out[start: start + CHUNK].float()
        err = (got - ref).abs().flatten(1).max(1).values
        bound = 2e-2 * ref.abs().flatten(1).max(1).values.clamp_min(1e-6)
        assert bool((err <= bound).all()), (r, int((err > bound).sum()))
        start += CHUNK


def test_mixed_step_is_deterministic_and_order_free(step):
    """The same step again on a fresh copy of the pool gives the same bits, and
    so does running the prefill before the decode."""
    s, _, _, out, _ = step
    k2, v2 = s["k"].clone(), s["v"].clone()
    again, _ = run_step(s, k2, v2)
    assert torch.equal(again, out)
    Bd = len(s["dec_lens"])
    k3, v3 = s["k"].clone(), s["v"].clone()
    start_d = torch.tensor(s["starts"], dtype=torch.int32, device=DEV)
    n_d = torch.tensor(s["counts"], dtype=torch.int32, device=DEV)
    cu, _, slots, ctx = ops.step_metadata(s["bt"], start_d, n_d, s["T"], BS, s["nb"])
    ops.reshape_and_cache(s["k_new"], s["v_new"], k3, v3, slots)
    swapped = torch.empty_like(out)
    ops.prefill_attention(s["q"][Bd:], k3, v3, s["bt"][Bd:], cu[Bd:] - Bd, ctx[Bd:], D ** -0.5,
                          max_query_len=CHUNK, out=swapped[Bd:])
    ops.paged_attention_batched(s["q"][:Bd], k3, v3, s["bt"], ctx[:Bd], D ** -0.5,
                                out=swapped[:Bd])
    assert ops.take_status() == 0
    assert torch.equal(swapped, out)
