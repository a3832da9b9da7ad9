"""The paged backend on the GPU against the reference's own paged backend.

Golden tokens (tests/golden/engine_tokens.npz, from make_engine_golden.py) come
from the reference TorchModel + PagedBackend driven by its BatchingScheduler on
the CPU: 24 token-id prompts, random-init Qwen2.5-0.5B-shaped weights (seed 0,
N(0, 0.02), RMSNorm 1), max 8 concurrent, 256 blocks of 16, prefill chunk 64.

* fp32: the GPU engine (fp32 weights, fp32 pool, IEEE fp32 GEMMs) must give the
  reference's greedy token ids for the first 32 tokens of every sequence, up to
  a near-tie: where the reference's best and second-best logits lie within
  2e-3 of the largest (tests/golden/engine_margins.npz, from
  make_engine_margins.py) the last bits of another GEMM kernel may pick the
  other one, and the two runs part there.
* bf16: free-running greedy decoding in bf16 flips on near-ties (the
  reference's own bf16 run leaves its fp32 run within 0-88 tokens), so bf16 is
  held to the reference's fp32 logits teacher-forced along the fp32 token
  stream: logits at the reference's top-16 ids within the reference bf16
  model's own error envelope (2.19e-2 of the largest, + 2**-8), on average
  within twice its mean error, and every greedy pick a near-tie of the
  reference's best.  fp32 is held to 1e-3 and the same pick on the same test.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from batchstream_inference_engine_b200.backend import PagedBackend
from batchstream_inference_engine_b200.serve import BlockBudget, engine_workload, serve
from batchstream_inference_engine_b200.torch_model import (QWEN25_05B, PagedKVPool, TorchModel,
                                                          random_weights)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLDEN = Path(__file__).resolve().parent / "golden" / "engine_tokens.npz"
MARGINS = Path(__file__).resolve().parent / "golden" / "engine_margins.npz"
NEAR_TIE = 2e-3  # twice the fp32 logit tolerance of the teacher-forced test
NUM_BLOCKS, BLOCK_SIZE, PREFILL_CHUNK, MAX_CONCURRENT = 256, 16, 64, 8


def unpack(values, offsets):
    return [values[offsets[i]: offsets[i + 1]].tolist() for i in range(len(offsets) - 1)]


@pytest.fixture(scope="module")
def golden():
    g = np.load(GOLDEN)
    return {
        "prompts": unpack(g["prompts"], g["prompt_offsets"]),
        "max_tokens": g["max_tokens"].tolist(),
        "fp32": unpack(g["tokens_fp32"], g["offsets_fp32"]),
        "bf16": unpack(g["tokens_bf16"], g["offsets_bf16"]),
    }


@pytest.fixture(scope="module")
def weights():
    return random_weights()


def run_engine(weights, dtype, step_graphs=True, pipelined=False):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        model = TorchModel(QWEN25_05B, weights, device=DEV, dtype=dtype, step_graphs=step_graphs)
        backend = PagedBackend(model, NUM_BLOCKS, BLOCK_SIZE, PREFILL_CHUNK)
        requests = serve(backend, engine_workload(), MAX_CONCURRENT,
                         BlockBudget(NUM_BLOCKS, BLOCK_SIZE), pipelined=pipelined)
        assert backend.blocks_in_use == 0
        if step_graphs:  # every step of this workload fits a step graph
            assert model.stats["steps"] > 0 and len(model._graphs) > 0
        return [r.tokens for r in requests], requests
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_workload_matches_the_fixture(golden):
    specs = engine_workload()
    assert [p for p, _ in specs] == golden["prompts"]
    assert [m for _, m in specs] == golden["max_tokens"]


@pytest.mark.parametrize("step_graphs,pipelined", [(True, True), (True, False), (False, False)],
                         ids=["graphs-pipelined", "graphs", "eager"])
def test_fp32_greedy_tokens_match_the_reference(golden, weights, step_graphs, pipelined):
    tokens, requests = run_engine(weights, torch.float32, step_graphs, pipelined)
    assert not any(r.failed for r in requests)
    margins = np.load(MARGINS)["margins_fp32"]
    for i, (ours, ref) in enumerate(zip(tokens, golden["fp32"])):
        n = min(32, len(ref))
        k = first_divergence(ours[:n], ref[:n])
        if k < n:
            # Only at a near-tie of the reference's own logits.
            assert margins[i, k] <= NEAR_TIE, (i, k, float(margins[i, k]), ours[:n], ref[:n])
        else:
            assert len(ours) == len(ref), i


def first_divergence(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return min(len(a), len(b))


def test_bf16_engine_runs_the_workload_to_completion(golden, weights):
    tokens, requests = run_engine(weights, torch.bfloat16, pipelined=True)
    assert not any(r.failed for r in requests)
    # Every sequence runs to its own max_tokens, as in the reference's bf16 run.
    assert [len(t) for t in tokens] == [len(t) for t in golden["bf16"]]
    # Free-running greedy bf16 decoding leaves any other bf16 run at the first
    # near-tie (the reference's own bf16 run leaves its fp32 run after 0-88
    # tokens); the teacher-forced test below holds the logits to tolerance.
    agree = [first_divergence(ours, ref) for ours, ref in zip(tokens, golden["bf16"])]
    print("bf16 tokens agreeing with the reference bf16 run:", agree)


def teacher_forced(weights, dtype, golden):
    """Last-token logits along each fixture sequence's fp32 token stream: the
    prompt as one chunk, then one token per step."""
    g = np.load(GOLDEN)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        model = TorchModel(QWEN25_05B, weights, device=DEV, dtype=dtype)
        out = []
        for s in g["logit_seqs"].tolist():
            pool = PagedKVPool(QWEN25_05B, NUM_BLOCKS, BLOCK_SIZE, device=DEV, dtype=dtype)
            cache = pool.new_cache(0)
            feed, rows = golden["prompts"][s], []
            for step in range(g["logit_ids"].shape[1]):
                rows.append(model.forward_batch([(feed, cache)])[0].float().cpu())
                feed = [golden["fp32"][s][step]]
            out.append(torch.stack(rows))
        return out, g["logit_ids"], g["logit_values"]
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("dtype,rel", [(torch.float32, 1e-3), (torch.bfloat16, 2e-2)])
def test_teacher_forced_logits_against_the_reference_fp32(golden, weights, dtype, rel):
    """At every position: logits at the reference's top-16 ids within `rel` of
    the largest, and the greedy choice a near-tie (within 2 * rel) of the
    reference's best (for fp32: the same token).

    For bf16 the error at a position is rounding noise accumulated over 24
    layers, and the reference's own bf16 model shows how large it gets on this
    workload: up to 2.19e-2 of the largest logit.  So bf16 is held at every
    position to max(2e-2, that envelope + 2**-8), and on average to at most
    twice the reference bf16 model's mean error (a systematic error fails)."""
    logits, ids, values = teacher_forced(weights, dtype, golden)
    ref_bf16 = np.load(GOLDEN)["ref_bf16_logit_err"]
    bound = rel if dtype == torch.float32 else max(rel, float(ref_bf16.max()) + 2.0 ** -8)
    errors = np.zeros(ref_bf16.shape)
    for n, seq in enumerate(logits):
        for step in range(ids.shape[1]):
            ref_ids = torch.from_numpy(ids[n, step]).long()
            ref = torch.from_numpy(values[n, step])
            scale = ref.abs().max().item()
            tol = bound * scale
            ours = seq[step][ref_ids]
            errors[n, step] = (ours - ref).abs().max().item() / scale
            assert errors[n, step] <= bound, (n, step, errors[n, step], bound)
            pick = int(seq[step].argmax())
            if dtype == torch.float32:
                assert pick == int(ref_ids[0]), (n, step)
            else:
                hit = (ref_ids == pick).nonzero()
                assert hit.numel() == 1, (n, step, pick)
                assert ref[hit[0, 0]].item() >= ref[0].item() - 2 * tol, (n, step)
    print(f"{dtype}: relative logit error max {errors.max():.4f} mean {errors.mean():.4f}; "
          f"reference bf16 model max {ref_bf16.max():.4f} mean {ref_bf16.mean():.4f}")
    if dtype == torch.bfloat16:
        assert errors.mean() <= 2 * ref_bf16.mean(), (errors.mean(), ref_bf16.mean())
