"""Pins the oracle's CPU model step (oracle/engine.py) against the reference's
own fp32 logits stored in tests/golden/engine_tokens.npz: the first position of
fixture sequence 0 (its whole prompt as one chunk) and the next position (one
decode token), top-16 logits within 1e-4 of the largest."""

from pathlib import Path

import numpy as np
import torch

from batchstream_inference_engine_b200.serve import engine_workload
from batchstream_inference_engine_b200.torch_model import QWEN25_05B, random_weights
from oracle.engine import cpu_backend

GOLDEN = Path(__file__).resolve().parent / "golden" / "engine_tokens.npz"


def test_oracle_model_step_matches_reference_logits():
    g = np.load(GOLDEN)
    seq = int(g["logit_seqs"][0])
    prompt = engine_workload()[seq][0]
    first_token = int(g["tokens_fp32"][g["offsets_fp32"][seq]])
    backend = cpu_backend(random_weights(), torch.float32, QWEN25_05B, 256, 16, 1024)
    model = backend._model
    cache = backend.pool.new_cache(0)
    for step, feed in enumerate((prompt, [first_token])):
        logits = model.forward_batch([(feed, cache)])[0]
        ids = torch.from_numpy(g["logit_ids"][0, step]).long()
        ref = torch.from_numpy(g["logit_values"][0, step])
        assert (logits[ids] - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()
        assert int(logits.argmax()) == int(ids[0])


def test_oracle_backend_reproduces_the_reference_token_streams():
    """The restated reference backend and admission loop (the engine's CPU
    baseline) give the reference's own fp32 greedy tokens: the first 3 tokens
    of the first 4 fixture sequences, 4 concurrent."""
    from oracle.engine import run_for

    g = np.load(GOLDEN)
    specs = [(p, 3) for p, _ in engine_workload()[:4]]
    backend = cpu_backend(random_weights(), torch.float32, QWEN25_05B, 256, 16, 64)
    seen: dict[int, list[int]] = {}
    step = backend.step

    def recording_step():
        out = step()
        for s, (tok, _) in out.items():
            seen.setdefault(s, []).append(tok)
        return out

    backend.step = recording_step
    generated, _, _ = run_for(backend, specs, 4, 256, 16, seconds=600.0, warmup=False)
    assert generated == 12
    for s in range(4):
        start = g["offsets_fp32"][s]
        assert seen[s][:3] == g["tokens_fp32"][start: start + 3].tolist()
