"""Generates tests/golden/engine_margins.npz: for every sequence of the engine
fixture (tests/golden/engine_tokens.npz) and each of its first 32 generated
positions, the reference fp32 model's margin between its best and second-best
logit, relative to the largest |logit|, teacher-forced along the sequence's
own fp32 token stream (the prompt in one forward, then one token per forward).

A greedy fp32 run that differs from the reference only in the last bits of its
GEMMs (another kernel, another summation order) may take the other token where
this margin is within that noise; the engine test accepts a first divergence
only there.

Runs the reference's TorchModel (src/server/torch_model.py) on the CPU with the
same random-init weights as make_engine_golden.py.
Usage: BS_REFERENCE_DIR=<reference checkout> python tests/golden/make_engine_margins.py
"""

import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
if not os.environ.get("BS_REFERENCE_DIR"):
    raise SystemExit("set BS_REFERENCE_DIR to the reference checkout")
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(os.environ["BS_REFERENCE_DIR"]) / "src"))

from batchstream_inference_engine_b200.serve import engine_workload  # noqa: E402
from batchstream_inference_engine_b200.torch_model import random_weights  # noqa: E402
from tests.golden.make_engine_golden import (BLOCK_SIZE, NUM_BLOCKS,  # noqa: E402
                                             _stub_llama_cpp)

STEPS = 32


def main():
    _stub_llama_cpp()
    from server.torch_model import ModelConfig, PagedKVPool, TorchModel

    g = np.load(ROOT / "tests" / "golden" / "engine_tokens.npz")
    offsets = g["offsets_fp32"]
    tokens = [g["tokens_fp32"][offsets[i]: offsets[i + 1]].tolist() for i in range(len(offsets) - 1)]
    config = ModelConfig(num_layers=24, hidden_size=896, num_heads=14, num_kv_heads=2,
                         rope_theta=1_000_000.0, rms_norm_eps=1e-6)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    model = TorchModel(config, random_weights())
    specs = engine_workload()
    margins = np.full((len(specs), STEPS), np.inf, dtype=np.float32)
    with torch.inference_mode():
        for s, (prompt, _) in enumerate(specs):
            pool = PagedKVPool(config, NUM_BLOCKS, BLOCK_SIZE)
            pool.keys = torch.zeros_like(pool.keys, dtype=torch.float32)
            pool.values = torch.zeros_like(pool.values, dtype=torch.float32)
            cache = pool.new_cache(0)
            feed = list(prompt)
            for step in range(min(STEPS, len(tokens[s]))):
                logits = model.forward_batch([(feed, cache)])[0].float()
                top = torch.topk(logits, 2).values
                margins[s, step] = float((top[0] - top[1]) / logits.abs().max())
                feed = [tokens[s][step]]
            print(s, float(margins[s].min()), flush=True)
    np.savez_compressed(ROOT / "tests" / "golden" / "engine_margins.npz", margins_fp32=margins)


if __name__ == "__main__":
    main()
