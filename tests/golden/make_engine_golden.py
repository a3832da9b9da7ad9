"""Generates tests/golden/engine_tokens.npz: greedy token ids of the reference's
paged backend on the random-init Qwen2.5-0.5B-shaped model.

Runs the reference itself (src/server/torch_model.py TorchModel + PagedKVPool,
src/server/backend/paged.py PagedBackend, src/server/scheduler.py
BatchingScheduler, src/server/kv_budget.py BlockBudget) on the CPU:

* weights: ``random_weights`` of this package (seed 0, N(0, 0.02), RMSNorm 1),
  identical on both sides;
* workload: ``engine_workload`` (24 token-id prompts, lengths U[4, 277],
  max_tokens U[16, 128], seed 0), all queued at once, max 8 concurrent,
  BlockBudget(256 blocks, block 16), prefill_chunk 64;
* fp32 run: weights fp32 and the pool tensors reassigned to fp32 (the reference
  hard-codes bf16 pools, torch_model.py:121-122); bf16 run: weights bf16, the
  reference's bf16 pool.  Both use the reference's default Python attention op.
* vocabulary: token ids only; end of generation = Qwen2.5's 151643 / 151645
  (the GGUF vocabulary and llama.cpp are not on this path).

Usage: BS_REFERENCE_DIR=<reference checkout> python tests/golden/make_engine_golden.py
(takes a few minutes on 8 cores).
"""

import asyncio
import os
import sys
import time
import types
from itertools import count
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

NUM_BLOCKS = 256
BLOCK_SIZE = 16
PREFILL_CHUNK = 64
MAX_CONCURRENT = 8
EOG = (151643, 151645)


def _stub_llama_cpp():
    """paged.py and llamacpp.py import llama_cpp at module level; neither the
    model nor the attention path uses it."""
    stub = types.ModuleType("llama_cpp")
    stub.llama_backend_init = lambda: None
    sys.modules.setdefault("llama_cpp", stub)


class _Ids:
    def is_end_of_generation(self, token: int) -> bool:
        return token in EOG


def reference_backend(dtype: torch.dtype):
    _stub_llama_cpp()
    from server.backend.paged import PagedBackend
    from server.torch_model import ModelConfig, PagedKVPool, TorchModel

    config = ModelConfig(num_layers=24, hidden_size=896, num_heads=14, num_kv_heads=2,
                         rope_theta=1_000_000.0, rms_norm_eps=1e-6)
    weights = {k: v.to(dtype) for k, v in random_weights().items()}
    backend = PagedBackend.__new__(PagedBackend)
    backend._model = TorchModel(config, weights)
    backend._pool = PagedKVPool(config, NUM_BLOCKS, BLOCK_SIZE)
    if dtype == torch.float32:
        backend._pool.keys = torch.zeros_like(backend._pool.keys, dtype=torch.float32)
        backend._pool.values = torch.zeros_like(backend._pool.values, dtype=torch.float32)
    backend._num_blocks = NUM_BLOCKS
    backend._prefill_chunk = PREFILL_CHUNK
    backend._vocab = _Ids()
    backend._ids = count()
    backend._sequences = {}
    return backend


def run(dtype: torch.dtype) -> list[list[int]]:
    from server.kv_budget import BlockBudget
    from server.scheduler import BatchingScheduler

    backend = reference_backend(dtype)
    scheduler = BatchingScheduler(backend, MAX_CONCURRENT, BlockBudget(NUM_BLOCKS, BLOCK_SIZE),
                                  max_queue=1024)

    async def serve():
        loop_task = asyncio.create_task(scheduler.run())
        requests = [scheduler.submit(p, m) for p, m in engine_workload()]
        await asyncio.gather(*(r.done.wait() for r in requests))
        loop_task.cancel()
        return requests

    requests = asyncio.run(serve())
    assert not any(r.failed for r in requests)
    return [list(r.tokens) for r in requests]


LOGIT_SEQS = (0, 1, 2, 3)
LOGIT_STEPS = 32
TOPK = 16


def teacher_forced_logits(fp32_tokens):
    """Reference fp32 last-token logits along each sequence's own fp32 token
    stream: the prompt in one forward, then one token per forward.  Keeps the
    top-16 ids and values of each of the first 32 positions."""
    _stub_llama_cpp()
    from server.torch_model import ModelConfig, PagedKVPool, TorchModel

    config = ModelConfig(num_layers=24, hidden_size=896, num_heads=14, num_kv_heads=2,
                         rope_theta=1_000_000.0, rms_norm_eps=1e-6)
    model = TorchModel(config, random_weights())
    specs = engine_workload()
    ids = np.zeros((len(LOGIT_SEQS), LOGIT_STEPS, TOPK), dtype=np.int32)
    vals = np.zeros((len(LOGIT_SEQS), LOGIT_STEPS, TOPK), dtype=np.float32)
    for n, s in enumerate(LOGIT_SEQS):
        pool = PagedKVPool(config, NUM_BLOCKS, BLOCK_SIZE)
        pool.keys = torch.zeros_like(pool.keys, dtype=torch.float32)
        pool.values = torch.zeros_like(pool.values, dtype=torch.float32)
        cache = pool.new_cache(0)
        feed = list(specs[s][0])
        for step in range(LOGIT_STEPS):
            logits = model.forward_batch([(feed, cache)])[0].float()
            top = torch.topk(logits, TOPK)
            ids[n, step], vals[n, step] = top.indices.numpy(), top.values.numpy()
            feed = [fp32_tokens[s][step]]
    return ids, vals


def reference_bf16_logit_error(fp32_tokens, ids, vals):
    """How far the reference's own bf16 model (bf16 weights and pool) is from
    its fp32 logits along the same teacher-forced streams: per position,
    max |bf16 - fp32| over the top-16 ids / max |fp32|."""
    _stub_llama_cpp()
    from server.torch_model import ModelConfig, PagedKVPool, TorchModel

    config = ModelConfig(num_layers=24, hidden_size=896, num_heads=14, num_kv_heads=2,
                         rope_theta=1_000_000.0, rms_norm_eps=1e-6)
    model = TorchModel(config, {k: v.bfloat16() for k, v in random_weights().items()})
    specs = engine_workload()
    err = np.zeros(ids.shape[:2], dtype=np.float32)
    for n, s in enumerate(LOGIT_SEQS):
        pool = PagedKVPool(config, NUM_BLOCKS, BLOCK_SIZE)
        cache = pool.new_cache(0)
        feed = list(specs[s][0])
        for step in range(LOGIT_STEPS):
            logits = model.forward_batch([(feed, cache)])[0].float()
            ref = torch.from_numpy(vals[n, step])
            got = logits[torch.from_numpy(ids[n, step]).long()]
            err[n, step] = ((got - ref).abs().max() / ref.abs().max()).item()
            feed = [fp32_tokens[s][step]]
    return err


def pack(lists):
    offsets = np.concatenate([[0], np.cumsum([len(x) for x in lists])]).astype(np.int64)
    return np.concatenate([np.asarray(x, dtype=np.int32) for x in lists]), offsets


def main():
    torch.set_num_threads(8)
    specs = engine_workload()
    out = {}
    prompts, prompt_off = pack([p for p, _ in specs])
    out.update(prompts=prompts, prompt_offsets=prompt_off,
               max_tokens=np.asarray([m for _, m in specs], dtype=np.int32))
    tokens_by = {}
    for name, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        t0 = time.time()
        tokens_by[name] = run(dtype)
        print(f"{name}: {sum(map(len, tokens_by[name]))} tokens in {time.time() - t0:.0f} s")
        out[f"tokens_{name}"], out[f"offsets_{name}"] = pack(tokens_by[name])
    t0 = time.time()
    out["logit_seqs"] = np.asarray(LOGIT_SEQS, dtype=np.int32)
    out["logit_ids"], out["logit_values"] = teacher_forced_logits(tokens_by["fp32"])
    out["ref_bf16_logit_err"] = reference_bf16_logit_error(tokens_by["fp32"], out["logit_ids"],
                                                           out["logit_values"])
    print(f"teacher-forced logits in {time.time() - t0:.0f} s")
    np.savez_compressed(Path(__file__).with_name("engine_tokens.npz"), **out)


if __name__ == "__main__":
    main()
