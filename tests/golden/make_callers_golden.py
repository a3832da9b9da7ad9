"""Generates tests/golden/reference_callers.npz: what the reference's own callers
hand to the attention op and to the backend, recorded while they run unchanged.

Two recordings, both made here on the CPU by the reference itself (its sources
are read from the checkout given by --reference or BS_REFERENCE_DIR; its
compiled C++ op from baseline/_ref, the reference's own setup.py build, or
oracle/_ref):

* op calls -- the reference TorchModel (src/server/torch_model.py) over its own
  PagedKVPool / PagedKVCache with the reference C++ op injected through
  ``attention=`` (torch_model.py:116-119) and wrapped in a recorder: for every
  call, the query exactly as PagedKVCache.attend passes it (a view of the step's queries,
  :155-164), the blocks the table names from the layer view of the pool (a
  view into the 5-D pool tensor), the table (a list of ints), the length, block
  size, groups and scaling, and the op's output.  Model: 2 layers of the
  Qwen2.5-0.5B attention shape (hidden 896, 14 / 2 heads, head_dim 64), bf16
  random weights (seed 0) over a 2048-token vocabulary, 3 prompts of 7, 23 and
  40 tokens and 5 greedy decode steps;

* scheduler trace -- the reference BatchingScheduler (src/server/scheduler.py:
  112-158) with its BlockBudget (src/server/kv_budget.py) driving the
  reference PagedBackend (src/server/backend/paged.py) on the engine workload of
  tests/golden/engine_tokens.npz (fp32, 24 prompts, 8 concurrent, 256 blocks of
  16, prefill chunk 64): the ordered backend calls (start_sequence with its
  prompt and returned id, step with its {seq_id: (token, finished)} outputs,
  release_sequence with its id).

Usage: python tests/golden/make_callers_golden.py --reference <checkout>
(a few minutes on 8 cores).
"""

import argparse
import asyncio
import os
import sys
import types
from itertools import count
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from batchstream_inference_engine_b200.serve import engine_workload  # noqa: E402
from batchstream_inference_engine_b200.torch_model import random_weights  # noqa: E402
from tests.golden import inputs  # noqa: E402

EOG = (151643, 151645)


def _stub_llama_cpp():
    """paged.py imports llama_cpp at module level; nothing on this path uses it."""
    stub = types.ModuleType("llama_cpp")
    stub.llama_backend_init = lambda: None
    sys.modules.setdefault("llama_cpp", stub)


def reference_op():
    """The reference's compiled op: its own setup.py build if installed in
    baseline/_ref, else the build of oracle/_ref."""
    installed = ROOT / "baseline" / "_ref"
    if (installed / "server").is_dir() and list((installed / "server").glob("paged_attention_cpp*.so")):
        import importlib.machinery
        import importlib.util

        so = sorted((installed / "server").glob("paged_attention_cpp*.so"))[0]
        loader = importlib.machinery.ExtensionFileLoader("paged_attention_cpp", str(so))
        spec = importlib.util.spec_from_loader("paged_attention_cpp", loader)
        module = importlib.util.module_from_spec(spec)
        loader.exec_module(module)
        return module.paged_attention, "baseline/_ref"
    import oracle

    op = oracle.load_reference_op()
    if op is None:
        raise SystemExit("no compiled reference op (build oracle/_ref first)")
    return op, "oracle/_ref"


def record_op_calls(op):
    from server.torch_model import ModelConfig, PagedKVPool, TorchModel

    config = ModelConfig(num_layers=2, hidden_size=896, num_heads=14, num_kv_heads=2,
                         rope_theta=1_000_000.0, rms_norm_eps=1e-6)
    weights = {k: v.bfloat16() for k, v in random_weights(
        config, vocab_size=2048, intermediate_size=512).items()}
    calls = []

    def recorder(query, keys, values, table, length, block_size, groups, scaling):
        out = op(query, keys, values, table, length, block_size, groups, scaling)
        need = -(-length // block_size)
        rows = torch.tensor(table[:need], dtype=torch.long)
        calls.append(dict(
            q_shape=list(query.shape), q_stride=list(query.stride()),
            q_offset=query.storage_offset(), q=inputs.bf16_bits(query.contiguous()),
            pool_shape=list(keys.shape), pool_offset=keys.storage_offset(),
            pool_stride=list(keys.stride()), table=list(table), length=int(length),
            block_size=int(block_size), groups=int(groups), scaling=float(scaling),
            k_blocks=inputs.bf16_bits(keys.index_select(1, rows).contiguous()),
            v_blocks=inputs.bf16_bits(values.index_select(1, rows).contiguous()),
            out=inputs.bf16_bits(out.contiguous())))
        return out

    model = TorchModel(config, weights)
    pool = PagedKVPool(config, 64, 16, attention=recorder)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 2048, (n,), generator=g).tolist() for n in (7, 23, 40)]
    caches = [pool.new_cache(i) for i in range(len(prompts))]
    logits = model.forward_batch(list(zip(prompts, caches)))
    for _ in range(5):
        nxt = logits.float().argmax(-1).tolist()
        logits = model.forward_batch([([t], c) for t, c in zip(nxt, caches)])
    return calls


class RecordingBackend:
    """Forwards to the reference PagedBackend and records every call."""

    def __init__(self, inner, events):
        self.inner = inner
        self.events = events

    def start_sequence(self, prompt_tokens):
        seq_id = self.inner.start_sequence(prompt_tokens)
        self.events.append(("start", seq_id, list(prompt_tokens)))
        return seq_id

    def step(self):
        outputs = self.inner.step()
        self.events.append(("step", {s: (o.token, o.finished) for s, o in outputs.items()}))
        return outputs

    def release_sequence(self, seq_id):
        self.inner.release_sequence(seq_id)
        self.events.append(("release", seq_id))


def record_scheduler_trace():
    _stub_llama_cpp()
    from server.backend.paged import PagedBackend
    from server.kv_budget import BlockBudget
    from server.scheduler import BatchingScheduler
    from server.torch_model import ModelConfig, PagedKVPool, TorchModel

    class Ids:
        def is_end_of_generation(self, token):
            return token in EOG

    config = ModelConfig(num_layers=24, hidden_size=896, num_heads=14, num_kv_heads=2,
                         rope_theta=1_000_000.0, rms_norm_eps=1e-6)
    backend = PagedBackend.__new__(PagedBackend)
    backend._model = TorchModel(config, random_weights())
    backend._pool = PagedKVPool(config, 256, 16)
    backend._pool.keys = torch.zeros_like(backend._pool.keys, dtype=torch.float32)
    backend._pool.values = torch.zeros_like(backend._pool.values, dtype=torch.float32)
    backend._num_blocks = 256
    backend._prefill_chunk = 64
    backend._vocab = Ids()
    backend._ids = count()
    backend._sequences = {}
    events = []
    scheduler = BatchingScheduler(RecordingBackend(backend, events), 8, BlockBudget(256, 16),
                                  max_queue=1024)

    async def serve():
        loop_task = asyncio.create_task(scheduler.run())
        requests = [scheduler.submit(p, m) for p, m in engine_workload()]
        await asyncio.gather(*(r.done.wait() for r in requests))
        loop_task.cancel()
        return requests

    requests = asyncio.run(serve())
    assert not any(r.failed for r in requests)
    return events


def pack_calls(calls):
    out = {"n_calls": np.int64(len(calls))}
    for i, c in enumerate(calls):
        for key, val in c.items():
            out[f"c{i}_{key}"] = np.asarray(val)
    return out


def pack_events(events):
    """Flat int64 rows: kind (0 start, 1 step, 2 release), id or n, payload."""
    flat = []
    for ev in events:
        if ev[0] == "start":
            flat += [0, ev[1], len(ev[2])] + ev[2]
        elif ev[0] == "step":
            flat += [1, len(ev[1])]
            for s, (tok, fin) in sorted(ev[1].items()):
                flat += [s, tok, int(fin)]
        else:
            flat += [2, ev[1]]
    return np.asarray(flat, dtype=np.int64)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--reference", default=os.environ.get("BS_REFERENCE_DIR"),
                   help="checkout of the reference (its src/ holds the server package)")
    args = p.parse_args()
    if not args.reference:
        raise SystemExit("give the reference checkout with --reference or BS_REFERENCE_DIR")
    sys.path.insert(0, str(Path(args.reference) / "src"))
    torch.set_num_threads(os.cpu_count() or 8)
    op, source = reference_op()
    calls = record_op_calls(op)
    print(f"{len(calls)} op calls recorded (reference op from {source})")
    events = record_scheduler_trace()
    print(f"{len(events)} backend calls recorded")
    np.savez_compressed(Path(__file__).with_name("reference_callers.npz"),
                        events=pack_events(events), **pack_calls(calls))


if __name__ == "__main__":
    main()
