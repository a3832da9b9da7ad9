"""The reference's callers, unchanged, on this path.

The reference's Python package cannot travel to the GPU machine (its setup.py
installs only the compiled op, and its sources are not vendored here), so what
its callers do was recorded where they run (tests/golden/make_callers_golden.py)
and is replayed here against this package:

* the reference's op tests (tests/test_paged_attention.py:161-202 of the
  reference), which call the op on host tensors, run with this package's op in
  its place, against the reference C++ op's recorded outputs;
* every call that the reference's PagedKVPool / PagedKVCache.attend made to its
  injected op (src/server/torch_model.py:116-119, 155-164) is made again, with
  the same argument forms -- host tensors, the query as the same view,
  the pool as the layer view of a 5-D tensor, the table as a list of ints --
  through ``paged_attention_cuda.paged_attention``, and must give the reference
  op's output;
* the ordered backend calls that the reference's BatchingScheduler
  (src/server/scheduler.py:112-158) made to the reference PagedBackend drive
  this package's PagedBackend, which must answer every step with the same
  sequences, finished flags and (for each sequence's first 32 tokens, the
  stated greedy bound) the same tokens.

Bounds: bf16 element-wise within 0.01 + 2**-7 |cpp| of the reference C++ op
(its CPP_TOLERANCE plus one bf16 step), as in the other decode tests.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from batchstream_inference_engine_b200.paged_attention_cuda import paged_attention
from tests.golden import inputs
from tests.test_decode_gpu import cpp_close

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def golden(name):
    return np.load(GOLDEN / name)


# ------------------------------------------------------------------ the reference's op tests


@pytest.mark.parametrize("length", inputs.SCATTERED_LENGTHS)
def test_reference_op_test_scattered_blocks_on_host_tensors(length):
    """tests/test_paged_attention.py:176-186: the op on the host tensors of
    bf16_attention_inputs, against the reference C++ op's output."""
    gold = golden("decode_scattered.npz")
    query, keys, values, table = inputs.scattered_bf16(length, seed=length)
    actual = paged_attention(query, keys, values, table, length, 4, 2, 8 ** -0.5)
    assert actual.dtype == torch.bfloat16 and actual.shape == (4, 8) and not actual.is_cuda
    assert cpp_close(actual, inputs.from_bits(gold[f"cpp_{length}"]).float())


def test_reference_op_test_non_contiguous_query_on_host_tensors():
    """tests/test_paged_attention.py:189-196."""
    query, keys, values, table = inputs.scattered_bf16(5)
    strided = torch.zeros(4, 3, 8, dtype=torch.bfloat16)
    strided[:, 1] = query
    actual = paged_attention(strided[:, 1], keys, values, table, 5, 4, 2, 0.5)
    assert torch.equal(actual, paged_attention(query, keys, values, table, 5, 4, 2, 0.5))


def test_reference_op_test_never_reads_past_length_on_host_tensors():
    """tests/test_paged_attention.py:199-202: unused slots hold NaN."""
    query, keys, values, table = inputs.scattered_bf16(5)
    assert not paged_attention(query, keys, values, table, 5, 4, 2, 0.5).isnan().any()


# ------------------------------------------------------------------ PagedKVPool's calls


def _calls():
    data = golden("reference_callers.npz")
    return [{k[len(f"c{i}_"):]: data[k] for k in data.files if k.startswith(f"c{i}_")}
            for i in range(int(data["n_calls"]))]


def _rebuild(call, layers=2):
    """Host tensors in the forms PagedKVCache.attend passed them: the query as
    the same view of a larger tensor, keys and values as the layer view
    of a zero-initialised 5-D pool holding the sequence's blocks."""
    shape, stride, offset = call["q_shape"].tolist(), call["q_stride"].tolist(), int(call["q_offset"])
    extent = offset + sum((n - 1) * s for n, s in zip(shape, stride)) + 1
    base = torch.zeros(extent, dtype=torch.bfloat16)
    query = base.as_strided(shape, stride, offset)
    query.copy_(inputs.from_bits(call["q"]).view(shape))
    pshape = call["pool_shape"].tolist()
    layer = int(call["pool_offset"]) // int(np.prod(pshape))
    need = -(-int(call["length"]) // int(call["block_size"]))
    table = [int(t) for t in call["table"].tolist()]
    pools = []
    for name in ("k_blocks", "v_blocks"):
        pool = torch.zeros([max(layers, layer + 1)] + pshape, dtype=torch.bfloat16)
        blocks = inputs.from_bits(call[name]).view(pshape[0], need, *pshape[2:])
        pool[layer][:, torch.tensor(table[:need])] = blocks
        view = pool[layer]
        assert view.storage_offset() == int(call["pool_offset"])
        assert list(view.stride()) == call["pool_stride"].tolist()
        pools.append(view)
    return query, pools[0], pools[1], table


def test_every_call_of_the_reference_pool_gives_the_reference_op_output():
    calls = _calls()
    assert len(calls) == 30  # 2 layers x 3 sequences x 5 decode steps
    views = 0
    for i, call in enumerate(calls):
        query, keys, values, table = _rebuild(call)
        views += query.storage_offset() > 0
        out = paged_attention(query, keys, values, table, int(call["length"]),
                              int(call["block_size"]), int(call["groups"]),
                              float(call["scaling"]))
        assert out.dtype == torch.bfloat16 and not out.is_cuda
        ref = inputs.from_bits(call["out"]).view(out.shape).float()
        assert cpp_close(out, ref), i
    # The reference passes queries[:, 0] of the step's [heads, tokens, head_dim]
    # queries: for every sequence but the first, a view at an offset.
    assert views == 20


# ------------------------------------------------------------------ BatchingScheduler's calls


def _events():
    flat = golden("reference_callers.npz")["events"].tolist()
    events, i = [], 0
    while i < len(flat):
        kind = flat[i]
        if kind == 0:
            n = flat[i + 2]
            events.append(("start", flat[i + 1], flat[i + 3: i + 3 + n]))
            i += 3 + n
        elif kind == 1:
            n = flat[i + 1]
            rows = flat[i + 2: i + 2 + 3 * n]
            events.append(("step", {rows[j]: (rows[j + 1], bool(rows[j + 2]))
                                    for j in range(0, 3 * n, 3)}))
            i += 2 + 3 * n
        else:
            events.append(("release", flat[i + 1]))
            i += 2
    return events


def test_the_reference_schedulers_backend_calls_replay_on_this_backend():
    from batchstream_inference_engine_b200.backend import PagedBackend
    from batchstream_inference_engine_b200.torch_model import (QWEN25_05B, TorchModel,
                                                              random_weights)

    model = TorchModel(QWEN25_05B, random_weights(), device="cuda:0", dtype=torch.float32)
    backend = PagedBackend(model, 256, 16, 64, max_seqs=64)
    events = _events()
    assert sum(e[0] == "start" for e in events) == 24
    produced = {}
    steps = 0
    for ev in events:
        if ev[0] == "start":
            assert backend.start_sequence(ev[2]) == ev[1]
        elif ev[0] == "release":
            backend.release_sequence(ev[1])
        else:
            steps += 1
            got = backend.step()
            assert sorted(got) == sorted(ev[1]), steps
            for seq, (token, finished) in ev[1].items():
                assert got[seq].finished == finished, (steps, seq)
                n = produced.get(seq, 0)
                if n < 32:
                    assert got[seq].token == token, (steps, seq, n)
                produced[seq] = n + 1
    assert len(produced) == 24
