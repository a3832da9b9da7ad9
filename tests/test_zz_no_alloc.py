"""The allocation-free decode entry point against the regular one.

bs_paged_attention_batched_noalloc is for callers that cannot allocate device
memory when they run attention (a host whose GPU memory is already handed out to
a fixed pool, an FFI caller with no allocator of its own, a step that must not
block on an allocation).  It keeps its scratch in one static device array per
GPU instead of a caller-provided workspace.  Here it is called through the C ABI
twice in a row (so the second call runs on whatever the first left in the shared
array) and must match the workspace entry point each time, within the same
tolerance as the other bf16 decode tests.  This file is collected last on
purpose and also passes on its own in a fresh process.
"""

import math

import numpy as np
import pytest
import torch

from batchstream_inference_engine_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def ragged(num_seqs, heads, kv_heads, head_dim, seed, median=400.0, dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    lens = np.clip(np.rint(rng.lognormal(math.log(median), 1.0, num_seqs)), 1, 8192).astype(int)
    need = [-(-int(n) // 16) for n in lens]
    nb = sum(need) + 8
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed)).to(torch.int32)
    bt = torch.full((num_seqs, max(need)), -1, dtype=torch.int32)
    cur = 0
    for i, m in enumerate(need):
        bt[i, :m] = perm[cur: cur + m]
        cur += m
    g = torch.Generator(device=DEV).manual_seed(seed)
    k = torch.randn((kv_heads, nb, 16, head_dim), generator=g, device=DEV).to(dtype)
    v = torch.randn((kv_heads, nb, 16, head_dim), generator=g, device=DEV).to(dtype)
    q = torch.randn((num_seqs, heads, head_dim), generator=g, device=DEV).to(dtype)
    lens_d = torch.tensor(lens.tolist(), dtype=torch.int32, device=DEV)
    return q, k, v, bt.to(DEV), lens_d


def call_noalloc(q, k, v, bt, lens, scale, out, status, seq_rows=None):
    B, H, D = q.shape
    Hkv, NB, bs, _ = k.shape
    code = _lib.BS_BF16 if q.dtype == torch.bfloat16 else _lib.BS_F32
    return _lib.lib().bs_paged_attention_batched_noalloc(
        q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), bt.data_ptr(), bt.stride(0),
        bt.size(0), seq_rows.data_ptr() if seq_rows is not None else None, lens.data_ptr(), B,
        H, Hkv, D, bs, NB, bt.size(1), code, scale, out.data_ptr(), out.stride(0),
        status.data_ptr() if status is not None else None,
        torch.cuda.current_stream().cuda_stream)


def close(out, ref):
    """The decode tests' bounds: max-abs 1e-4 for fp32; for bf16 the
    reference C++ op's 0.01 plus one bf16 step of the value."""
    err = (out.float() - ref.float()).abs()
    if out.dtype == torch.float32:
        return err.max().item() <= 1e-4
    return bool((err <= 0.01 + 2.0 ** -7 * ref.float().abs()).all())


# Tensor-core shapes (bf16, head_dim 64 / 128) and SIMT shapes (fp32, and a
# head_dim the tensor-core kernel does not take), all in one process: each
# shape must get its own grid, whatever ran before it.
SHAPES = [(14, 2, 64, torch.bfloat16), (28, 4, 128, torch.bfloat16),
          (14, 2, 64, torch.float32), (14, 2, 96, torch.float32), (32, 2, 32, torch.bfloat16)]


@pytest.mark.parametrize("heads,kv_heads,head_dim,dtype", SHAPES)
def test_noalloc_matches_the_workspace_entry_point_twice_in_a_row(heads, kv_heads, head_dim,
                                                                   dtype):
    scale = head_dim ** -0.5
    q, k, v, bt, lens = ragged(96, heads, kv_heads, head_dim, seed=head_dim, dtype=dtype)
    ref = ops.paged_attention_batched(q, k, v, bt, lens, scale)
    assert ops.take_status() == 0
    before = ops.kernel_launches()
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        rc = call_noalloc(q, k, v, bt, lens, scale, out, status)
        assert rc == 0, _lib.lib().bs_last_error().decode()
        torch.cuda.synchronize()
        assert status.item() == 0
        assert not out.isnan().any()
        assert close(out, ref)
    assert ops.kernel_launches() - before == 2  # its launches are counted too


def test_noalloc_with_sequence_rows():
    """Sequences that read their table through seq_rows (several sequences
    sharing one row, as the tokens of a prompt chunk do)."""
    q, k, v, bt, lens = ragged(24, 14, 2, 64, seed=5, median=300.0)
    rows = torch.arange(24, dtype=torch.int32, device=DEV).flip(0) % 12
    lens = lens[rows.long()].contiguous()  # a sequence's length must fit the row it reads
    ref = ops.paged_attention_batched(q, k, v, bt, lens, 0.125, seq_rows=rows)
    assert ops.take_status() == 0
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        assert call_noalloc(q, k, v, bt, lens, 0.125, out, status, seq_rows=rows) == 0
        torch.cuda.synchronize()
        assert status.item() == 0
        assert close(out, ref)


def test_noalloc_requires_a_status_word():
    q, k, v, bt, lens = ragged(4, 14, 2, 64, seed=3)
    out = torch.empty_like(q)
    assert call_noalloc(q, k, v, bt, lens, 0.125, out, None) != 0
    assert b"device_status" in _lib.lib().bs_last_error()


def test_noalloc_after_a_wait_that_ran_out_the_next_call_is_correct():
    """The shared array's per-segment counters survive a launch whose wait gave
    up (test hook: one warp waits on stages that nothing fills, 200 us limit):
    the warp walks the rest of its span without data, so every counter the
    launch touched returns to zero and the next call merges correctly."""
    q, k, v, bt, lens = ragged(96, 14, 2, 64, seed=17, median=800.0)
    ref = ops.paged_attention_batched(q, k, v, bt, lens, 0.125)
    assert ops.take_status() == 0
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.empty_like(ref)
    ops.set_wait_probe(True, 200_000)
    try:
        assert call_noalloc(q, k, v, bt, lens, 0.125, out, status) == 0
        torch.cuda.synchronize()
    finally:
        ops.set_wait_probe(False, 0)
    assert status.item() & 0x4  # BS_STATUS_WAIT_TIMEOUT
    for _ in range(2):
        status.zero_()
        out = torch.full_like(ref, float("nan"))
        assert call_noalloc(q, k, v, bt, lens, 0.125, out, status) == 0
        torch.cuda.synchronize()
        assert status.item() == 0
        assert close(out, ref)


def test_noalloc_rejects_a_batch_beyond_its_limit_with_a_message():
    q, k, v, bt, lens = ragged(4, 14, 2, 64, seed=3)
    big = 16384 // 2 + 1  # (sequence, kv head) pairs over the limit
    out = torch.empty((big, 14, 64), dtype=torch.bfloat16, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib = _lib.lib()
    rc = lib.bs_paged_attention_batched_noalloc(
        q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), bt.data_ptr(), bt.stride(0),
        bt.size(0), None, lens.data_ptr(), big, 14, 2, 64, 16, k.size(1), bt.size(1),
        _lib.BS_BF16, 0.125, out.data_ptr(), out.stride(0), status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"16384" in lib.bs_last_error()
