"""Seeded input recipes shared by the golden-fixture generator and the tests.

Every recipe draws from a ``torch.Generator`` on the CPU in a fixed order, so
the same torch build regenerates identical tensors on any machine; fixtures
store outputs plus a digest of the inputs that produced them.
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch


def digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()[:16]


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 numpy array of its bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def scattered_bf16(length: int, block_size: int = 4, seed: int = 0):
    """The scattered-block bf16 case of the reference's op tests
    (tests/test_paged_attention.py:161-173): 2 kv heads, 4 query heads, head_dim 8,
    ceil(L/bs) + 3 blocks of which a random subset holds the sequence, every other
    slot NaN.  Returns (query [4, 8], keys, values [2, NB, bs, 8], table)."""
    g = torch.Generator().manual_seed(seed)
    needed = -(-length // block_size)
    num_blocks = needed + 3
    table = torch.randperm(num_blocks, generator=g)[:needed].tolist()
    keys = torch.full((2, num_blocks, block_size, 8), float("nan"), dtype=torch.bfloat16)
    values = torch.full((2, num_blocks, block_size, 8), float("nan"), dtype=torch.bfloat16)
    for pos in range(length):
        blk, off = table[pos // block_size], pos % block_size
        keys[:, blk, off] = torch.randn(2, 8, generator=g).to(torch.bfloat16)
        values[:, blk, off] = torch.randn(2, 8, generator=g).to(torch.bfloat16)
    query = torch.randn(4, 8, generator=g).to(torch.bfloat16)
    return query, keys, values, table


def scattered_f32(length: int):
    """The fp32 scattered-block case of tests/test_paged_attention.py:31-53:
    table [9, 2, 14, 0] prefix, block size 4, 16 blocks, head_dim 4, 2 kv heads,
    4 query heads, NaN in unused slots.  Returns (query, keys, values, table,
    contiguous keys, contiguous values)."""
    table = [9, 2, 14, 0][: -(-length // 4)]
    g = torch.Generator().manual_seed(0)
    keys = torch.randn(2, length, 4, generator=g)
    values = torch.randn(2, length, 4, generator=g)
    pool_k = torch.full((2, 16, 4, 4), float("nan"))
    pool_v = torch.full((2, 16, 4, 4), float("nan"))
    for pos in range(length):
        pool_k[:, table[pos // 4], pos % 4] = keys[:, pos]
        pool_v[:, table[pos // 4], pos % 4] = values[:, pos]
    query = torch.randn(4, 4, generator=g)
    return query, pool_k, pool_v, table, keys, values


def op_level_batch(seed: int = 0):
    """The op-level decode batch: 8 sequences, 14 query / 2 kv heads, head_dim 64,
    block size 16, a 256-block pool, lengths uniform in [4, 341], disjoint random
    tables (sequential slices of one permutation), N(0,1) fp32, scale 1/8.
    Returns (lengths, tables, query [8, 14, 64], keys, values [2, 256, 16, 64])."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(4, 342, (8,), generator=g).tolist()
    perm = torch.randperm(256, generator=g).tolist()
    tables, cursor = [], 0
    for length in lengths:
        need = -(-length // 16)
        tables.append(perm[cursor: cursor + need])
        cursor += need
    query = torch.randn(8, 14, 64, generator=g)
    keys = torch.randn(2, 256, 16, 64, generator=g)
    values = torch.randn(2, 256, 16, 64, generator=g)
    return lengths, tables, query, keys, values


def prefill_case(n: int, past: int, heads: int = 14, kv_heads: int = 2, head_dim: int = 64,
                 block_size: int = 16, seed: int = 0):
    """One prefill chunk of n tokens after `past` cached ones, paged over a
    shuffled pool with NaN in every unused slot.  Returns (query [n, H, D],
    keys, values [Hkv, NB, bs, D], table) in fp32."""
    g = torch.Generator().manual_seed(seed)
    total = past + n
    need = -(-total // block_size)
    num_blocks = need + 5
    table = torch.randperm(num_blocks, generator=g)[:need].tolist()
    keys = torch.full((kv_heads, num_blocks, block_size, head_dim), float("nan"))
    values = torch.full((kv_heads, num_blocks, block_size, head_dim), float("nan"))
    k = torch.randn(kv_heads, total, head_dim, generator=g)
    v = torch.randn(kv_heads, total, head_dim, generator=g)
    for pos in range(total):
        keys[:, table[pos // block_size], pos % block_size] = k[:, pos]
        values[:, table[pos // block_size], pos % block_size] = v[:, pos]
    query = torch.randn(n, heads, head_dim, generator=g)
    return query, keys, values, table


# (n, past, heads, kv_heads); head_dim 64, block size 16.
PREFILL_CASES = [(1, 0, 4, 2), (5, 0, 4, 2), (16, 0, 4, 2), (17, 3, 4, 2), (33, 15, 4, 2),
                 (40, 16, 4, 2), (24, 9, 14, 2)]
SCATTERED_LENGTHS = [1, 3, 4, 5, 8, 9, 15, 16, 17, 100, 1000]
F32_LENGTHS = [1, 3, 4, 5, 8, 9, 15]


def mixed_step_shapes():
    """The mixed chunked-prefill + decode step of one GPU, all from
    ``np.random.default_rng(0)``: 8 chunk priors U[0, 4096], then 248 decode
    context lengths log-normal (median 768, sigma 1), rounded and clipped to
    [16, 8192] (each counting the step's new token)."""
    import math

    rng = np.random.default_rng(0)
    priors = rng.integers(0, 4097, 8).astype(np.int64)
    lens = np.clip(np.rint(rng.lognormal(math.log(768.0), 1.0, 248)), 16, 8192).astype(np.int64)
    return priors, lens
