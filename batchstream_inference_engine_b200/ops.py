"""Torch-facing wrappers of the C ABI: the paged-attention path on CUDA tensors.

PyTorch provides device memory, the current stream and the tensors; every
computation runs in the sm_100a kernels of ``libbatchstream_b200.so``.  Errors
surface as ``RuntimeError``, as the reference op raises them through
``TORCH_CHECK`` (csrc/paged_attention.cpp:22-44).
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from ._lib import BS_BF16, BS_F32, check, i64_array, lib

_DTYPES = {torch.bfloat16: BS_BF16, torch.float32: BS_F32}


def dtype_code(dtype: torch.dtype) -> int:
    """C-ABI dtype code; any other dtype maps to an invalid code the C side rejects."""
    return _DTYPES.get(dtype, -1)


def _stream_of(t: torch.Tensor) -> int:
    if t.is_cuda:
        return torch.cuda.current_stream(t.device).cuda_stream
    return 0


def _require_cuda(name: str, *tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{name}: every tensor must be a CUDA tensor")
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError(f"{name}: tensors are on different devices")
    return device


class _Workspaces:
    """Zero-filled scratch buffers, one per (device, stream), grown on demand.

    The kernels leave the counter region zero after every call, so a buffer is
    zero-filled only when it is (re)allocated.
    """

    def __init__(self):
        self._lock = threading.Lock()
        self._buffers: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
        with self._lock:
            buf = self._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                if buf is not None:
                    size = max(size, 2 * buf.numel())
                fresh = torch.zeros(size, dtype=torch.uint8, device=device)
                if buf is not None:  # keep status bits not yet taken
                    fresh[:4].copy_(buf[:4])
                buf = fresh
                self._buffers[key] = buf
            return buf


_workspaces = _Workspaces()


def workspace_for(device: torch.device, nbytes: int) -> torch.Tensor:
    """The scratch buffer used for calls on the current stream of `device`."""
    return _workspaces.get(device, torch.cuda.current_stream(device).cuda_stream, nbytes)


def take_status(device: torch.device | None = None) -> int:
    """Synchronise the current stream and raise if a kernel set a status bit.

    Returns 0 when no bit was set (kernels never fault on bad tables, lengths or
    slots; they record the problem here instead).
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(device).cuda_stream
    ws = _workspaces.get(device, stream, 0)
    bits = ctypes.c_uint32(0)
    rc = lib().bs_take_status(ws.data_ptr(), stream, ctypes.byref(bits))
    if bits.value:
        # A launch that reported a problem may have left segment counters set:
        # clear them so that the next call on this workspace starts clean.
        check(lib().bs_reset_workspace(ws.data_ptr(), stream))
    check(rc)
    return bits.value


def set_wait_probe(unarmed: bool, wait_limit_ns: int = 0) -> None:
    """Test hook of the bounded-wait error path (bs_set_wait_probe): the wait
    limit of the tensor-core decode kernel (0: the default of about 2 s) and,
    with ``unarmed``, one warp that waits on stages nothing fills."""
    check(lib().bs_set_wait_probe(1 if unarmed else 0, int(wait_limit_ns)))


def decode_workspace_bytes(num_seqs: int, num_heads: int, num_kv_heads: int, head_dim: int,
                           block_size: int, dtype: torch.dtype) -> int:
    """Workspace that ``paged_attention_batched`` needs for this shape."""
    got = ctypes.c_uint64(0)
    check(lib().bs_paged_attention_batched_workspace_bytes(
        num_seqs, num_heads, num_kv_heads, head_dim, block_size, dtype_code(dtype),
        ctypes.byref(got)))
    return got.value


def prefill_workspace_bytes(num_tokens: int, num_rows: int, max_query_len: int, num_heads: int,
                            num_kv_heads: int, head_dim: int, block_size: int,
                            dtype: torch.dtype) -> int:
    """Workspace that ``prefill_attention`` needs for this shape."""
    got = ctypes.c_uint64(0)
    check(lib().bs_prefill_attention_workspace_bytes(
        num_tokens, num_rows, max_query_len, num_heads, num_kv_heads, head_dim, block_size,
        dtype_code(dtype), ctypes.byref(got)))
    return got.value


def kernel_launches() -> int:
    """Kernels this package's library has launched (or recorded into a CUDA
    graph) in this process."""
    return int(lib().bs_kernel_launches())


def _shape_args(t: torch.Tensor):
    return t.dim(), i64_array(t.shape), i64_array(t.stride())


def paged_attention(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                    block_table: list[int], length: int, block_size: int, groups: int,
                    scaling: float) -> torch.Tensor:
    """Drop-in for the reference op ``paged_attention`` (csrc/paged_attention.cpp:76-105).

    Same positional signature and the same malformed-input errors; accepts
    float32 when query, keys and values are all float32.  Returns
    [heads, head_dim] in the query dtype on the query's device.

    The attention always runs in this library's CUDA kernels.  The reference's
    own callers keep the pool on the host (PagedKVPool allocates it with
    torch.zeros, src/server/torch_model.py:120-122): when query, keys and values
    are all host tensors, the inputs are checked as the reference checks them,
    the sequence's blocks (and the query) are staged on the current CUDA device,
    and the result comes back as a host tensor -- so the op drops into those
    callers unchanged.
    """
    if not (query.is_cuda or keys.is_cuda or values.is_cuda):
        return _paged_attention_from_host(query, keys, values, block_table, length, block_size,
                                          groups, scaling)
    if query.dim() == 2:
        query = query.contiguous()  # the reference copies it too (paged_attention.cpp:81)
    table = [int(b) for b in block_table]
    qn, qs, qst = _shape_args(query)
    kn, ks, kst = _shape_args(keys)
    vn, vs, vst = _shape_args(values)
    device = query.device
    stream = _stream_of(query)
    if query.dim() == 2 and query.is_cuda:
        out = torch.empty(query.shape, dtype=query.dtype, device=device)
    else:
        out = torch.empty(0)
    ws_ptr, ws_bytes = 0, 0
    if query.is_cuda and keys.dim() == 4 and query.dim() == 2 and keys.size(0) > 0:
        with torch.cuda.device(device):
            need = ctypes.c_uint64(0)
            check(lib().bs_paged_attention_workspace_bytes(
                query.size(0), keys.size(0), query.size(1), len(table), dtype_code(query.dtype),
                block_size, ctypes.byref(need)))
            ws = workspace_for(device, need.value)
            ws_ptr, ws_bytes = ws.data_ptr(), ws.numel()
    ctx = torch.cuda.device(device) if query.is_cuda else _NullContext()
    with ctx:
        check(lib().bs_paged_attention(
            query.data_ptr(), dtype_code(query.dtype), qn, qs, qst,
            keys.data_ptr(), dtype_code(keys.dtype), kn, ks, kst,
            values.data_ptr(), dtype_code(values.dtype), vn, vs, vst,
            i64_array(table), len(table), int(length), int(block_size), int(groups),
            float(scaling), out.data_ptr(), ws_ptr, ws_bytes, stream))
    return out


def _paged_attention_from_host(query, keys, values, block_table, length, block_size, groups,
                               scaling):
    """paged_attention on host tensors: validate, stage the blocks the table
    names (in table order, so the staged table is 0 .. n - 1) and the query on
    the current device, run the device op, return the output on the host."""
    table = [int(b) for b in block_table]
    qn, qs, qst = _shape_args(query)
    kn, ks, kst = _shape_args(keys)
    vn, vs, vst = _shape_args(values)
    check(lib().bs_paged_attention_check(
        dtype_code(query.dtype), qn, qs, qst, dtype_code(keys.dtype), kn, ks, kst,
        dtype_code(values.dtype), vn, vs, vst, i64_array(table), len(table), int(length),
        int(block_size), int(groups)))
    if not torch.cuda.is_available():
        raise RuntimeError("paged_attention: no CUDA device to run on")
    device = torch.device("cuda", torch.cuda.current_device())
    need = -(-int(length) // int(block_size))
    rows = torch.tensor(table[:need], dtype=torch.long)
    k_dev = keys.index_select(1, rows).to(device, non_blocking=False)
    v_dev = values.index_select(1, rows).to(device, non_blocking=False)
    q_dev = query.contiguous().to(device)
    out = paged_attention(q_dev, k_dev, v_dev, list(range(need)), length, block_size, groups,
                          scaling)
    return out.cpu()


class _NullContext:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_batched_ws_bytes: dict[tuple, int] = {}


def paged_attention_batched(query: torch.Tensor, key_pool: torch.Tensor, value_pool: torch.Tensor,
                            block_tables: torch.Tensor, context_lens: torch.Tensor, scaling: float,
                            seq_rows: torch.Tensor | None = None, out: torch.Tensor | None = None,
                            max_blocks_per_seq: int | None = None,
                            units_hint: int = 0, lens_ready: bool = False,
                            after_append: bool = False) -> torch.Tensor:
    """Decode attention for a whole ragged batch in one launch.

    query [B, H, D]; key_pool/value_pool [Hkv, NB, bs, D] (one layer of the
    pool, contiguous); block_tables int32 [rows, max_blocks]; context_lens int32
    [B]; seq_rows int32 [B] (row of each sequence in block_tables, default b).
    Returns [B, H, D] in the query dtype.  Bad tables or lengths never fault: they
    set a status bit that ``take_status`` raises.
    """
    device = _require_cuda("paged_attention_batched", query, key_pool, value_pool, block_tables,
                           context_lens, seq_rows, out)
    if query.dim() != 3 or key_pool.dim() != 4 or value_pool.shape != key_pool.shape:
        raise RuntimeError("query must be [B, H, D] and the pools [Hkv, NB, bs, D]")
    if query.dtype != key_pool.dtype or value_pool.dtype != key_pool.dtype:
        raise RuntimeError("query and pools must share a dtype")
    if not (key_pool.is_contiguous() and value_pool.is_contiguous()):
        raise RuntimeError("pools must be contiguous")
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise RuntimeError("block_tables and context_lens must be int32")
    if seq_rows is not None and seq_rows.dtype != torch.int32:
        raise RuntimeError("seq_rows must be int32")
    B, H, D = query.shape
    Hkv, NB, bs, Dk = key_pool.shape
    if Dk != D:
        raise RuntimeError("query and pools disagree on head_dim")
    if context_lens.numel() < B or (seq_rows is not None and seq_rows.numel() < B):
        raise RuntimeError("context_lens / seq_rows must hold one entry per sequence")
    if query.stride(2) != 1 or query.stride(1) != D:
        query = query.contiguous()
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    if out is None:
        out = torch.empty((B, H, D), dtype=query.dtype, device=device)
    elif out.shape != (B, H, D) or out.stride(2) != 1 or out.stride(1) != D:
        raise RuntimeError("out must be [B, H, D] with contiguous heads")
    mb = block_tables.size(1) if max_blocks_per_seq is None else int(max_blocks_per_seq)
    code = dtype_code(query.dtype)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        key = (device.index, B, H, Hkv, D, bs, code)
        need = _batched_ws_bytes.get(key)
        if need is None:
            got = ctypes.c_uint64(0)
            check(lib().bs_paged_attention_batched_workspace_bytes(B, H, Hkv, D, bs, code,
                                                                   ctypes.byref(got)))
            need = _batched_ws_bytes[key] = got.value
        ws = workspace_for(device, need)
        check(lib().bs_paged_attention_batched(
            query.data_ptr(), query.stride(0), key_pool.data_ptr(), value_pool.data_ptr(),
            block_tables.data_ptr(), block_tables.stride(0), block_tables.size(0),
            seq_rows.data_ptr() if seq_rows is not None else None, context_lens.data_ptr(),
            B, H, Hkv, D, bs, NB, mb, code, float(scaling), int(units_hint),
            (1 if lens_ready else 0) | (2 if after_append else 0), out.data_ptr(),
            out.stride(0), ws.data_ptr(), ws.numel(), stream))
    return out


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, key_pool: torch.Tensor,
                      value_pool: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Write rows [T, Hkv, D] (or [T, Hkv*D]) into pool[h, slot // bs, slot % bs].

    The batched form of PagedKVCache.append (src/server/torch_model.py:149-153);
    an fp32 input into a bf16 pool is rounded to nearest-even.
    """
    device = _require_cuda("reshape_and_cache", key, value, key_pool, value_pool, slot_mapping)
    Hkv, NB, bs, D = key_pool.shape
    T = slot_mapping.numel()
    if slot_mapping.dtype != torch.int32:
        raise RuntimeError("slot_mapping must be int32")
    if key.dtype != value.dtype or key_pool.dtype != value_pool.dtype or value_pool.shape != key_pool.shape:
        raise RuntimeError("key/value dtypes or pool shapes disagree")
    if not (key_pool.is_contiguous() and value_pool.is_contiguous()):
        raise RuntimeError("pools must be contiguous")
    k2 = key.reshape(key.size(0), -1) if key.dim() != 2 else key
    v2 = value.reshape(value.size(0), -1) if value.dim() != 2 else value
    if k2.size(0) < T or v2.size(0) < T or k2.size(1) != Hkv * D or v2.size(1) != Hkv * D:
        raise RuntimeError("key/value must be [T, kv_heads, head_dim]")
    if k2.stride(1) != 1:
        k2 = k2.contiguous()
    if v2.stride(1) != 1:
        v2 = v2.contiguous()
    ws = workspace_for(device, 0)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(lib().bs_reshape_and_cache(
            k2.data_ptr(), v2.data_ptr(), k2.stride(0), v2.stride(0), dtype_code(key.dtype),
            slot_mapping.data_ptr(), T, key_pool.data_ptr(), value_pool.data_ptr(),
            dtype_code(key_pool.dtype), Hkv, NB, bs, D, ws.data_ptr(), stream))


def step_metadata(block_tables: torch.Tensor, start_pos: torch.Tensor, n_new: torch.Tensor,
                  num_tokens: int, block_size: int, num_blocks: int,
                  seq_rows: torch.Tensor | None = None, max_blocks_per_seq: int | None = None):
    """Device metadata of one step: (cu_q, positions, slot_mapping, context_lens), all int32.

    Rows r hold n_new[r] new tokens after start_pos[r] cached ones; the slot of a
    token is the reference's BlockAllocator.locate flattened to
    block * block_size + offset (src/server/block_allocator.py:28-30).
    """
    device = _require_cuda("step_metadata", block_tables, start_pos, n_new, seq_rows)
    R = start_pos.numel()
    for name, t in (("block_tables", block_tables), ("start_pos", start_pos), ("n_new", n_new)):
        if t.dtype != torch.int32:
            raise RuntimeError(f"{name} must be int32")
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    cu_q = torch.empty(R + 1, dtype=torch.int32, device=device)
    positions = torch.empty(max(num_tokens, 1), dtype=torch.int32, device=device)
    slots = torch.empty(max(num_tokens, 1), dtype=torch.int32, device=device)
    context = torch.empty(max(R, 1), dtype=torch.int32, device=device)
    mb = block_tables.size(1) if max_blocks_per_seq is None else int(max_blocks_per_seq)
    ws = workspace_for(device, 0)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(lib().bs_step_metadata(
            seq_rows.data_ptr() if seq_rows is not None else None, start_pos.data_ptr(),
            n_new.data_ptr(), R, block_tables.data_ptr(), block_tables.stride(0),
            block_tables.size(0), mb, block_size, num_blocks, num_tokens, cu_q.data_ptr(),
            positions.data_ptr(), slots.data_ptr(), context.data_ptr(), ws.data_ptr(), stream))
    return cu_q, positions[:num_tokens], slots[:num_tokens], context[:R]


def decode_append(key: torch.Tensor, value: torch.Tensor, key_pool: torch.Tensor,
                  value_pool: torch.Tensor, block_tables: torch.Tensor, start_pos: torch.Tensor,
                  seq_rows: torch.Tensor | None = None, max_blocks_per_seq: int | None = None,
                  context_lens: torch.Tensor | None = None, slots: torch.Tensor | None = None):
    """One decode step's K/V append in one launch: row r ([Hkv, D] of key/value)
    lands at position start_pos[r] of its sequence.  Returns (context_lens,
    slot_mapping) int32 [B] — what step_metadata + reshape_and_cache give for a
    step of one new token per row (PagedKVCache.append,
    src/server/torch_model.py:149-153, through BlockAllocator.locate)."""
    device = _require_cuda("decode_append", key, value, key_pool, value_pool, block_tables,
                           start_pos, seq_rows)
    if key is None or value is None:
        if key is not value:
            raise RuntimeError("key and value must both be given or both be None")
        return _locate(key_pool, value_pool, block_tables, start_pos, seq_rows,
                       max_blocks_per_seq, context_lens, slots, device)
    Hkv, NB, bs, D = key_pool.shape
    B = start_pos.numel()
    for name, t in (("block_tables", block_tables), ("start_pos", start_pos)):
        if t.dtype != torch.int32:
            raise RuntimeError(f"{name} must be int32")
    if seq_rows is not None and (seq_rows.dtype != torch.int32 or seq_rows.numel() < B):
        raise RuntimeError("seq_rows must be int32 with one entry per row")
    if key.dtype != value.dtype or value_pool.shape != key_pool.shape:
        raise RuntimeError("key/value dtypes or pool shapes disagree")
    if not (key_pool.is_contiguous() and value_pool.is_contiguous()):
        raise RuntimeError("pools must be contiguous")
    k2 = key.reshape(key.size(0), -1) if key.dim() != 2 else key
    v2 = value.reshape(value.size(0), -1) if value.dim() != 2 else value
    if k2.size(0) < B or v2.size(0) < B or k2.size(1) != Hkv * D or v2.size(1) != Hkv * D:
        raise RuntimeError("key/value must be [B, kv_heads, head_dim]")
    if k2.stride(1) != 1:
        k2 = k2.contiguous()
    if v2.stride(1) != 1:
        v2 = v2.contiguous()
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    ctx = context_lens if context_lens is not None else torch.empty(
        max(B, 1), dtype=torch.int32, device=device)
    sl = slots if slots is not None else torch.empty(max(B, 1), dtype=torch.int32, device=device)
    mb = block_tables.size(1) if max_blocks_per_seq is None else int(max_blocks_per_seq)
    ws = workspace_for(device, 0)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(lib().bs_decode_append(
            seq_rows.data_ptr() if seq_rows is not None else None, start_pos.data_ptr(), B,
            block_tables.data_ptr(), block_tables.stride(0), block_tables.size(0), mb,
            k2.data_ptr(), v2.data_ptr(), k2.stride(0), v2.stride(0), dtype_code(key.dtype),
            key_pool.data_ptr(), value_pool.data_ptr(), dtype_code(key_pool.dtype), Hkv, NB, bs, D,
            ctx.data_ptr(), sl.data_ptr(), ws.data_ptr(), stream))
    return ctx[:B], sl[:B]


def _locate(key_pool, value_pool, block_tables, start_pos, seq_rows, max_blocks_per_seq,
            context_lens, slots, device):
    """decode_append without rows: context lengths and slots only."""
    Hkv, NB, bs, D = key_pool.shape
    B = start_pos.numel()
    for name, t in (("block_tables", block_tables), ("start_pos", start_pos)):
        if t.dtype != torch.int32:
            raise RuntimeError(f"{name} must be int32")
    if seq_rows is not None and (seq_rows.dtype != torch.int32 or seq_rows.numel() < B):
        raise RuntimeError("seq_rows must be int32 with one entry per row")
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    ctx = context_lens if context_lens is not None else torch.empty(
        max(B, 1), dtype=torch.int32, device=device)
    sl = slots if slots is not None else torch.empty(max(B, 1), dtype=torch.int32, device=device)
    mb = block_tables.size(1) if max_blocks_per_seq is None else int(max_blocks_per_seq)
    ws = workspace_for(device, 0)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(lib().bs_decode_append(
            seq_rows.data_ptr() if seq_rows is not None else None, start_pos.data_ptr(), B,
            block_tables.data_ptr(), block_tables.stride(0), block_tables.size(0), mb, None, None,
            Hkv * D, Hkv * D, dtype_code(key_pool.dtype), key_pool.data_ptr(),
            value_pool.data_ptr(), dtype_code(key_pool.dtype), Hkv, NB, bs, D, ctx.data_ptr(),
            sl.data_ptr(), ws.data_ptr(), stream))
    return ctx[:B], sl[:B]


def _rows_2d(name: str, t: torch.Tensor, width: int) -> torch.Tensor:
    t2 = t if t.dim() == 2 else t.reshape(t.size(0), -1)
    if t2.size(1) != width:
        raise RuntimeError(f"{name} rows must hold {width} elements")
    return t2 if t2.stride(1) == 1 else t2.contiguous()


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, add: torch.Tensor | None = None,
             row_index: torch.Tensor | None = None, sum_out: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm of the reference TorchModel (src/server/torch_model.py:283-287)
    with the residual add before it fused: per output row r (source row
    i = row_index[r], or r), s = (x[i] + add[i]) in x's dtype, sum_out[r] = s,
    and returns weight * (s_f32 * rsqrt(mean(s_f32^2) + eps)).to(dtype).
    ``sum_out`` may be ``x`` (the residual stream updated in place) only
    without ``row_index``."""
    device = _require_cuda("rms_norm", x, weight, add, row_index, sum_out, out)
    hidden = weight.numel()
    x2 = _rows_2d("x", x, hidden)
    if x2.dtype != weight.dtype or (add is not None and add.dtype != x2.dtype):
        raise RuntimeError("x, add and weight must share a dtype")
    a2 = _rows_2d("add", add, hidden) if add is not None else None
    if a2 is not None and a2.size(0) < x2.size(0):
        raise RuntimeError("add must have a row for every row of x")
    if row_index is not None:
        if row_index.dtype != torch.int32:
            raise RuntimeError("row_index must be int32")
        rows = row_index.numel()
    else:
        rows = x2.size(0)
    o2 = out if out is not None else torch.empty((rows, hidden), dtype=x2.dtype, device=device)
    s2 = sum_out
    for name, t in (("out", o2), ("sum_out", s2)):
        if t is not None and (t.dim() != 2 or t.stride(1) != 1 or t.size(1) != hidden
                              or t.size(0) < rows or t.dtype != x2.dtype):
            raise RuntimeError(f"{name} must be [rows, hidden] with unit inner stride in x's dtype")
    ws = workspace_for(device, 0)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(lib().bs_rms_norm(
            x2.data_ptr(), x2.stride(0), x2.size(0), a2.data_ptr() if a2 is not None else None,
            a2.stride(0) if a2 is not None else 0,
            row_index.data_ptr() if row_index is not None else None, weight.contiguous().data_ptr(),
            rows, hidden, float(eps), dtype_code(x2.dtype), o2.data_ptr(), o2.stride(0),
            s2.data_ptr() if s2 is not None else None, s2.stride(0) if s2 is not None else 0,
            ws.data_ptr(), stream))
    return o2


def rope_append(qkv: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor,
                positions: torch.Tensor, slot_mapping: torch.Tensor, key_pool: torch.Tensor,
                value_pool: torch.Tensor, num_heads: int, query_out: torch.Tensor | None = None
                ) -> torch.Tensor:
    """Rotary embedding and K/V append in one launch.  ``qkv`` rows are the
    fused projection [q heads | k heads | v heads] ([T, (H + 2 Hkv) D]); q and
    k are rotated with the cos/sin tables gathered at ``positions``
    (src/server/torch_model.py:190-192, 262-264, same rounding points), q is
    returned as [T, H, D] and k, v are written at ``slot_mapping`` into the
    pools [Hkv, blocks, block_size, D] (PagedKVCache.append, :149-153); a
    negative slot skips the row's write."""
    device = _require_cuda("rope_append", qkv, cos_table, sin_table, positions, slot_mapping,
                           key_pool, value_pool, query_out)
    Hkv, NB, bs, D = key_pool.shape
    T = positions.numel()
    if positions.dtype != torch.int32 or slot_mapping.dtype != torch.int32:
        raise RuntimeError("positions and slot_mapping must be int32")
    if slot_mapping.numel() < T or qkv.size(0) < T:
        raise RuntimeError("qkv and slot_mapping need a row per position")
    if value_pool.shape != key_pool.shape or value_pool.dtype != key_pool.dtype:
        raise RuntimeError("key/value pools disagree")
    if not (key_pool.is_contiguous() and value_pool.is_contiguous()):
        raise RuntimeError("pools must be contiguous")
    if cos_table.shape != sin_table.shape or cos_table.size(-1) != D or cos_table.dtype != qkv.dtype:
        raise RuntimeError("cos/sin tables must be [positions, head_dim] in the qkv dtype")
    q2 = _rows_2d("qkv", qkv, (num_heads + 2 * Hkv) * D)
    cos_c, sin_c = cos_table.contiguous(), sin_table.contiguous()
    q_out = query_out if query_out is not None else torch.empty(
        (T, num_heads, D), dtype=qkv.dtype, device=device)
    if not q_out.is_contiguous() or q_out.numel() < T * num_heads * D:
        raise RuntimeError("query_out must be contiguous [T, heads, head_dim]")
    ws = workspace_for(device, 0)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(lib().bs_rope_append(
            q2.data_ptr(), q2.stride(0), dtype_code(qkv.dtype), cos_c.data_ptr(), sin_c.data_ptr(),
            cos_c.size(0), positions.data_ptr(), slot_mapping.data_ptr(), T, num_heads, Hkv, D,
            q_out.data_ptr(), key_pool.data_ptr(), value_pool.data_ptr(),
            dtype_code(key_pool.dtype), NB, bs, ws.data_ptr(), stream))
    return q_out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """SwiGLU gating of the reference MLP (src/server/torch_model.py:278-281):
    rows [gate | up] -> silu(gate) * up, rounded to the dtype after each op."""
    device = _require_cuda("silu_mul", gate_up, out)
    if gate_up.dim() != 2 or gate_up.stride(1) != 1 or gate_up.size(1) % 2:
        raise RuntimeError("gate_up must be [T, 2 * intermediate] with unit inner stride")
    T, inter = gate_up.size(0), gate_up.size(1) // 2
    o = out if out is not None else torch.empty((T, inter), dtype=gate_up.dtype, device=device)
    if not o.is_contiguous() or o.shape != (T, inter) or o.dtype != gate_up.dtype:
        raise RuntimeError("out must be contiguous [T, intermediate] in the input dtype")
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(lib().bs_silu_mul(gate_up.data_ptr(), gate_up.stride(0), T, inter,
                                dtype_code(gate_up.dtype), o.data_ptr(), stream))
    return o


def argmax_rows(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """int32 greedy token of each row of `logits` [R, V]: the first index of
    the maximum (a NaN counts as the maximum), as torch.argmax."""
    device = _require_cuda("argmax_rows", logits, out)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise RuntimeError("logits must be [rows, vocab] with unit inner stride")
    R, V = logits.shape
    o = out if out is not None else torch.empty(R, dtype=torch.int32, device=device)
    if o.dtype != torch.int32 or o.numel() < R or not o.is_contiguous():
        raise RuntimeError("out must be int32 with a slot per row")
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(lib().bs_argmax_rows(logits.data_ptr(), logits.stride(0), R, V,
                                   dtype_code(logits.dtype), o.data_ptr(), stream))
    return o


__all__ = [
    "paged_attention",
    "paged_attention_batched",
    "reshape_and_cache",
    "decode_append",
    "step_metadata",
    "rms_norm",
    "rope_append",
    "silu_mul",
    "argmax_rows",
    "take_status",
    "kernel_launches",
    "decode_workspace_bytes",
    "prefill_workspace_bytes",
    "workspace_for",
    "dtype_code",
    "_lib",
]


BS_PREFILL_PER_TOKEN = 0x2
_prefill_ws_bytes: dict[tuple, int] = {}


def prefill_attention(query: torch.Tensor, key_pool: torch.Tensor, value_pool: torch.Tensor,
                      block_tables: torch.Tensor, cu_q: torch.Tensor, context_lens: torch.Tensor,
                      scaling: float, max_query_len: int, seq_rows: torch.Tensor | None = None,
                      out: torch.Tensor | None = None, per_token: bool = False,
                      max_blocks_per_seq: int | None = None) -> torch.Tensor:
    """Causal attention of prompt chunks over their paged context, in one call.

    query [T, H, D] holds the chunks back to back (chunk r is rows cu_q[r] ..
    cu_q[r+1]); context_lens[r] counts the sequence's cached tokens including the
    chunk (its K/V must already be in the pool).  Query token i of chunk r sees
    keys 0 .. context_lens[r] - n_r + i — the reference's attend() with
    _causal_mask (src/server/torch_model.py:39-55, 295-297).  bf16 at head_dim 64
    runs on the tcgen05 tensor cores; other shapes (or per_token=True) run each
    token as a decode query over its causal length.  Returns [T, H, D].
    """
    device = _require_cuda("prefill_attention", query, key_pool, value_pool, block_tables, cu_q,
                           context_lens, seq_rows, out)
    if query.dim() != 3 or key_pool.dim() != 4 or value_pool.shape != key_pool.shape:
        raise RuntimeError("query must be [T, H, D] and the pools [Hkv, NB, bs, D]")
    if query.dtype != key_pool.dtype or value_pool.dtype != key_pool.dtype:
        raise RuntimeError("query and pools must share a dtype")
    if not (key_pool.is_contiguous() and value_pool.is_contiguous()):
        raise RuntimeError("pools must be contiguous")
    for name, t in (("block_tables", block_tables), ("cu_q", cu_q), ("context_lens", context_lens)):
        if t.dtype != torch.int32:
            raise RuntimeError(f"{name} must be int32")
    if seq_rows is not None and seq_rows.dtype != torch.int32:
        raise RuntimeError("seq_rows must be int32")
    T, H, D = query.shape
    Hkv, NB, bs, Dk = key_pool.shape
    if Dk != D:
        raise RuntimeError("query and pools disagree on head_dim")
    R = context_lens.numel()
    if cu_q.numel() < R + 1:
        raise RuntimeError("cu_q must hold num_rows + 1 offsets")
    if not query.is_contiguous():
        query = query.contiguous()
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    if out is None:
        out = torch.empty((T, H, D), dtype=query.dtype, device=device)
    elif out.shape != (T, H, D) or out.stride(2) != 1 or out.stride(1) != D:
        raise RuntimeError("out must be [T, H, D] with contiguous heads")
    mb = block_tables.size(1) if max_blocks_per_seq is None else int(max_blocks_per_seq)
    code = dtype_code(query.dtype)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        key = (device.index, T, R, int(max_query_len), H, Hkv, D, bs, code)
        need = _prefill_ws_bytes.get(key)
        if need is None:
            got = ctypes.c_uint64(0)
            check(lib().bs_prefill_attention_workspace_bytes(T, R, int(max_query_len), H, Hkv, D,
                                                             bs, code, ctypes.byref(got)))
            need = _prefill_ws_bytes[key] = got.value
        ws = workspace_for(device, need)
        check(lib().bs_prefill_attention(
            query.data_ptr(), query.stride(0), cu_q.data_ptr(), R, T, int(max_query_len),
            context_lens.data_ptr(), seq_rows.data_ptr() if seq_rows is not None else None,
            key_pool.data_ptr(), value_pool.data_ptr(), block_tables.data_ptr(),
            block_tables.stride(0), block_tables.size(0), mb, H, Hkv, D, bs, NB, code,
            float(scaling), BS_PREFILL_PER_TOKEN if per_token else 0, out.data_ptr(),
            out.stride(0), ws.data_ptr(), ws.numel(), stream))
    return out
