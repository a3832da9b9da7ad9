"""ORACLE — test infrastructure only, never part of the product path.

CPU restatement of the BatchStream reference's paged-attention arithmetic
(plain C in ``paged_attention_oracle.c``, loaded through ctypes) plus a pure
Python restatement of its block allocator.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
this package, and only as the parity reference or the timed CPU baseline.

Pinning: the golden fixtures under ``tests/golden/`` were produced by the
reference itself (its compiled C++ op and its Python op, see
``tests/golden/make_golden.py``); ``tests/test_oracle.py`` checks every function
here against them.

``oracle/_ref/`` (built by ``build_ref.py`` from the reference sources, never
committed) holds the reference's own C++ op for the CPU baseline of kind
"reference".
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "paged_attention_oracle.c"
LIBRARY = HERE / "libbs_oracle.so"
REF_DIR = HERE / "_ref"

_lib = None


def build(force: bool = False) -> Path:
    """Compile the C restatement (gcc, no fast-math so sums keep their order)."""
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < SOURCE.stat().st_mtime:
        tmp = LIBRARY.with_suffix(".so.tmp")
        subprocess.run(
            ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", str(SOURCE), "-o", str(tmp), "-lm"],
            check=True,
        )
        tmp.replace(LIBRARY)
    return LIBRARY


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIBRARY))
        i64, p, dbl = ctypes.c_int64, ctypes.c_void_p, ctypes.c_double
        lib.oracle_decode_bf16.argtypes = [p, p, p, i64, i64, i64, i64, i64, p, i64, i64, dbl, p]
        lib.oracle_decode_f32.argtypes = [p, p, p, i64, i64, i64, i64, i64, p, i64, i64, dbl, p]
        lib.oracle_prefill.argtypes = [
            p, p, p, ctypes.c_int32, i64, i64, i64, i64, i64, i64, i64, p, i64, dbl, p,
        ]
        lib.oracle_slot_mapping.argtypes = [p, i64, p, p, i64, i64, p, p]
        lib.oracle_slot_mapping.restype = i64
        _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _table(table) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(table, dtype=np.int64))


def decode(query: np.ndarray, keys: np.ndarray, values: np.ndarray, table, length: int,
           block_size: int, groups: int, scaling: float) -> np.ndarray:
    """One decode token.  bf16 arrays are uint16 bit patterns; fp32 arrays float32.

    Shapes: query [H, D], keys/values [Hkv, NB, bs, D]; returns [H, D] of the
    same storage type.
    """
    lib = _load()
    H, D = query.shape
    Hkv, NB, bs, _ = keys.shape
    assert bs == block_size
    q = np.ascontiguousarray(query)
    k = np.ascontiguousarray(keys)
    v = np.ascontiguousarray(values)
    tab = _table(table)
    out = np.empty((H, D), dtype=q.dtype)
    fn = lib.oracle_decode_bf16 if q.dtype == np.uint16 else lib.oracle_decode_f32
    if q.dtype not in (np.uint16, np.float32):
        raise TypeError("oracle decode takes uint16 (bf16 bits) or float32 arrays")
    rc = fn(_ptr(q), _ptr(k), _ptr(v), H, Hkv, NB, bs, D, _ptr(tab), length, groups, scaling,
            _ptr(out))
    if rc != 0:
        raise MemoryError("oracle scratch allocation failed")
    return out


def prefill(query: np.ndarray, keys: np.ndarray, values: np.ndarray, table, past: int,
            block_size: int, groups: int, scaling: float) -> np.ndarray:
    """A causal prefill chunk: query [n, H, D] at positions past .. past+n-1."""
    lib = _load()
    n, H, D = query.shape
    Hkv, NB, bs, _ = keys.shape
    assert bs == block_size
    q = np.ascontiguousarray(query)
    k = np.ascontiguousarray(keys)
    v = np.ascontiguousarray(values)
    tab = _table(table)
    out = np.empty_like(q)
    dtype = 0 if q.dtype == np.uint16 else 1
    rc = lib.oracle_prefill(_ptr(q), _ptr(k), _ptr(v), dtype, n, past, H, Hkv, NB, bs, D,
                            _ptr(tab), groups, scaling, _ptr(out))
    if rc != 0:
        raise MemoryError("oracle scratch allocation failed")
    return out


def slot_mapping(tables: list[list[int]], start_pos, n_new, block_size: int):
    """(positions, slots) of every new token, rows in order (locate, flattened)."""
    lib = _load()
    R = len(tables)
    width = max([len(t) for t in tables] + [1])
    tab = np.full((R, width), -1, dtype=np.int64)
    for r, t in enumerate(tables):
        tab[r, : len(t)] = t
    sp = np.ascontiguousarray(np.asarray(start_pos, dtype=np.int64))
    nn = np.ascontiguousarray(np.asarray(n_new, dtype=np.int64))
    T = int(nn.sum())
    pos = np.empty(max(T, 1), dtype=np.int64)
    slots = np.empty(max(T, 1), dtype=np.int64)
    got = lib.oracle_slot_mapping(_ptr(tab), width, _ptr(sp), _ptr(nn), R, block_size, _ptr(pos),
                                  _ptr(slots))
    assert got == T
    return pos[:T], slots[:T]


class OutOfBlocks(RuntimeError):
    """Raised when a table cannot grow (block_allocator.py:1-2)."""


class Allocator:
    """Restatement of the reference BlockAllocator (src/server/block_allocator.py:5-33).

    LIFO free list starting as range(num_blocks), tables grow to
    ceil(tokens / block_size) blocks, all-or-nothing allocation, free returns a
    table's blocks in table order.
    """

    def __init__(self, num_blocks: int, block_size: int):
        self.block_size = block_size
        self.free_list = list(range(num_blocks))
        self.tables: dict[int, list[int]] = {}

    def allocate(self, seq_id: int, total_tokens: int) -> None:
        table = self.tables.get(seq_id, [])
        need = -(-total_tokens // self.block_size) - len(table)
        if need > len(self.free_list):
            raise OutOfBlocks(f"need {need} blocks, {len(self.free_list)} free")
        for _ in range(need):
            table.append(self.free_list.pop())
        self.tables[seq_id] = table

    def locate(self, seq_id: int, position: int) -> tuple[int, int]:
        index, offset = divmod(position, self.block_size)
        return self.tables[seq_id][index], offset

    def free(self, seq_id: int) -> None:
        self.free_list.extend(self.tables.pop(seq_id))


def load_reference_op():
    """The reference's own C++ op built into oracle/_ref (None when absent)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (loads libc10/libtorch that the module links against)

    hits = sorted(REF_DIR.glob("paged_attention_cpp*.so"))
    if not hits:
        return None
    loader = importlib.machinery.ExtensionFileLoader("paged_attention_cpp", str(hits[0]))
    spec = importlib.util.spec_from_loader("paged_attention_cpp", loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    return module.paged_attention
