"""ctypes binding of ``libbatchstream_b200.so`` (the C ABI in include/batchstream_b200.h).

The library is loaded once per process.  A missing library is an ImportError
with the build command in the message: there is no fallback path.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libbatchstream_b200.so"

BS_BF16 = 0
BS_F32 = 1

# Every symbol the header declares; tests check they are all exported.
EXPORTS = (
    "bs_last_error",
    "bs_version",
    "bs_paged_attention",
    "bs_paged_attention_check",
    "bs_paged_attention_workspace_bytes",
    "bs_paged_attention_batched",
    "bs_paged_attention_batched_workspace_bytes",
    "bs_paged_attention_batched_noalloc",
    "bs_prefill_attention",
    "bs_prefill_attention_workspace_bytes",
    "bs_reshape_and_cache",
    "bs_decode_append",
    "bs_step_metadata",
    "bs_take_status",
    "bs_reset_workspace",
    "bs_set_wait_probe",
    "bs_rms_norm",
    "bs_rope_append",
    "bs_silu_mul",
    "bs_kernel_launches",
    "bs_argmax_rows",
)

_i32, _i64, _u64, _p, _dbl = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_double
_pi64 = ctypes.POINTER(ctypes.c_int64)

_SIGNATURES = {
    "bs_last_error": ([], ctypes.c_char_p),
    "bs_version": ([], ctypes.c_char_p),
    "bs_paged_attention": (
        [_p, _i32, _i32, _pi64, _pi64,
         _p, _i32, _i32, _pi64, _pi64,
         _p, _i32, _i32, _pi64, _pi64,
         _pi64, _i64, _i64, _i64, _i64, _dbl, _p, _p, _u64, _p],
        ctypes.c_int,
    ),
    "bs_paged_attention_check": (
        [_i32, _i32, _pi64, _pi64, _i32, _i32, _pi64, _pi64, _i32, _i32, _pi64, _pi64,
         _pi64, _i64, _i64, _i64, _i64],
        ctypes.c_int,
    ),
    "bs_paged_attention_workspace_bytes": (
        [_i64, _i64, _i64, _i64, _i32, _i64, ctypes.POINTER(_u64)], ctypes.c_int,
    ),
    "bs_paged_attention_batched": (
        [_p, _i64, _p, _p, _p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
         _i32, _dbl, _i64, _i32, _p, _i64, _p, _u64, _p],
        ctypes.c_int,
    ),
    "bs_paged_attention_batched_noalloc": (
        [_p, _i64, _p, _p, _p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
         _i32, _dbl, _p, _i64, _p, _p],
        ctypes.c_int,
    ),
    "bs_paged_attention_batched_workspace_bytes": (
        [_i64, _i64, _i64, _i64, _i64, _i32, ctypes.POINTER(_u64)], ctypes.c_int,
    ),
    "bs_prefill_attention": (
        [_p, _i64, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
         _i64, _i64, _i32, _dbl, _i32, _p, _i64, _p, _u64, _p],
        ctypes.c_int,
    ),
    "bs_prefill_attention_workspace_bytes": (
        [_i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, ctypes.POINTER(_u64)], ctypes.c_int,
    ),
    "bs_reshape_and_cache": (
        [_p, _p, _i64, _i64, _i32, _p, _i64, _p, _p, _i32, _i64, _i64, _i64, _i64, _p, _p],
        ctypes.c_int,
    ),
    "bs_decode_append": (
        [_p, _p, _i64, _p, _i64, _i64, _i64, _p, _p, _i64, _i64, _i32, _p, _p, _i32, _i64, _i64,
         _i64, _i64, _p, _p, _p, _p],
        ctypes.c_int,
    ),
    "bs_step_metadata": (
        [_p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p],
        ctypes.c_int,
    ),
    "bs_take_status": ([_p, _p, ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
    "bs_reset_workspace": ([_p, _p], ctypes.c_int),
    "bs_set_wait_probe": ([_i32, _u64], ctypes.c_int),
    "bs_rms_norm": (
        [_p, _i64, _i64, _p, _i64, _p, _p, _i64, _i64, _dbl, _i32, _p, _i64, _p, _i64, _p, _p],
        ctypes.c_int,
    ),
    "bs_rope_append": (
        [_p, _i64, _i32, _p, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _i32, _i64,
         _i64, _p, _p],
        ctypes.c_int,
    ),
    "bs_silu_mul": ([_p, _i64, _i64, _i64, _i32, _p, _p], ctypes.c_int),
    "bs_kernel_launches": ([], ctypes.c_uint64),
    "bs_argmax_rows": ([_p, _i64, _i64, _i64, _i32, _p, _p], ctypes.c_int),
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first use)."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise ImportError(
                f"{LIBRARY.name} is not built; run `python -m batchstream_inference_engine_b200.build`"
            )
        handle = ctypes.CDLL(str(LIBRARY))
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = res
        _lib = handle
    return _lib


def check(rc: int) -> None:
    """Raise the reference's RuntimeError for a failing call."""
    if rc != 0:
        message = lib().bs_last_error().decode(errors="replace")
        raise RuntimeError(message or f"batchstream_b200 call failed with code {rc}")


def i64_array(values) -> ctypes.Array:
    seq = list(values)
    return (ctypes.c_int64 * max(len(seq), 1))(*seq)
