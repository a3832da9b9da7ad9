"""The C ABI library loads, exports what the header declares, and validates input
on the host exactly like the reference op (no GPU needed for any of this)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from batchstream_inference_engine_b200 import _lib
from batchstream_inference_engine_b200.paged_attention_cuda import paged_attention
from tests.golden import inputs

HEADER_DIR = Path(__file__).resolve().parent.parent / "include"


def declared_symbols():
    names = set()
    for header in HEADER_DIR.glob("*.h"):
        text = header.read_text()
        names.update(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(bs_\w+)\(", text, re.M))
    return names


def test_library_loads_and_reports_version():
    assert _lib.lib().bs_version().decode().startswith("batchstream_b200")


def test_every_declared_symbol_is_exported():
    declared = declared_symbols()
    assert declared, "no declarations found in include/"
    handle = ctypes.CDLL(str(_lib.LIBRARY))
    for name in declared:
        assert hasattr(handle, name), name
    assert declared == set(_lib.EXPORTS)


def test_library_does_not_link_the_cuda_runtime_or_driver_dynamically():
    # Static runtime, driver reached through the entry-point query: loads anywhere.
    import subprocess

    out = subprocess.run(["ldd", str(_lib.LIBRARY)], capture_output=True, text=True).stdout
    assert "libcudart" not in out and "libcuda.so" not in out


# The reference's malformed-input cases (tests/test_paged_attention.py:205-237).
BAD_INPUTS = [
    {"length": 0},
    {"length": -1},
    {"length": 13},
    {"table": []},
    {"table": [999, 0]},
    {"table": [-1, 0]},
    {"block_size": 0},
    {"block_size": 8},
    {"groups": 0},
    {"groups": 3},
    {"query": torch.zeros(4, 7, dtype=torch.bfloat16)},
    {"query": torch.zeros(4, 8, dtype=torch.float32)},
    {"query": torch.zeros(8, dtype=torch.bfloat16)},
    {"keys": torch.zeros(2, 3, 4, 8, dtype=torch.float32)},
    {"keys": torch.zeros(3, 8, dtype=torch.bfloat16)},
    {"values": torch.zeros(2, 2, 4, 8, dtype=torch.bfloat16)},
]


@pytest.mark.parametrize("change", BAD_INPUTS)
def test_host_validation_rejects_bad_input_with_runtime_error(change):
    query, keys, values, table = inputs.scattered_bf16(5)
    args = dict(query=query, keys=keys, values=values, table=table, length=5, block_size=4,
                groups=2)
    args.update(change)
    with pytest.raises(RuntimeError) as err:
        paged_attention(args["query"], args["keys"], args["values"], args["table"],
                        args["length"], args["block_size"], args["groups"], 0.5)
    # The error comes from the library's input checks, before any device work.
    assert "CUDA" not in str(err.value) and "cuda" not in str(err.value)


def test_valid_host_tensors_are_never_computed_on_the_host():
    # Host tensors pass the reference's checks and are then staged on a CUDA
    # device; without one the call is refused -- there is no host arithmetic.
    query, keys, values, table = inputs.scattered_bf16(5)
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present: the host-tensor path runs on it (gpu tests)")
    with pytest.raises(RuntimeError, match="no CUDA device"):
        paged_attention(query, keys, values, table, 5, 4, 2, 0.5)


def test_check_entry_point_runs_the_reference_checks_alone():
    from batchstream_inference_engine_b200._lib import i64_array

    lib = _lib.lib()
    args = lambda length, table: (  # noqa: E731
        _lib.BS_BF16, 2, i64_array([4, 8]), i64_array([8, 1]), _lib.BS_BF16, 4,
        i64_array([2, 5, 4, 8]), i64_array([160, 32, 8, 1]), _lib.BS_BF16, 4,
        i64_array([2, 5, 4, 8]), i64_array([160, 32, 8, 1]), i64_array(table), len(table),
        length, 4, 2)
    assert lib.bs_paged_attention_check(*args(5, [3, 1])) == 0
    assert lib.bs_paged_attention_check(*args(13, [3, 1])) != 0
    assert b"too short" in lib.bs_last_error()
    assert lib.bs_paged_attention_check(*args(5, [3, 5])) != 0
    assert b"out of range" in lib.bs_last_error()


def test_error_codes_come_with_messages():
    lib = _lib.lib()
    need = ctypes.c_uint64(0)
    rc = lib.bs_paged_attention_workspace_bytes(4, 3, 8, 2, 0, 4, ctypes.byref(need))
    assert rc != 0
    assert b"kv_heads" in lib.bs_last_error()
