"""CPU checks of the C-ABI boundary: the library loads without a GPU, exports every symbol the header
declares with the binding's arity, and rejects bad arguments before touching the device."""

from __future__ import annotations

import ctypes
import re

import pytest

import cuda_loader
import paged_kv_ops


def _declared_symbols() -> dict[str, int]:
    text = cuda_loader.HEADER_PATH.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for match in re.finditer(r"PKV_API\s+[\w\s\*]+?\b(pkv_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a for a in match.group(2).split(",") if a.strip() and a.strip() != "void"]
        out[match.group(1)] = len(args)
    return out


def test_header_declares_the_bound_symbols() -> None:
    declared = _declared_symbols()
    assert declared, "no declarations parsed"
    assert set(declared) == set(cuda_loader.SIGNATURES)
    for name, arity in declared.items():
        assert len(cuda_loader.SIGNATURES[name][1]) == arity, name


def test_library_loads_and_exports_every_declared_symbol() -> None:
    lib = cuda_loader.load_paged_kv_library()
    raw = ctypes.CDLL(str(cuda_loader.library_path()))
    for name in _declared_symbols():
        assert hasattr(raw, name), name
    assert lib.pkv_abi_version() == 1


def test_stats_are_readable_without_a_gpu() -> None:
    lib = cuda_loader.load_paged_kv_library()
    n = lib.pkv_stats(None, 0)
    assert n == len(paged_kv_ops.STAT_NAMES) == 14
    buf = (ctypes.c_int64 * n)()
    lib.pkv_reset_stats()
    assert lib.pkv_stats(buf, n) == n
    assert list(buf) == [0] * n


def test_workspace_size_is_host_only_and_grows_with_the_table() -> None:
    lib = cuda_loader.load_paged_kv_library()
    small = lib.pkv_paged_decode_workspace_size(64, 16, 2, 256, 512, 16, 32)
    large = lib.pkv_paged_decode_workspace_size(64, 16, 2, 256, 1024, 16, 32)
    auto = lib.pkv_paged_decode_workspace_size(64, 16, 2, 256, 512, 16, 0)
    assert 0 < small < large
    assert auto > 0 and auto % 256 == 0
    assert lib.pkv_paged_decode_workspace_size(1, 0, 2, 256, 8, 16, 0) == -1


@pytest.mark.parametrize(
    "call,message",
    [
        (lambda lib: lib.pkv_kv_append(None, 0, 0, None, 0, 0, None, 1, None, None, 1, 1, 16, 64, 0, 0, 0, 9, None,
                                       None), "unsupported dtype"),
        (lambda lib: lib.pkv_kv_append(None, 0, 0, None, 0, 0, None, 1, None, None, 1, 1, 16, 64, 0, 0, 0, 1, None,
                                       None), "null pointer"),
        (lambda lib: lib.pkv_paged_decode(None, 0, 0, None, None, 4, 3, 16, 64, 0, 0, 0, None, 0, 4, None, 0, 2, 16,
                                          1.0, 0, None, 0, None, 0, 0, 1, None, None), "multiple of num_kv_heads"),
        (lambda lib: lib.pkv_paged_attention_decode(None, None, 1, None, None, 1, 1, 1, 2, 8, 0, None, 0, None,
                                                    None), "sequence_length must be positive"),
        (lambda lib: lib.pkv_copy_pages(None, None, 1, 0, 4, 0, 1, 0, 0, None, None, 1, None, None), "bad sizes"),
        (lambda lib: lib.pkv_lse_merge(None, None, 0, 1, 8, None, 8, None, 0, None), "bad sizes"),
    ],
)
def test_invalid_arguments_are_rejected_on_the_host(call, message) -> None:
    lib = cuda_loader.load_paged_kv_library()
    status = call(lib)
    assert status == 1  # PKV_ERR_INVALID_ARGUMENT
    assert message in cuda_loader.last_error()


def test_empty_work_returns_ok_without_device_calls() -> None:
    lib = cuda_loader.load_paged_kv_library()
    assert lib.pkv_kv_append(None, 0, 0, None, 0, 0, None, 0, None, None, 1, 1, 16, 64, 0, 0, 0, 1, None, None) == 0
    assert lib.pkv_copy_pages(None, None, 1, 0, 4, 0, 1, 0, 16, None, None, 0, None, None) == 0


def test_output_stage_sizes_without_a_gpu() -> None:
    """Workspace and exchange-buffer sizes of the output stage (host arithmetic only)."""
    lib = cuda_loader.load_paged_kv_library()
    # hi and lo f16 planes, fp32 split-k sums (tokens x hidden), tile counters (256-byte aligned)
    assert lib.pkv_o_proj_workspace_size(64, 4096, 2048) == 2 * 64 * 4096 * 2 + 64 * 2048 * 4 + 256
    assert lib.pkv_o_proj_workspace_size(-1, 128, 128) == -1
    two = lib.pkv_o_proj_comm_bytes(2, 64, 2048, paged_kv_ops.DTYPE_BF16)
    one = lib.pkv_o_proj_comm_bytes(1, 64, 2048, paged_kv_ops.DTYPE_BF16)
    # data after a 256-byte header: two parities x world slots x capacity x hidden values, as 8-byte words
    # of two bf16 values and the call's epoch (4 bytes per value; fp32: one value per word, 8 bytes)
    assert two - one == 2 * 64 * 2048 * 4
    assert two == 256 + 2 * 2 * 64 * 2048 * 4
    assert lib.pkv_o_proj_comm_bytes(2, 64, 2048, paged_kv_ops.DTYPE_F32) == 256 + 2 * 2 * 64 * 2048 * 8
    for bad in ((0, 64, 2048), (9, 64, 2048), (2, 0, 2048), (2, 64, 100)):
        assert lib.pkv_o_proj_comm_bytes(*bad, paged_kv_ops.DTYPE_BF16) == -1
