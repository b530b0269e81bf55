"""The allocation-free decode entry point, checked against the regular one through the C ABI.

pkv_paged_decode_static_scratch serves callers that cannot allocate device memory (a runtime that has
reserved its HBM for page pools, or an FFI host holding only raw pointers): it keeps its scratch in a
library-owned array instead of a caller workspace. It must give the same attention outputs as
pkv_paged_decode with a caller workspace, on consecutive calls that share the array.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import cuda_loader
import paged_kv_ops as ops
import pkv_testlib as lib

STATIC_SCRATCH_BYTES = 32 << 20


def _problem(dtype: torch.dtype, head_dim: int, lens: list[int], seed: int):
    gen = torch.Generator().manual_seed(seed)
    block_size, hq, hkv = 16, 16, 2
    need = [(n + block_size - 1) // block_size for n in lens]
    num_pages = sum(need) + 7
    perm = torch.randperm(num_pages, generator=gen)
    tables = torch.full((len(lens), max(need)), -1, dtype=torch.int32)
    used = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[used : used + n].to(torch.int32)
        used += n
    key_pool = torch.randn((num_pages, hkv, block_size, head_dim), generator=gen).to(dtype).cuda()
    value_pool = torch.randn((num_pages, hkv, block_size, head_dim), generator=gen).to(dtype).cuda()
    query = torch.randn((len(lens), hq, head_dim), generator=gen).to(dtype).cuda()
    return query, key_pool, value_pool, tables.cuda(), torch.tensor(lens, dtype=torch.int32).cuda()


def _call_static(query, key_pool, value_pool, tables, seq_lens, out, flag) -> int:
    lib_ = cuda_loader.load_paged_kv_library()
    num_pages, hkv, block_size, head_dim = key_pool.shape
    return lib_.pkv_paged_decode_static_scratch(
        query.data_ptr(), query.stride(0), query.stride(1), key_pool.data_ptr(), value_pool.data_ptr(),
        num_pages, hkv, block_size, head_dim, key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        tables.data_ptr(), tables.stride(0), tables.shape[1], seq_lens.data_ptr(), ops.INDEX_I32, query.shape[0],
        query.shape[1], head_dim ** -0.5, 0, out.data_ptr(), out.stride(0), out.stride(1),
        ops.dtype_code(query.dtype), flag.data_ptr(), torch.cuda.current_stream().cuda_stream,
    )


@pytest.mark.gpu
@pytest.mark.parametrize(
    "dtype,head_dim,lens",
    [
        (torch.float16, 128, [1, 15, 17, 300, 1024, 2049, 0, 77]),
        (torch.bfloat16, 256, [4096, 33, 1, 2500, 700]),
        (torch.float32, 64, [5, 130, 64]),
    ],
)
def test_static_scratch_decode_matches_workspace_decode_twice(dtype, head_dim, lens) -> None:
    query, key_pool, value_pool, tables, seq_lens = _problem(dtype, head_dim, lens, seed=head_dim + len(lens))
    expected = ops.paged_decode(query, key_pool, value_pool, tables, seq_lens)
    name = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32"}[dtype]
    want = lib.as_f32(lib.np_bits(expected), name)
    for _ in range(2):  # consecutive calls share the library's scratch array
        out = torch.full_like(query, float("nan"))
        flag = ops.new_error_flag(query.device)
        status = _call_static(query, key_pool, value_pool, tables, seq_lens, out, flag)
        assert status == 0, cuda_loader.last_error()
        torch.cuda.synchronize()
        assert int(flag.item()) == 0
        got = lib.as_f32(lib.np_bits(out), name)
        assert np.isfinite(got).all()
        lib.assert_close(got, want, name, "static scratch vs caller workspace")


def test_static_scratch_decode_rejects_calls_beyond_its_scratch() -> None:
    lib_ = cuda_loader.load_paged_kv_library()
    batch, hq, hkv, head_dim, max_blocks = 4096, 16, 2, 256, 4096
    assert ops.paged_decode_workspace_size(batch, hq, hkv, head_dim, max_blocks, 16, 1) > STATIC_SCRATCH_BYTES
    status = lib_.pkv_paged_decode_static_scratch(
        None, 0, 0, None, None, 1, hkv, 16, head_dim, 0, 0, 0, None, 0, max_blocks, None, 0, batch, hq, 1.0, 1,
        None, 0, 0, 1, None, None,
    )
    assert status == 1  # PKV_ERR_INVALID_ARGUMENT, nothing launched
    assert "static scratch holds" in cuda_loader.last_error()
    assert ctypes.c_int64(STATIC_SCRATCH_BYTES).value == 32 * 1024 * 1024


@pytest.mark.parametrize(
    "change,message",
    [
        ({"max_blocks": 1 << 30}, "max_blocks"),
        ({"batch": 1 << 30}, "batch"),
        ({"dtype": 7}, "dtype"),
        ({"index_dtype": 5}, "index dtype"),
        ({"num_kv_heads": 512, "num_q_heads": 512}, "KV heads"),
        ({"query": None}, "null pointer"),
    ],
)
def test_static_scratch_decode_checks_arguments_before_any_device_work(change, message) -> None:
    """A rejected call returns PKV_ERR_INVALID_ARGUMENT before it touches the device (no GPU here: a call
    that reached the CUDA runtime would fail with PKV_ERR_CUDA instead), so the shared array is never
    cleared or written for a call that is then refused."""
    lib_ = cuda_loader.load_paged_kv_library()
    fake = 1 << 20  # stands in for device addresses; a rejected call never dereferences them
    args = {"query": fake, "batch": 4, "num_q_heads": 16, "num_kv_heads": 2, "max_blocks": 8, "dtype": 1,
            "index_dtype": 0}
    args.update(change)
    status = lib_.pkv_paged_decode_static_scratch(
        args["query"], 16 * 64, 64, fake, fake, 32, args["num_kv_heads"], 16, 64, 2 * 16 * 64, 16 * 64, 64, fake,
        8, args["max_blocks"], fake, args["index_dtype"], args["batch"], args["num_q_heads"], 0.125, 0, fake, 16 * 64,
        64, args["dtype"], None, None,
    )
    assert status == 1, cuda_loader.last_error()
    assert message in cuda_loader.last_error()


@pytest.mark.gpu
def test_static_scratch_decode_after_a_call_that_flagged_a_bad_page() -> None:
    """A call whose table names a page outside the pool is bounded (the kernel skips that page and sets
    PKV_DEVERR_PAGE_OUT_OF_RANGE); the next call on the shared array must again match the regular
    entry point exactly as if the first had not happened."""
    lens = [300, 1024, 17, 2049]
    query, key_pool, value_pool, tables, seq_lens = _problem(torch.float16, 256, lens, seed=31)
    expected = ops.paged_decode(query, key_pool, value_pool, tables, seq_lens)
    want = lib.as_f32(lib.np_bits(expected), "float16")
    bad = tables.clone()
    bad[1, 3] = key_pool.shape[0] + 1000
    out = torch.empty_like(query)
    flag = ops.new_error_flag(query.device)
    assert _call_static(query, key_pool, value_pool, bad, seq_lens, out, flag) == 0, cuda_loader.last_error()
    torch.cuda.synchronize()
    assert int(flag.item()) & ops.DEVERR_PAGE_OUT_OF_RANGE
    out = torch.full_like(query, float("nan"))
    flag = ops.new_error_flag(query.device)
    assert _call_static(query, key_pool, value_pool, tables, seq_lens, out, flag) == 0, cuda_loader.last_error()
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    lib.assert_close(lib.as_f32(lib.np_bits(out), "float16"), want, "float16", "static scratch after a flagged call")
