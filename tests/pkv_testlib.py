"""Helpers shared by the tests: fixture access and oracle-side builds of the seeded cases."""

from __future__ import annotations

import hashlib
from functools import lru_cache
from pathlib import Path

import numpy as np

import cases
from oracle import paged_kv_oracle as oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden.npz"

# attention tolerances: fp32 as the reference kernel tests (tests/unit/test_fp8_cuda.py:54),
# fp16/bf16 as the north-star bar (max-abs 2e-3, relative 1e-2)
TOL = {"float32": (2e-5, 2e-5), "float16": (2e-3, 1e-2), "bfloat16": (2e-3, 1e-2)}


@lru_cache(maxsize=1)
def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN) as data:
        return {key: data[key] for key in data.files}


def golden_sha(key: str) -> str:
    return golden()[key].tobytes().hex()


def sha(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def np_bits(tensor) -> np.ndarray:
    return cases.to_bits(tensor)


def np_dtype(case) -> np.dtype:
    """numpy storage dtype of a case's tensors (bfloat16 as uint16 bits)."""
    return {"float32": np.dtype(np.float32), "float16": np.dtype(np.float16),
            "bfloat16": np.dtype(np.uint16)}[cases.dtype_name(case.dtype)]


def as_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    return oracle.to_f32(bits, dtype)


def assert_close(actual: np.ndarray, expected: np.ndarray, dtype: str, what: str = "",
                 extra: np.ndarray | float = 0.0) -> None:
    """|actual - expected| <= atol + rtol * |expected| + extra, elementwise. `extra` carries the
    reference's own probability-rounding bound when `expected` comes from the reference."""
    atol, rtol = TOL[dtype]
    actual = np.asarray(actual, dtype=np.float32)
    expected = np.asarray(expected, dtype=np.float32)
    assert actual.shape == expected.shape, (what, actual.shape, expected.shape)
    bad = ~(np.abs(actual - expected) <= atol + rtol * np.abs(expected) + extra)
    if bad.any():
        idx = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {bad.size} elements out of tolerance (atol={atol}, rtol={rtol}); "
            f"max abs err {float(np.abs(actual - expected).max()):.3e}; first at {tuple(idx)}: "
            f"{actual[tuple(idx)]} vs {expected[tuple(idx)]}"
        )


def reference_layout_pools(case) -> list[tuple[np.ndarray, np.ndarray]]:
    """Per request, the reference-layout pools (1, Hq, P, bs, D) the reference builds for `case`,
    via the oracle's restatement of append_blocks (repeated heads, zero-initialised)."""
    group = case.num_q_heads // case.num_kv_heads
    pools = []
    tables = case.tables()
    for b in range(case.batch):
        shape = (1, case.num_q_heads, case.pages_per_request, case.block_size, case.head_dim)
        dt = np_dtype(case)
        pk = np.zeros(shape, dtype=dt)
        pv = np.zeros(shape, dtype=dt)
        valid = 0
        chunks = [(case.prefix_k[b], case.prefix_v[b])]
        if isinstance(case, cases.DecodeCase):
            if case.append_new:
                chunks.append((case.new_k[b][None], case.new_v[b][None]))
        else:
            chunks.append((case.chunk_k[b], case.chunk_v[b]))
        for k, v in chunks:
            if k.shape[0] == 0:
                continue
            kk = oracle.repeat_kv(np_bits(k).transpose(1, 0, 2)[None], group)
            vv = oracle.repeat_kv(np_bits(v).transpose(1, 0, 2)[None], group)
            oracle.append_blocks_reference_layout(pk, tables[b], valid, kk)
            valid = oracle.append_blocks_reference_layout(pv, tables[b], valid, vv)
        pools.append((pk, pv))
    return pools


def shared_pool_layout(case) -> tuple[int, list[list[int]]]:
    """The native shared pool used for a case on the new path: request b's pool pages p map to
    shared page b * pages_per_request + p, so every request keeps its seeded page permutation."""
    tables = [[b * case.pages_per_request + p for p in t] for b, t in enumerate(case.tables())]
    return case.batch * case.pages_per_request, tables


def native_pools(case) -> tuple[np.ndarray, np.ndarray, list[list[int]]]:
    """Oracle build of the native (P, Hkv, bs, D) shared pools for a case, through slot mappings."""
    num_pages, tables = shared_pool_layout(case)
    shape = (num_pages, case.num_kv_heads, case.block_size, case.head_dim)
    pk = np.zeros(shape, dtype=np_dtype(case))
    pv = np.zeros(shape, dtype=np_dtype(case))
    for b in range(case.batch):
        start = 0
        chunks = [(case.prefix_k[b], case.prefix_v[b])]
        if isinstance(case, cases.DecodeCase):
            if case.append_new:
                chunks.append((case.new_k[b][None], case.new_v[b][None]))
        else:
            chunks.append((case.chunk_k[b], case.chunk_v[b]))
        for k, v in chunks:
            n = k.shape[0]
            if n == 0:
                continue
            slots = oracle.slot_mapping(tables[b], start, n, case.block_size)
            oracle.append_slots(pk, slots, np_bits(k))
            oracle.append_slots(pv, slots, np_bits(v))
            start += n
    return pk, pv, tables


def ulp_distance(actual: np.ndarray, expected: np.ndarray, dtype: str) -> np.ndarray:
    """Units in the last place of `dtype` between two float32 arrays holding dtype values."""
    if dtype == "bfloat16":
        bits = lambda x: oracle.f32_to_bf16(x).astype(np.int64)  # noqa: E731
        sign = 0x8000
    elif dtype == "float16":
        bits = lambda x: np.asarray(x, dtype=np.float16).view(np.uint16).astype(np.int64)  # noqa: E731
        sign = 0x8000
    else:
        bits = lambda x: np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.int64)  # noqa: E731
        sign = 0x80000000

    def ordered(x: np.ndarray) -> np.ndarray:
        b = bits(np.asarray(x, dtype=np.float32))
        return np.where(b & sign, -(b & (sign - 1)), b)

    return np.abs(ordered(actual) - ordered(expected))


def assert_ulp_close(actual: np.ndarray, expected: np.ndarray, dtype: str, what: str = "", *, max_ulp: int = 2,
                     min_exact: float = 0.99) -> None:
    """At least min_exact of the elements bit-identical, and every element within max_ulp units in the
    last place of dtype at the magnitude of its row (the last axis): the tolerance of a reduction whose
    order differs from the reference's, whose one-unit change in a normalised value can grow, relative
    to a small result, where the rotary sum cancels."""
    actual = np.asarray(actual, dtype=np.float32)
    expected = np.asarray(expected, dtype=np.float32)
    assert actual.shape == expected.shape, (what, actual.shape, expected.shape)
    if actual.size == 0:
        return
    bits = {"bfloat16": 7, "float16": 10, "float32": 23}[dtype]
    row_max = np.max(np.abs(expected), axis=-1, keepdims=True)
    _, exp = np.frexp(np.maximum(row_max, np.float32(2.0 ** -14)))
    ulp = np.ldexp(np.float32(1.0), exp - 1 - bits)
    err = np.abs(actual - expected)
    exact = float((ulp_distance(actual, expected, dtype) == 0).mean())
    worst = float((err / ulp).max())
    assert worst <= max_ulp and exact >= min_exact, (
        f"{what}: max {worst:.2f} row-ulp (allowed {max_ulp}), {exact:.5f} bit-identical (need {min_exact})")


def oproj_rank_arrays(case, rank: int) -> tuple[np.ndarray, str, np.ndarray, str, np.ndarray, np.ndarray]:
    """One rank's output-stage inputs as the oracle takes them: heads as (tokens, K_local) rows in the
    reference's order (heads.transpose(1, 2).reshape), gate rows, and their dtype names; e4m3 codes
    (hidden, K_local) and bf16 scale bits (hidden / 128, K_local / 128)."""
    heads, gate, weight, scale = case.rank_inputs(rank)
    hd, gd = cases.dtype_name(heads.dtype), cases.dtype_name(gate.dtype)
    b, hl, s, d = heads.shape
    h = as_f32(np_bits(heads.transpose(1, 2).reshape(b * s, hl * d)), hd)
    g = as_f32(np_bits(gate.reshape(b * s, hl * d)), gd)
    import torch

    return h, hd, g, gd, weight.contiguous().view(torch.uint8).numpy(), np_bits(scale.contiguous())


def rounding_unit(x: np.ndarray, dtype: str) -> np.ndarray:
    """One unit in the last place of `dtype` at |x| (subnormal spacing below the normal range)."""
    bits, emin = {"bfloat16": (7, -126), "float16": (10, -14), "float32": (23, -126)}[dtype]
    _, e = np.frexp(np.maximum(np.abs(np.asarray(x, dtype=np.float32)), np.float32(2.0 ** emin)))
    return np.ldexp(np.float32(1.0), e - 1 - bits)


def partial_rounding_bound(partials, dtype: str) -> np.ndarray | float:
    """The reference rounds every rank's partial to the hidden dtype before the all-reduce
    (src/tp_runtime.py:693-695): a partial that lies next to a rounding boundary may round the other
    way under another summation order, moving the sum by one unit of that partial. With one rank the
    output rounding itself is covered by the tolerance."""
    if len(partials) <= 1:
        return 0.0
    return sum(rounding_unit(p, dtype) for p in partials)
