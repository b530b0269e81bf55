"""Pins the CPU oracle against fixtures produced by the reference's own code (tests/golden/make_golden.py).

Append: the oracle's restatement of append_blocks reproduces the reference's pools bit for bit
(sha256 of every request's K and V pool). Attention: the oracle's dense decode / causal prefill over
the native shared-pool layout (built through slot mappings) matches the reference's dense attention
within the path's tolerances. Gather and the free list match the reference's decode_state results.
"""

from __future__ import annotations

import numpy as np
import pytest

import cases
import pkv_testlib as lib
from oracle import paged_kv_oracle as oracle


@pytest.mark.parametrize("make", cases.DECODE_CASES + cases.PREFILL_CASES, ids=lambda m: m.__name__)
def test_oracle_append_matches_reference_pools_bit_exact(make) -> None:
    case = make()
    g = lib.golden()
    for b, (pk, pv) in enumerate(lib.reference_layout_pools(case)):
        assert lib.sha(pk) == g[f"{case.name}/pool_k_sha/{b}"].tobytes().hex(), (case.name, b)
        assert lib.sha(pv) == g[f"{case.name}/pool_v_sha/{b}"].tobytes().hex(), (case.name, b)


@pytest.mark.parametrize("make", cases.DECODE_CASES + cases.PREFILL_CASES, ids=lambda m: m.__name__)
def test_native_pool_pages_equal_reference_repeated_heads(make) -> None:
    """Native page [p, kvh] holds what the reference stores for every repeated head kvh*G + r."""
    case = make()
    group = case.num_q_heads // case.num_kv_heads
    pk, pv, tables = lib.native_pools(case)
    ref = lib.reference_layout_pools(case)
    for b, table in enumerate(tables):
        for logical, page in enumerate(table):
            ref_page = case.tables()[b][logical]
            for kvh in range(case.num_kv_heads):
                for r in range(group):
                    assert np.array_equal(pk[page, kvh], ref[b][0][0, kvh * group + r, ref_page])
                    assert np.array_equal(pv[page, kvh], ref[b][1][0, kvh * group + r, ref_page])


@pytest.mark.parametrize("round_probs", [True, False], ids=["reference-rounding", "exact"])
@pytest.mark.parametrize("make", cases.DECODE_CASES, ids=lambda m: m.__name__)
def test_oracle_decode_matches_reference_dense_attention(make, round_probs) -> None:
    case = make()
    dtype = cases.dtype_name(case.dtype)
    pk, pv, tables = lib.native_pools(case)
    q = lib.as_f32(lib.np_bits(case.query), dtype)
    out = oracle.decode_attention(q, pk, pv, tables, case.lens, dtype=dtype, round_probs=round_probs)
    expected = lib.as_f32(lib.golden()[f"{case.name}/out"], dtype)
    # the exact mode differs from the reference by at most the reference's own rounding of probs
    extra = 0.0 if round_probs else oracle.decode_rounding_bound(q, pk, pv, tables, case.lens, dtype=dtype)
    lib.assert_close(out, expected, dtype, case.name, extra=extra)


@pytest.mark.parametrize("round_probs", [True, False], ids=["reference-rounding", "exact"])
@pytest.mark.parametrize("make", cases.PREFILL_CASES, ids=lambda m: m.__name__)
def test_oracle_prefill_matches_reference_causal_attention(make, round_probs) -> None:
    case = make()
    dtype = cases.dtype_name(case.dtype)
    pk, pv, tables = lib.native_pools(case)
    for b in range(case.batch):
        q = lib.as_f32(lib.np_bits(case.query[b]), dtype).transpose(1, 0, 2)
        out = oracle.prefill_attention(q, pk, pv, tables[b], case.lens[b], dtype=dtype,
                                       round_probs=round_probs).transpose(1, 0, 2)
        expected = lib.as_f32(lib.golden()[f"{case.name}/out/{b}"], dtype)
        extra = 0.0
        if not round_probs:
            extra = oracle.prefill_rounding_bound(q, pk, pv, tables[b], case.lens[b], dtype=dtype).transpose(1, 0, 2)
        lib.assert_close(out, expected, dtype, f"{case.name}[{b}]", extra=extra)


def test_oracle_slot_append_and_gather_match_reference_decode_state() -> None:
    g = lib.golden()
    table = g["decode_state/block_table"].tolist()
    assert table == [0, 1, 2, 3]  # tests/unit/test_decode_state.py:62
    assert int(g["decode_state/growth_events"][0]) >= 1
    pool_k = np.zeros((len(table), 2, 2, 4), dtype=np.float32)
    pool_v = np.zeros_like(pool_k)
    start = 0
    for step, seq in ((0, 3), (1, 1), (2, 1), (3, 1)):
        count = 2 * seq * 4
        key = (step * 1000.0 + np.arange(count, dtype=np.float32)).reshape(2, seq, 4).transpose(1, 0, 2)
        value = key + np.float32(0.5)
        slots = oracle.slot_mapping(table, start, seq, 2)
        oracle.append_slots(pool_k, slots, key)
        oracle.append_slots(pool_v, slots, value)
        start += seq
    valid = int(g["decode_state/valid"][0])
    assert np.array_equal(oracle.gather_blocks(pool_k, table, valid)[None], g["decode_state/k_dense"])
    assert np.array_equal(oracle.gather_blocks(pool_v, table, valid)[None], g["decode_state/v_dense"])


def test_oracle_gather_follows_reordered_table() -> None:
    g = lib.golden()
    pool = np.zeros((3, 2, 2, 4), dtype=np.float32)
    for i, page in enumerate((2, 0, 1)):
        pool[page] = (i * 1000.0 + np.arange(16, dtype=np.float32)).reshape(2, 2, 4)
    assert np.array_equal(oracle.gather_blocks(pool, [2, 0, 1], 6)[None], g["decode_state/reordered_k"])


def test_oracle_free_list_matches_reference_pool_allocator() -> None:
    g = lib.golden()
    free = None
    results: list[int] = []
    for op, arg in cases.allocator_script():
        if op == "init":
            free = oracle.FreeList(list(range(arg)))
        elif op == "allocate":
            results.extend(free.allocate(arg))
            results.append(-1)
        else:
            free.release(list(arg))
    assert results == g["allocator/results"].tolist()
    assert free.free == g["allocator/free"].tolist()


def test_oracle_lse_merge_equals_whole_context_softmax() -> None:
    rng = np.random.default_rng(5)
    keys = rng.standard_normal((300, 64)).astype(np.float32)
    values = rng.standard_normal((300, 64)).astype(np.float32)
    query = rng.standard_normal(64).astype(np.float32)
    scale = 64 ** -0.5
    outs, lses = oracle.split_decode_partials(query, keys, values, [(0, 100), (100, 256), (256, 300)], scale)
    merged, lse = oracle.lse_merge(outs[:, None, :], lses[:, None])
    whole, whole_lse = oracle.split_decode_partials(query, keys, values, [(0, 300)], scale)
    np.testing.assert_allclose(merged[0], whole[0], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(lse[0], whole_lse[0], atol=1e-5, rtol=1e-5)


def test_bf16_rounding_helpers_round_to_nearest_even() -> None:
    x = np.asarray([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 0.0], dtype=np.float32)
    bits = oracle.f32_to_bf16(x)
    back = oracle.bf16_to_f32(bits)
    assert back[0] == 1.0
    assert back[1] == 1.0  # halfway -> even
    assert back[2] == 1.015625  # halfway -> even (odd mantissa rounds up)
    assert back[3] == -2.5
    assert np.isfinite(back[4]) or np.isinf(back[4])
    assert back[5] == 0.0


@pytest.mark.parametrize("make", cases.NORM_ROPE_CASES, ids=lambda m: m.__name__)
def test_oracle_norm_rope_matches_reference_layer(make) -> None:
    """The oracle's RMSNorm + rotary composition, fed the reference's cos/sin rows, reproduces the
    query the reference's layer attends with and the key its cache stores (bit-exact except where the
    mean of squares rounds differently: at most one unit in the last place); the value is stored
    unchanged."""
    case = make()
    dtype = cases.dtype_name(case.dtype)
    g = lib.golden()
    f32 = lambda t: oracle.to_f32(cases.to_bits(t), dtype)  # noqa: E731
    kv0 = case.rank * case.local_kv_heads
    for b in range(case.batch):
        cos = oracle.to_f32(g[f"{case.name}/cos/{b}"], dtype)
        sin = oracle.to_f32(g[f"{case.name}/sin/{b}"], dtype)
        query = f32(case.q_proj[b][:, :, : case.head_dim].contiguous())
        key = f32(case.key[b])[:, kv0 : kv0 + case.local_kv_heads]
        q, k = oracle.qk_norm_rope(query, key, f32(case.q_norm), f32(case.k_norm), case.eps, cos, sin, dtype=dtype)
        lib.assert_ulp_close(q, oracle.to_f32(g[f"{case.name}/query/{b}"], dtype), dtype, f"{case.name}[{b}] query")
        lib.assert_ulp_close(k, oracle.to_f32(g[f"{case.name}/key/{b}"], dtype), dtype, f"{case.name}[{b}] key")
        np.testing.assert_array_equal(f32(case.value[b])[:, kv0 : kv0 + case.local_kv_heads],
                                      oracle.to_f32(g[f"{case.name}/value/{b}"], dtype))


@pytest.mark.parametrize("make", cases.NORM_ROPE_CASES, ids=lambda m: m.__name__)
def test_oracle_rope_table_matches_reference_to_rounding(make) -> None:
    case = make()
    dtype = cases.dtype_name(case.dtype)
    g = lib.golden()
    for b in range(case.batch):
        p0, t = case.prefix_lens[b], case.new_lens[b]
        cos, sin = oracle.rope_cos_sin(np.arange(p0, p0 + t), case.head_dim, case.partial_rotary_factor,
                                       case.rope_theta, dtype=dtype)
        lib.assert_ulp_close(cos, oracle.to_f32(g[f"{case.name}/cos/{b}"], dtype), dtype, "cos", min_exact=0.95)
        lib.assert_ulp_close(sin, oracle.to_f32(g[f"{case.name}/sin/{b}"], dtype), dtype, "sin", min_exact=0.95)


def test_oracle_e4m3_matches_torch_float8() -> None:
    """The oracle's e4m3 decoding and its round-to-nearest-even encoding equal torch's float8_e4m3fn
    (every code; random values over five decades, every midpoint between neighbours, signed zeros)."""
    import torch

    values = oracle.e4m3_values()
    torch_values = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(values, torch_values)
    gen = np.random.default_rng(3)
    x = np.concatenate([gen.standard_normal(50000).astype(np.float32) * s for s in (1, 30, 300, 1e-2, 1e-3)])
    mids = ((values[:126] + values[1:127]) / 2).astype(np.float32)
    x = np.clip(np.concatenate([x, mids, -mids, np.float32([0.0, -0.0, 448.0, -448.0])]), -448, 448)
    x = x.astype(np.float32)
    np.testing.assert_array_equal(oracle.round_to_e4m3(x),
                                  torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy())


def test_oracle_fp8_row_quantisation_bounds() -> None:
    """Rows quantise to within half an e4m3 step of their value: |x - dequant| <= 2^-4 |x| for normal
    codes (plus the subnormal step 2^-10 * scale); zero rows stay zero."""
    gen = np.random.default_rng(4)
    x = (gen.standard_normal((64, 256)) * gen.uniform(0.01, 100, (64, 1))).astype(np.float32)
    x[5] = 0.0
    codes, scales = oracle.quantize_fp8_rows(x)
    back = oracle.dequantize_fp8(codes, scales)
    assert scales[5] == 0 and np.all(back[5] == 0)
    err = np.abs(back - x)
    assert np.all(err <= np.abs(x) * 2.0 ** -4 + scales[:, None] * 2.0 ** -9 * 1.0001)
    assert np.all(np.abs(back).max(axis=1)[scales > 0] <= np.abs(x).max(axis=1)[scales > 0] * (1 + 1e-6))


@pytest.mark.parametrize("make", cases.OPROJ_CASES, ids=lambda m: m.__name__)
def test_oracle_output_stage_matches_reference(make) -> None:
    """The oracle's gate, FP8 block-scaled o_proj and all-reduce reproduce the reference's output stage
    per rank (partials) and summed: bit-identical except where the float32 GEMM order moves a value
    across a rounding boundary of the hidden dtype (within the path's tolerance; almost all equal)."""
    case = make()
    out_dtype = cases.dtype_name(case.hidden_dtype)
    g = lib.golden()
    partials = []
    for rank in range(case.world_size):
        h, hd, gt, gd, codes, scale = lib.oproj_rank_arrays(case, rank)
        x, _ = oracle.gate_heads(h, gt, hd, gd)
        p = oracle.o_proj_partial(x, codes, scale, out_dtype)
        ref = oracle.to_f32(g[f"{case.name}/partial{rank}"], out_dtype)
        lib.assert_close(p, ref, out_dtype, f"{case.name} partial {rank}")
        assert float((p == ref).mean()) >= 0.99
        partials.append(p)
    total = oracle.all_reduce_sum(partials, out_dtype)
    ref = oracle.to_f32(g[f"{case.name}/out"], out_dtype)
    lib.assert_close(total, ref, out_dtype, f"{case.name} all-reduce")
    assert float((total == ref).mean()) >= 0.99


def test_oracle_all_reduce_of_reference_partials_is_exact() -> None:
    """Fed the reference's own partials, the oracle's all-reduce equals the reference's sum bit for bit."""
    g = lib.golden()
    for make in cases.OPROJ_CASES:
        case = make()
        out_dtype = cases.dtype_name(case.hidden_dtype)
        parts = [oracle.to_f32(g[f"{case.name}/partial{r}"], out_dtype) for r in range(case.world_size)]
        np.testing.assert_array_equal(oracle.all_reduce_sum(parts, out_dtype),
                                      oracle.to_f32(g[f"{case.name}/out"], out_dtype))
