"""GPU parity of chunked-prefill paged causal attention (pkv_paged_prefill) against the reference's
dense causal prefill (fixtures) and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
import pkv_testlib as lib
from oracle import paged_kv_oracle as oracle

pytestmark = pytest.mark.gpu
DEVICE = "cuda:0"


def _ops():
    import paged_kv_ops

    return paged_kv_ops


def _build(case, index_dtype=torch.int32):
    """Pools with every request's prefix + chunk appended through kv_append (one call per chunk)."""
    ops = _ops()
    num_pages, tables = lib.shared_pool_layout(case)
    shape = (num_pages, case.num_kv_heads, case.block_size, case.head_dim)
    key_pool = torch.zeros(shape, dtype=case.dtype, device=DEVICE)
    value_pool = torch.zeros(shape, dtype=case.dtype, device=DEVICE)
    for b in range(case.batch):
        start = 0
        for k, v in ((case.prefix_k[b], case.prefix_v[b]), (case.chunk_k[b], case.chunk_v[b])):
            if k.shape[0] == 0:
                continue
            slots = torch.from_numpy(oracle.slot_mapping(tables[b], start, k.shape[0], case.block_size)).to(DEVICE)
            ops.kv_append(k.to(DEVICE), v.to(DEVICE), slots, key_pool, value_pool)
            start += k.shape[0]
    bt = torch.from_numpy(oracle.padded_block_tables(tables)).to(DEVICE, index_dtype)
    lens = torch.tensor(case.lens, dtype=index_dtype, device=DEVICE)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(case.chunk_lens)]), dtype=torch.int32, device=DEVICE)
    query = torch.cat(case.query).to(DEVICE)
    return key_pool, value_pool, tables, bt, lens, cu, query


@pytest.mark.parametrize("make", cases.PREFILL_CASES, ids=lambda m: m.__name__)
@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("round_probs", [False, True], ids=["exact_p", "round_p"])
def test_paged_prefill_matches_reference_fixture_and_oracle(make, index_dtype, round_probs) -> None:
    """Exact probabilities: within the tolerance of the exact oracle. Rounded probabilities (the
    reference's own probs.to(dtype)): within the tolerance plus the oracle's bound of that rounding, against
    both the exact oracle and the reference's fixture."""
    ops = _ops()
    case = make()
    dtype = cases.dtype_name(case.dtype)
    key_pool, value_pool, tables, bt, lens, cu, query = _build(case, index_dtype)
    flag = ops.new_error_flag(DEVICE)
    out = ops.paged_prefill(query, cu, key_pool, value_pool, bt, lens, error_flag=flag, round_probs=round_probs)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    pk, pv, _ = lib.native_pools(case)
    got_all = lib.as_f32(lib.np_bits(out), dtype)
    offset = 0
    for b in range(case.batch):
        t = case.chunk_lens[b]
        got = got_all[offset : offset + t]
        q = lib.as_f32(lib.np_bits(case.query[b]), dtype).transpose(1, 0, 2)
        exact = oracle.prefill_attention(q, pk, pv, tables[b], case.lens[b], dtype=dtype,
                                         round_probs=False).transpose(1, 0, 2)
        bound = oracle.prefill_rounding_bound(q, pk, pv, tables[b], case.lens[b], dtype=dtype).transpose(1, 0, 2)
        lib.assert_close(got, exact, dtype, f"{case.name}[{b}] vs oracle", extra=bound if round_probs else 0.0)
        ref = lib.as_f32(lib.golden()[f"{case.name}/out/{b}"], dtype)
        lib.assert_close(got, ref, dtype, f"{case.name}[{b}] vs reference", extra=bound)
        offset += t


@pytest.mark.parametrize(
    "dtype,head_dim,hq,hkv,block_size",
    [
        (torch.bfloat16, 256, 16, 2, 16),  # the chunked-prefill configuration's shape (tensor cores)
        (torch.float16, 256, 8, 1, 32),  # TP=2 rank layout, block_size 32 (tensor cores)
        (torch.float16, 128, 16, 4, 16),  # group 4 -> generic path
        (torch.float32, 64, 8, 2, 16),  # fp32 -> generic path
    ],
)
@pytest.mark.parametrize("round_probs", [False, True], ids=["exact_p", "round_p"])
def test_paged_prefill_shapes_match_oracle(dtype, head_dim, hq, hkv, block_size, round_probs) -> None:
    case = cases.make_prefill_case("shape", prefix_lens=[0, 53, 200], chunk_lens=[70, 1, 96], dtype=dtype,
                                   head_dim=head_dim, seed=head_dim + hq, num_q_heads=hq, num_kv_heads=hkv,
                                   block_size=block_size, pages_per_request=24)
    ops = _ops()
    name = cases.dtype_name(dtype)
    key_pool, value_pool, tables, bt, lens, cu, query = _build(case)
    out = ops.paged_prefill(query, cu, key_pool, value_pool, bt, lens, round_probs=round_probs)
    pk, pv, _ = lib.native_pools(case)
    got_all = lib.as_f32(lib.np_bits(out), name)
    offset = 0
    for b in range(case.batch):
        t = case.chunk_lens[b]
        q = lib.as_f32(lib.np_bits(case.query[b]), name).transpose(1, 0, 2)
        exact = oracle.prefill_attention(q, pk, pv, tables[b], case.lens[b], dtype=name,
                                         round_probs=False).transpose(1, 0, 2)
        bound = 0.0
        if round_probs and name != "float32":
            bound = oracle.prefill_rounding_bound(q, pk, pv, tables[b], case.lens[b], dtype=name).transpose(1, 0, 2)
        lib.assert_close(got_all[offset : offset + t], exact, name, f"request {b}", extra=bound)
        offset += t


def test_paged_prefill_large_chunk_sampled_rows_and_unwritten_garbage() -> None:
    """A chunk of 2048 tokens on a 3000-token prefix (bf16, head_dim 256): rows sampled across the chunk
    match the oracle, and NaN in never-written tail slots of the last page does not leak."""
    ops = _ops()
    gen = torch.Generator().manual_seed(31)
    prefix, chunk, hq, hkv, d, bs = 3000, 2048, 16, 2, 256, 16
    total = prefix + chunk
    pages = (total + bs - 1) // bs
    perm = torch.randperm(pages + 5, generator=gen)[:pages].tolist()
    key_pool = torch.randn((pages + 5, hkv, bs, d), generator=gen).bfloat16()
    value_pool = torch.randn((pages + 5, hkv, bs, d), generator=gen).bfloat16()
    last = perm[-1]
    used_in_last = total - (pages - 1) * bs
    key_pool[last, :, used_in_last:] = float("nan")
    value_pool[last, :, used_in_last:] = float("nan")
    query = torch.randn((chunk, hq, d), generator=gen).bfloat16()
    out = ops.paged_prefill(query.to(DEVICE), torch.tensor([0, chunk], dtype=torch.int32, device=DEVICE),
                            key_pool.to(DEVICE), value_pool.to(DEVICE),
                            torch.tensor([perm], dtype=torch.int32, device=DEVICE),
                            torch.tensor([total], dtype=torch.int32, device=DEVICE))
    got = lib.as_f32(lib.np_bits(out), "bfloat16")
    assert np.isfinite(got).all()
    rows = [0, 1, 15, 16, 17, 511, 1024, 2046, 2047]
    pk, pv = lib.np_bits(key_pool), lib.np_bits(value_pool)
    q = lib.as_f32(lib.np_bits(query), "bfloat16")
    for r in rows:
        pos = prefix + r
        exp = oracle.prefill_attention(q[r : r + 1].transpose(1, 0, 2), pk, pv, perm, pos + 1, dtype="bfloat16",
                                       round_probs=False)
        lib.assert_close(got[r], exp.transpose(1, 0, 2)[0], "bfloat16", f"row {r}")


@pytest.mark.parametrize(
    "dtype,head_dim,hq,hkv,block_size",
    [
        (torch.bfloat16, 64, 4, 4, 16),  # G = 1: 128 tokens per tile
        (torch.float16, 128, 4, 2, 32),  # G = 2
        (torch.bfloat16, 128, 16, 1, 64),  # G = 16: 8 tokens per tile
        (torch.float16, 256, 32, 2, 16),  # G = 16 at head_dim 256
        (torch.bfloat16, 128, 6, 2, 16),  # G = 3 -> generic path
    ],
)
def test_paged_prefill_group_sizes_match_oracle(dtype, head_dim, hq, hkv, block_size) -> None:
    case = cases.make_prefill_case("groups", prefix_lens=[0, 130, 17], chunk_lens=[200, 129, 1], dtype=dtype,
                                   head_dim=head_dim, seed=hq * 7 + hkv, num_q_heads=hq, num_kv_heads=hkv,
                                   block_size=block_size, pages_per_request=(400 + block_size - 1) // block_size)
    ops = _ops()
    name = cases.dtype_name(dtype)
    key_pool, value_pool, tables, bt, lens, cu, query = _build(case)
    flag = ops.new_error_flag(DEVICE)
    out = ops.paged_prefill(query, cu, key_pool, value_pool, bt, lens, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    pk, pv, _ = lib.native_pools(case)
    got_all = lib.as_f32(lib.np_bits(out), name)
    offset = 0
    for b in range(case.batch):
        t = case.chunk_lens[b]
        q = lib.as_f32(lib.np_bits(case.query[b]), name).transpose(1, 0, 2)
        exact = oracle.prefill_attention(q, pk, pv, tables[b], case.lens[b], dtype=name,
                                         round_probs=False).transpose(1, 0, 2)
        lib.assert_close(got_all[offset : offset + t], exact, name, f"request {b}")
        offset += t


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_paged_prefill_growing_scores_rescale_accumulator(dtype) -> None:
    """Scores that grow along the context move every row's running max by more than 2^8 several times,
    so the accumulator is rescaled in place between tiles; the result still matches the oracle."""
    ops = _ops()
    name = cases.dtype_name(dtype)
    gen = torch.Generator().manual_seed(41)
    prefix, chunk, hq, hkv, d, bs = 700, 300, 16, 2, 128, 16
    total = prefix + chunk
    pages = (total + bs - 1) // bs
    perm = torch.randperm(pages + 3, generator=gen)[:pages].tolist()
    u = torch.randn((hkv, d), generator=gen)
    pos = torch.arange(total, dtype=torch.float32)[:, None, None]
    keys = 0.5 * torch.randn((total, hkv, d), generator=gen) + u[None] * (pos / 150.0)
    values = torch.randn((total, hkv, d), generator=gen)
    key_pool = torch.zeros((pages + 3, hkv, bs, d))
    value_pool = torch.zeros((pages + 3, hkv, bs, d))
    for p in range(total):
        key_pool[perm[p // bs], :, p % bs] = keys[p]
        value_pool[perm[p // bs], :, p % bs] = values[p]
    query = (u.repeat_interleave(hq // hkv, dim=0)[None] + 0.5 * torch.randn((chunk, hq, d), generator=gen))
    key_pool, value_pool, query = key_pool.to(dtype), value_pool.to(dtype), query.to(dtype)
    flag = ops.new_error_flag(DEVICE)
    out = ops.paged_prefill(query.to(DEVICE), torch.tensor([0, chunk], dtype=torch.int32, device=DEVICE),
                            key_pool.to(DEVICE), value_pool.to(DEVICE),
                            torch.tensor([perm], dtype=torch.int32, device=DEVICE),
                            torch.tensor([total], dtype=torch.int32, device=DEVICE), error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    got = lib.as_f32(lib.np_bits(out), name)
    pk, pv = lib.np_bits(key_pool), lib.np_bits(value_pool)
    q = lib.as_f32(lib.np_bits(query), name).transpose(1, 0, 2)
    exact = oracle.prefill_attention(q, pk, pv, perm, total, dtype=name, round_probs=False).transpose(1, 0, 2)
    lib.assert_close(got, exact, name, "growing scores")


def test_paged_prefill_strided_query_rows() -> None:
    """Queries read with their own token and head strides (a head-padded projection buffer): the tensor-core
    path loads each row directly, so the result matches the contiguous call."""
    ops = _ops()
    case = cases.make_prefill_case("strided", prefix_lens=[40, 300], chunk_lens=[77, 150], dtype=torch.bfloat16,
                                   head_dim=128, seed=5, num_q_heads=16, num_kv_heads=2, pages_per_request=30)
    key_pool, value_pool, tables, bt, lens, cu, query = _build(case)
    wide = torch.full((query.shape[0], query.shape[1], 192), float("nan"), dtype=query.dtype, device=DEVICE)
    wide[:, :, :128] = query
    strided = wide[:, :, :128]
    assert strided.stride(1) == 192
    flag = ops.new_error_flag(DEVICE)
    got = ops.paged_prefill(strided, cu, key_pool, value_pool, bt, lens, error_flag=flag)
    ref = ops.paged_prefill(query, cu, key_pool, value_pool, bt, lens, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    assert torch.equal(got.contiguous(), ref)


@pytest.mark.parametrize("group,head_dim", [(8, 128), (2, 64), (16, 256)])
def test_paged_prefill_many_ragged_requests_every_token(group, head_dim) -> None:
    """More requests than a warp has lanes, chunks of 0 to 150 tokens on prefixes of 0 to 400: the
    tensor-core kernel orders its CTAs longest-first from the lengths on the device, and every token of
    every chunk must come out once, matching the oracle."""
    ops = _ops()
    gen = torch.Generator().manual_seed(40 + group)
    hkv, bs = 2, 16
    hq = hkv * group
    batch = 37
    chunk = [int(x) for x in torch.randint(0, 151, (batch,), generator=gen)]
    chunk[3] = 0
    prefix = [int(x) for x in torch.randint(0, 401, (batch,), generator=gen)]
    lens = [p + c for p, c in zip(prefix, chunk)]
    need = [max(1, (n + bs - 1) // bs) for n in lens]
    pages = sum(need) + 2
    perm = torch.randperm(pages, generator=gen).tolist()
    tables, used = [], 0
    for n in need:
        tables.append(perm[used:used + n])
        used += n
    key_pool = torch.randn((pages, hkv, bs, head_dim), generator=gen).to(torch.bfloat16)
    value_pool = torch.randn((pages, hkv, bs, head_dim), generator=gen).to(torch.bfloat16)
    query = torch.randn((sum(chunk), hq, head_dim), generator=gen).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(chunk)]), dtype=torch.int32)
    bt = torch.from_numpy(oracle.padded_block_tables(tables)).to(torch.int32)
    flag = ops.new_error_flag(DEVICE)
    out = ops.paged_prefill(query.to(DEVICE), cu.to(DEVICE), key_pool.to(DEVICE), value_pool.to(DEVICE), bt.to(DEVICE),
                            torch.tensor(lens, dtype=torch.int32, device=DEVICE), error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    got = lib.as_f32(lib.np_bits(out), "bfloat16")
    pk, pv = lib.np_bits(key_pool), lib.np_bits(value_pool)
    for b in range(batch):
        if chunk[b] == 0:
            continue
        rows = slice(int(cu[b]), int(cu[b + 1]))
        q = lib.as_f32(lib.np_bits(query[rows]), "bfloat16").transpose(1, 0, 2)
        expected = oracle.prefill_attention(q, pk, pv, tables[b], lens[b], dtype="bfloat16",
                                            round_probs=False).transpose(1, 0, 2)
        lib.assert_close(got[rows], expected, "bfloat16", f"request {b}")
