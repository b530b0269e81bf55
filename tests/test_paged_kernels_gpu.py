"""GPU parity of the sm_100a kernels against the oracle and the reference fixtures.

Every test goes through the C ABI (paged_kv_ops -> libqwen36_paged_kv.so). Append, gather and page
copy must be bit-exact; attention must be within the tolerances of pkv_testlib.TOL. Several tests
mirror the reference's own kernel tests (tests/unit/test_fp8_cuda.py:37-199) on the reference-named
entry points.
"""

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


def _to_dev(array: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    if dtype == torch.bfloat16:
        return torch.from_numpy(array.view(np.int16).copy()).view(torch.bfloat16).to(DEVICE)
    return torch.from_numpy(np.ascontiguousarray(array)).to(DEVICE)


def _append_case(case, key_pool, value_pool, tables, index_dtype=torch.int64):
    """Appends every chunk of a case through kv_append (one call per chunk of all requests)."""
    ops = _ops()
    flag = ops.new_error_flag(DEVICE)
    chunks_per_request = []
    for b in range(case.batch):
        chunks = [(case.prefix_k[b], case.prefix_v[b])]
        if isinstance(case, cases.DecodeCase):
            if case.append_new:
                chunks.append((case.new_k[b][None], case.new_v[b][None]))
        else:
            chunks.append((case.chunk_k[b], case.chunk_v[b]))
        chunks_per_request.append(chunks)
    starts = [0] * case.batch
    for step in range(2):
        ks, vs, slots = [], [], []
        for b in range(case.batch):
            if step >= len(chunks_per_request[b]):
                continue
            k, v = chunks_per_request[b][step]
            if k.shape[0] == 0:
                continue
            ks.append(k)
            vs.append(v)
            slots.append(oracle.slot_mapping(tables[b], starts[b], k.shape[0], case.block_size))
            starts[b] += k.shape[0]
        if not ks:
            continue
        key = torch.cat(ks).to(DEVICE)
        value = torch.cat(vs).to(DEVICE)
        slot = torch.from_numpy(np.concatenate(slots)).to(DEVICE)
        ops.kv_append(key, value, slot, key_pool, value_pool, error_flag=flag)
    assert int(flag.item()) == 0


def _device_pools(case):
    num_pages, tables = lib.shared_pool_layout(case)
    shape = (num_pages, case.num_kv_heads, case.block_size, case.head_dim)
    key_pool = torch.zeros(shape, dtype=case.dtype, device=DEVICE)
    value_pool = torch.zeros(shape, dtype=case.dtype, device=DEVICE)
    _append_case(case, key_pool, value_pool, tables)
    return key_pool, value_pool, tables


def _tables_tensor(tables, index_dtype):
    return torch.from_numpy(oracle.padded_block_tables(tables)).to(DEVICE, index_dtype)


# ---- a1 append ----------------------------------------------------------------------------------------------
@pytest.mark.parametrize("make", cases.DECODE_CASES + cases.PREFILL_CASES, ids=lambda m: m.__name__)
def test_kv_append_is_bit_exact_with_oracle_and_reference(make) -> None:
    case = make()
    key_pool, value_pool, _ = _device_pools(case)
    pk, pv, _ = lib.native_pools(case)
    assert np.array_equal(lib.np_bits(key_pool), pk)
    assert np.array_equal(lib.np_bits(value_pool), pv)


def test_kv_append_strided_source_and_padding_slots() -> None:
    ops = _ops()
    torch.manual_seed(3)
    pool_k = torch.zeros((6, 2, 16, 64), dtype=torch.float16, device=DEVICE)
    pool_v = torch.zeros_like(pool_k)
    # key/value as non-contiguous views (token stride != heads * head_dim)
    big = torch.randn((5, 3, 64), dtype=torch.float16, device=DEVICE)
    key = big[:, :2]
    value = big[:, 1:]
    slots = torch.tensor([17, -1, 0, 95, 40], dtype=torch.int64, device=DEVICE)
    ops.kv_append(key, value, slots, pool_k, pool_v)
    ref_k = np.zeros((6, 2, 16, 64), dtype=np.float16)
    ref_v = np.zeros_like(ref_k)
    oracle.append_slots(ref_k, slots.cpu().numpy(), key.cpu().numpy())
    oracle.append_slots(ref_v, slots.cpu().numpy(), value.cpu().numpy())
    assert np.array_equal(pool_k.cpu().numpy(), ref_k)
    assert np.array_equal(pool_v.cpu().numpy(), ref_v)


def test_kv_append_flags_out_of_range_slot_without_writing() -> None:
    ops = _ops()
    pool_k = torch.zeros((2, 1, 16, 64), dtype=torch.bfloat16, device=DEVICE)
    pool_v = torch.zeros_like(pool_k)
    key = torch.ones((2, 1, 64), dtype=torch.bfloat16, device=DEVICE)
    slots = torch.tensor([3, 32], dtype=torch.int64, device=DEVICE)  # 32 == num_pages * block_size
    flag = ops.new_error_flag(DEVICE)
    ops.kv_append(key, key, slots, pool_k, pool_v, error_flag=flag)
    assert int(flag.item()) & 2  # PKV_DEVERR_SLOT_OUT_OF_RANGE
    assert float(pool_k.float().sum().item()) == 64.0  # only slot 3 was written


# ---- a3 gather -----------------------------------------------------------------------------------------------
@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_kv_gather_matches_oracle_batch_kv(index_dtype) -> None:
    ops = _ops()
    case = cases.decode_fp16()
    key_pool, value_pool, tables = _device_pools(case)
    bt = _tables_tensor(tables, index_dtype)
    lens = torch.tensor(case.lens, dtype=index_dtype, device=DEVICE)
    k, v = ops.kv_gather(key_pool, value_pool, bt, lens)
    pk, pv, _ = lib.native_pools(case)
    ek, mask = oracle.batch_kv(pk, tables, case.lens)
    ev, _ = oracle.batch_kv(pv, tables, case.lens)
    assert np.array_equal(lib.np_bits(k), ek)
    assert np.array_equal(lib.np_bits(v), ev)


# ---- a4-a6 decode ----------------------------------------------------------------------------------------------
@pytest.mark.parametrize("make", cases.DECODE_CASES, ids=lambda m: m.__name__)
@pytest.mark.parametrize("pages_per_split", [0, 1, 3])
@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_paged_decode_matches_reference_fixture(make, pages_per_split, index_dtype) -> None:
    ops = _ops()
    case = make()
    dtype = cases.dtype_name(case.dtype)
    key_pool, value_pool, tables = _device_pools(case)
    bt = _tables_tensor(tables, index_dtype)
    lens = torch.tensor(case.lens, dtype=index_dtype, device=DEVICE)
    flag = ops.new_error_flag(DEVICE)
    out = ops.paged_decode(case.query.to(DEVICE), key_pool, value_pool, bt, lens, pages_per_split=pages_per_split,
                           error_flag=flag)
    assert int(flag.item()) == 0
    expected = lib.as_f32(lib.golden()[f"{case.name}/out"], dtype)
    pk, pv, _ = lib.native_pools(case)
    q = lib.as_f32(lib.np_bits(case.query), dtype)
    bound = oracle.decode_rounding_bound(q, pk, pv, tables, case.lens, dtype=dtype)
    lib.assert_close(lib.as_f32(lib.np_bits(out), dtype), expected, dtype, f"{case.name} vs reference", extra=bound)
    lib.assert_close(lib.as_f32(lib.np_bits(out), dtype), oracle.decode_attention(q, pk, pv, tables, case.lens,
                     dtype=dtype, round_probs=False), dtype, f"{case.name} vs oracle")


@pytest.mark.parametrize(
    "dtype,head_dim,block_size,hq,hkv",
    [
        (torch.float16, 64, 16, 8, 8),  # MHA (group 1)
        (torch.bfloat16, 128, 32, 16, 2),  # block_size 32: two tiles per page
        (torch.float16, 256, 16, 8, 1),  # one KV head per rank (TP=2 layout)
        (torch.float16, 80, 16, 16, 2),  # head_dim 80 -> generic path
        (torch.bfloat16, 128, 8, 16, 2),  # block_size 8 -> generic path
        (torch.float16, 64, 16, 32, 2),  # group 16 -> generic path
        (torch.float32, 128, 16, 16, 2),  # fp32 -> generic path
    ],
)
def test_paged_decode_shapes_match_oracle(dtype, head_dim, block_size, hq, hkv) -> None:
    ops = _ops()
    gen = torch.Generator().manual_seed(head_dim * 131 + block_size + hq)
    lens = [1, block_size - 1, block_size, block_size + 1, 7 * block_size + 3, 300]
    num_pages = sum((x + block_size - 1) // block_size for x in lens) + 5
    perm = torch.randperm(num_pages, generator=gen).tolist()
    tables, used = [], 0
    for x in lens:
        n = (x + block_size - 1) // block_size
        tables.append(perm[used : used + n])
        used += n
    key_pool = torch.randn((num_pages, hkv, block_size, head_dim), generator=gen).to(dtype)
    value_pool = torch.randn((num_pages, hkv, block_size, head_dim), generator=gen).to(dtype)
    query = torch.randn((len(lens), hq, head_dim), generator=gen).to(dtype)
    name = cases.dtype_name(dtype)
    expected = oracle.decode_attention(lib.as_f32(lib.np_bits(query), name), lib.np_bits(key_pool),
                                       lib.np_bits(value_pool), tables, lens, dtype=name, round_probs=False)
    for pps in (0, 2):
        out = ops.paged_decode(query.to(DEVICE), key_pool.to(DEVICE), value_pool.to(DEVICE),
                               _tables_tensor(tables, torch.int32),
                               torch.tensor(lens, dtype=torch.int32, device=DEVICE), pages_per_split=pps)
        lib.assert_close(lib.as_f32(lib.np_bits(out), name), expected, name, f"pps={pps}")


def test_paged_decode_garbage_in_unused_slots_does_not_leak() -> None:
    """NaN/Inf bit patterns in the unused tail slots of a page must not reach the output."""
    ops = _ops()
    gen = torch.Generator().manual_seed(9)
    key_pool = torch.randn((4, 2, 16, 128), generator=gen).half()
    value_pool = torch.randn((4, 2, 16, 128), generator=gen).half()
    query = torch.randn((2, 16, 128), generator=gen).half()
    lens = [21, 5]
    tables = [[2, 0], [3]]
    key_pool[0, :, 5:] = float("nan")
    value_pool[0, :, 5:] = float("inf")
    key_pool[3, :, 5:] = float("nan")
    value_pool[3, :, 5:] = float("nan")
    key_pool[1] = float("nan")  # a page no table references
    expected = oracle.decode_attention(query.float().numpy(), key_pool.numpy(), value_pool.numpy(), tables, lens,
                                       dtype="float16", round_probs=False)
    out = ops.paged_decode(query.to(DEVICE), key_pool.to(DEVICE), value_pool.to(DEVICE),
                           _tables_tensor(tables, torch.int32), torch.tensor(lens, dtype=torch.int32, device=DEVICE))
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    lib.assert_close(got, expected, "float16", "garbage tails")


def test_paged_decode_flags_bad_page_id() -> None:
    ops = _ops()
    pool = torch.randn((4, 2, 16, 64), dtype=torch.float16, device=DEVICE)
    query = torch.randn((2, 16, 64), dtype=torch.float16, device=DEVICE)
    tables = torch.tensor([[0, 1], [2, 9]], dtype=torch.int32, device=DEVICE)  # 9 is outside the pool
    lens = torch.tensor([20, 30], dtype=torch.int32, device=DEVICE)
    flag = ops.new_error_flag(DEVICE)
    out = ops.paged_decode(query, pool, pool, tables, lens, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & 1  # PKV_DEVERR_PAGE_OUT_OF_RANGE
    assert torch.isfinite(out[0].float()).all()


def test_paged_decode_rejects_too_small_workspace() -> None:
    ops = _ops()
    pool = torch.zeros((4, 2, 16, 64), dtype=torch.float16, device=DEVICE)
    query = torch.zeros((2, 16, 64), dtype=torch.float16, device=DEVICE)
    tables = torch.zeros((2, 2), dtype=torch.int32, device=DEVICE)
    lens = torch.ones(2, dtype=torch.int32, device=DEVICE)
    workspace = torch.empty(256, dtype=torch.uint8, device=DEVICE)
    with pytest.raises(RuntimeError, match="workspace"):
        ops.paged_decode(query, pool, pool, tables, lens, workspace=workspace)


def test_lse_merge_matches_oracle() -> None:
    ops = _ops()
    rng = np.random.default_rng(4)
    parts = rng.standard_normal((5, 7, 96)).astype(np.float32)
    lse = rng.standard_normal((5, 7)).astype(np.float32) * 3
    lse[2, 3] = -np.inf
    out, out_lse = ops.lse_merge(torch.from_numpy(parts).to(DEVICE), torch.from_numpy(lse).to(DEVICE))
    exp_out, exp_lse = oracle.lse_merge(parts, lse)
    np.testing.assert_allclose(out.cpu().numpy(), exp_out, atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(out_lse.cpu().numpy(), exp_lse, atol=1e-5, rtol=1e-5)


# ---- a10 page copy --------------------------------------------------------------------------------------------
@pytest.mark.parametrize("layers", [1, 3])
def test_kv_copy_pages_bit_exact(layers) -> None:
    ops = _ops()
    gen = torch.Generator().manual_seed(layers)
    shape = (layers, 40, 2, 16, 128)
    key_pools = torch.randn(shape, generator=gen).half()
    value_pools = torch.randn(shape, generator=gen).half()
    src = [39, 38, 30, 25, 21]
    dst = [0, 3, 4, 7, 12]
    ek = key_pools.numpy().copy()
    ev = value_pools.numpy().copy()
    for layer in range(layers):
        oracle.copy_pages(ek[layer], src, dst)
        oracle.copy_pages(ev[layer], src, dst)
    kd, vd = key_pools.to(DEVICE), value_pools.to(DEVICE)
    flag = ops.new_error_flag(DEVICE)
    ops.kv_copy_pages(kd, vd, torch.tensor(src, device=DEVICE), torch.tensor(dst, device=DEVICE), error_flag=flag)
    assert int(flag.item()) == 0
    assert np.array_equal(kd.cpu().numpy(), ek)
    assert np.array_equal(vd.cpu().numpy(), ev)


def test_kv_copy_pages_then_remapped_table_gathers_same_tokens() -> None:
    """The compaction invariant: after copying src->dst and remapping the table, as_tensors-style gathers
    are unchanged (the page-copy oracle composition)."""
    ops = _ops()
    case = cases.decode_bf16()
    key_pool, value_pool, tables = _device_pools(case)
    lens = torch.tensor(case.lens, dtype=torch.int64, device=DEVICE)
    before = ops.kv_gather(key_pool, value_pool, _tables_tensor(tables, torch.int64), lens)
    used = sorted({p for t in tables for p in t})
    free = [p for p in range(key_pool.shape[0]) if p not in set(used)]
    moves = dict(zip(used[-len(free):][::-1][:10], free[:10]))
    src = list(moves.keys())
    dst = list(moves.values())
    ops.kv_copy_pages(key_pool, value_pool, torch.tensor(src, device=DEVICE), torch.tensor(dst, device=DEVICE))
    remapped = [[moves.get(p, p) for p in t] for t in tables]
    after = ops.kv_gather(key_pool, value_pool, _tables_tensor(remapped, torch.int64), lens)
    assert torch.equal(before[0], after[0]) and torch.equal(before[1], after[1])


# ---- reference entry points (mirror tests/unit/test_fp8_cuda.py:37-199) ------------------------------------------
def _dense_ref(query, dense_key, dense_value):
    scores = torch.matmul(query.float(), dense_key.float().transpose(2, 3)) * (query.shape[-1] ** -0.5)
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32)
    return torch.matmul(probs, dense_value.float())


def _pack(dense_key, dense_value, block_table, block_size, physical_blocks=None, fill=0.0):
    batch, heads, seq_len, head_dim = dense_key.shape
    if physical_blocks is None:
        physical_blocks = int(block_table.max().item()) + 1
    kb = torch.full((batch, heads, physical_blocks, block_size, head_dim), fill, device=dense_key.device,
                    dtype=dense_key.dtype)
    vb = torch.full_like(kb, fill)
    for token in range(seq_len):
        physical = int(block_table[token // block_size].item())
        kb[:, :, physical, token % block_size] = dense_key[:, :, token]
        vb[:, :, physical, token % block_size] = dense_value[:, :, token]
    return kb, vb


def test_reference_api_decode_contiguous_blocks() -> None:
    from fp8_cuda import paged_attention_decode

    torch.manual_seed(101)
    batch, heads, seq_len, head_dim, block_size = 1, 3, 5, 8, 2
    query = torch.randn((batch, heads, 1, head_dim), device=DEVICE)
    dk = torch.randn((batch, heads, seq_len, head_dim), device=DEVICE)
    dv = torch.randn((batch, heads, seq_len, head_dim), device=DEVICE)
    table = torch.arange((seq_len + block_size - 1) // block_size, device=DEVICE, dtype=torch.long)
    kb, vb = _pack(dk, dv, table, block_size)
    out = paged_attention_decode(query, table, kb, vb, seq_len, block_size)
    torch.testing.assert_close(out, _dense_ref(query, dk, dv), atol=2e-5, rtol=2e-5)


def test_reference_api_decode_non_contiguous_blocks_ignores_padding() -> None:
    from fp8_cuda import paged_attention_decode

    torch.manual_seed(102)
    batch, heads, seq_len, head_dim, block_size = 1, 2, 5, 8, 2
    query = torch.randn((batch, heads, 1, head_dim), device=DEVICE)
    dk = torch.randn((batch, heads, seq_len, head_dim), device=DEVICE)
    dv = torch.randn((batch, heads, seq_len, head_dim), device=DEVICE)
    table = torch.tensor([2, 0, 3], device=DEVICE, dtype=torch.long)
    kb, vb = _pack(dk, dv, table, block_size, physical_blocks=4, fill=1000.0)
    out = paged_attention_decode(query, table, kb, vb, seq_len, block_size)
    torch.testing.assert_close(out, _dense_ref(query, dk, dv), atol=2e-5, rtol=2e-5)


def test_reference_api_decode_rejects_mixed_dtypes() -> None:
    from fp8_cuda import paged_attention_decode

    query = torch.zeros((1, 1, 1, 8), device=DEVICE, dtype=torch.float16)
    table = torch.tensor([0], device=DEVICE, dtype=torch.long)
    kb = torch.zeros((1, 1, 1, 2, 8), device=DEVICE, dtype=torch.float32)
    with pytest.raises(RuntimeError, match="query must be float32"):
        paged_attention_decode(query, table, kb, kb.clone(), 1, 2)


def test_reference_api_batched_per_request_pools() -> None:
    from fp8_cuda import paged_attention_decode_batched

    torch.manual_seed(103)
    heads, head_dim, block_size = 3, 8, 2
    seq_lens = (3, 5, 8)
    rows = [torch.tensor(t, device=DEVICE, dtype=torch.long) for t in ([1, 0], [2, 0, 1], [0, 3, 1, 2])]
    block_tables = torch.full((3, 4), -1, device=DEVICE, dtype=torch.long)
    query = torch.randn((3, heads, 1, head_dim), device=DEVICE)
    kbs, vbs, refs = [], [], []
    for row, seq_len in enumerate(seq_lens):
        dk = torch.randn((1, heads, seq_len, head_dim), device=DEVICE)
        dv = torch.randn((1, heads, seq_len, head_dim), device=DEVICE)
        block_tables[row, : rows[row].numel()] = rows[row]
        kb, vb = _pack(dk, dv, rows[row], block_size, physical_blocks=int(rows[row].max().item()) + 1 + row,
                       fill=1000.0)
        kbs.append(kb)
        vbs.append(vb)
        refs.append(_dense_ref(query[row : row + 1], dk, dv))
    out = paged_attention_decode_batched(query, block_tables, kbs, vbs,
                                         torch.tensor(seq_lens, device=DEVICE, dtype=torch.long), block_size)
    torch.testing.assert_close(out, torch.cat(refs), atol=2e-5, rtol=2e-5)


def test_reference_api_batched_matches_single_and_zero_length_row() -> None:
    from fp8_cuda import paged_attention_decode, paged_attention_decode_batched

    torch.manual_seed(104)
    heads, head_dim, block_size = 2, 16, 4
    seq_lens = (1, 7, 0)
    query = torch.randn((3, heads, 1, head_dim), device=DEVICE)
    block_tables = torch.full((3, 2), -1, device=DEVICE, dtype=torch.long)
    kbs, vbs, singles = [], [], []
    for row, seq_len in enumerate(seq_lens):
        nblk = max(1, (seq_len + block_size - 1) // block_size)
        table = torch.arange(nblk, device=DEVICE, dtype=torch.long)
        block_tables[row, :nblk] = table
        kb = torch.randn((1, heads, nblk, block_size, head_dim), device=DEVICE)
        vb = torch.randn((1, heads, nblk, block_size, head_dim), device=DEVICE)
        kbs.append(kb)
        vbs.append(vb)
        if seq_len > 0:
            singles.append(paged_attention_decode(query[row : row + 1], table, kb, vb, seq_len, block_size))
        else:
            singles.append(torch.zeros_like(query[row : row + 1]))
    out = paged_attention_decode_batched(query, block_tables, kbs, vbs,
                                         torch.tensor(seq_lens, device=DEVICE, dtype=torch.long), block_size)
    torch.testing.assert_close(out, torch.cat(singles), atol=2e-5, rtol=2e-5)


def test_reference_api_batched_rejects_mismatched_pool_count() -> None:
    from fp8_cuda import paged_attention_decode_batched

    query = torch.zeros((2, 1, 1, 8), device=DEVICE)
    block_tables = torch.zeros((2, 1), device=DEVICE, dtype=torch.long)
    kb = [torch.zeros((1, 1, 1, 2, 8), device=DEVICE)]
    with pytest.raises(RuntimeError, match="key_blocks list length must match batch"):
        paged_attention_decode_batched(query, block_tables, kb, list(kb), torch.ones(2, device=DEVICE,
                                       dtype=torch.long), 2)


def test_reference_api_accepts_bf16_reference_layout() -> None:
    """The reference layout (B, H, P, bs, D) with repeated heads in bf16, against the oracle."""
    from fp8_cuda import paged_attention_decode

    gen = torch.Generator().manual_seed(77)
    heads, head_dim, block_size, seq_len = 4, 64, 16, 37
    query = torch.randn((2, heads, 1, head_dim), generator=gen).bfloat16()
    kb = torch.randn((2, heads, 5, block_size, head_dim), generator=gen).bfloat16()
    vb = torch.randn((2, heads, 5, block_size, head_dim), generator=gen).bfloat16()
    table = [4, 1, 3]
    out = paged_attention_decode(query.to(DEVICE), torch.tensor(table, device=DEVICE), kb.to(DEVICE), vb.to(DEVICE),
                                 seq_len, block_size)
    for b in range(2):
        pk = lib.np_bits(kb[b].permute(1, 0, 2, 3))
        pv = lib.np_bits(vb[b].permute(1, 0, 2, 3))
        q = lib.as_f32(lib.np_bits(query[b, :, 0]), "bfloat16")[None]
        exp = oracle.decode_attention(q, pk, pv, [table], [seq_len], dtype="bfloat16", round_probs=False)[0]
        lib.assert_close(lib.as_f32(lib.np_bits(out[b, :, 0]), "bfloat16"), exp, "bfloat16", f"row {b}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_cuda_core_formulation_matches_tensor_core_path_and_oracle(dtype) -> None:
    """PKV_DECODE_CUDA_CORES runs the CUDA-core formulation on shapes the tensor-core path serves; both
    match the oracle (the comparison behind the choice of the mma.sync formulation)."""
    ops = _ops()
    name = "float16" if dtype == torch.float16 else "bfloat16"
    gen = torch.Generator().manual_seed(71)
    lens = [1, 17, 300, 1025, 4096, 0, 2049]
    hq, hkv, d, bs = 16, 2, 256, 16
    need = [(n + bs - 1) // bs for n in lens]
    pages = sum(need) + 3
    perm = torch.randperm(pages, generator=gen).tolist()
    tables, used = [], 0
    for n in need:
        tables.append(perm[used:used + n])
        used += n
    key_pool = torch.randn((pages, hkv, bs, d), generator=gen).to(dtype)
    value_pool = torch.randn((pages, hkv, bs, d), generator=gen).to(dtype)
    query = torch.randn((len(lens), hq, d), generator=gen).to(dtype)
    bt = torch.from_numpy(oracle.padded_block_tables(tables)).to(torch.int32).to(DEVICE)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEVICE)
    kp, vp, q = key_pool.to(DEVICE), value_pool.to(DEVICE), query.to(DEVICE)
    before = ops.native_stats()
    cores = ops.paged_decode(q, kp, vp, bt, sl, cuda_cores=True)
    tensor = ops.paged_decode(q, kp, vp, bt, sl)
    after = ops.native_stats()
    assert after["decode_generic_calls"] == before["decode_generic_calls"] + 1
    assert after["decode_tensor_core_calls"] == before["decode_tensor_core_calls"] + 1
    expected = oracle.decode_attention(lib.as_f32(lib.np_bits(query), name), lib.np_bits(key_pool),
                                       lib.np_bits(value_pool), tables, lens, dtype=name, round_probs=False)
    for what, out in (("cuda cores", cores), ("tensor cores", tensor)):
        lib.assert_close(lib.as_f32(lib.np_bits(out), name), expected, name, what)
