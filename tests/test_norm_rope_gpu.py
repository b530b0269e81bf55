"""GPU parity of the fused q/k RMSNorm + partial rotary embedding + K/V append (pkv_qk_norm_rope_append):
against the reference's own layer (fixtures from tp_full_attention / _tp_full_attention_batch), and
against the oracle over head sizes, rotary widths, dtypes and index types; plus its error paths."""

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


def _pool_rows(pool: torch.Tensor, slots: np.ndarray, block_size: int) -> np.ndarray:
    """(T, Hkv, D) rows of a (P, Hkv, bs, D) pool at the given slots, as numpy bits."""
    bits = lib.np_bits(pool)
    return np.stack([bits[s // block_size, :, s % block_size] for s in slots])


@pytest.mark.parametrize("make", cases.NORM_ROPE_CASES, ids=lambda m: m.__name__)
def test_fused_norm_rope_append_reproduces_reference_layer(make) -> None:
    """Pre-norm projections -> fused kernel -> our paged attention equals the reference layer: the query
    it attends with and the K it caches (within one unit in the last place, from the mean-of-squares
    order), the V bit for bit, and the layer output within the attention tolerance plus the reference's
    own probability rounding."""
    ops = _ops()
    case = make()
    dtype = cases.dtype_name(case.dtype)
    g = lib.golden()
    d, bs, hkv, hq = case.head_dim, case.block_size, case.local_kv_heads, case.local_q_heads
    kv0 = case.rank * hkv
    num_pages, tables = lib.shared_pool_layout(case)
    shape = (num_pages, hkv, bs, d)
    key_pool = torch.zeros(shape, dtype=case.dtype, device=DEVICE)
    value_pool = torch.zeros(shape, dtype=case.dtype, device=DEVICE)
    for b in range(case.batch):  # the cache before the call (its contents are already rotated)
        if case.prefix_lens[b]:
            slots = torch.from_numpy(oracle.slot_mapping(tables[b], 0, case.prefix_lens[b], bs)).to(DEVICE)
            ops.kv_append(case.prefix_k[b][:, kv0 : kv0 + hkv].to(DEVICE), case.prefix_v[b][:, kv0 : kv0 + hkv].to(DEVICE),
                          slots, key_pool, value_pool)
    table = ops.rope_cos_sin_table(max(case.lens) + 16, d, case.partial_rotary_factor, case.rope_theta, case.dtype,
                                   DEVICE)
    q_proj = torch.cat(case.q_proj).to(DEVICE)  # (T, Hq_local, 2D): query | gate per head
    key = torch.cat(case.key).to(DEVICE)[:, kv0 : kv0 + hkv]
    value = torch.cat(case.value).to(DEVICE)[:, kv0 : kv0 + hkv]
    positions = np.concatenate([np.arange(p, p + t) for p, t in zip(case.prefix_lens, case.new_lens)])
    slot_list = [oracle.slot_mapping(tables[b], case.prefix_lens[b], case.new_lens[b], bs) for b in range(case.batch)]
    slots = np.concatenate(slot_list)
    flag = ops.new_error_flag(DEVICE)
    q_out = ops.qk_norm_rope_append(q_proj[:, :, :d], key, value, case.q_norm.to(DEVICE), case.k_norm.to(DEVICE), table,
                                    torch.from_numpy(positions).to(DEVICE, torch.int32),
                                    torch.from_numpy(slots).to(DEVICE), key_pool, value_pool, eps=case.eps,
                                    error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    got_q = lib.as_f32(lib.np_bits(q_out), dtype)
    offset = 0
    for b in range(case.batch):
        t = case.new_lens[b]
        lib.assert_ulp_close(got_q[offset : offset + t], oracle.to_f32(g[f"{case.name}/query/{b}"], dtype), dtype,
                             f"query[{b}]")
        rows_k = lib.as_f32(_pool_rows(key_pool, slot_list[b], bs), dtype)
        lib.assert_ulp_close(rows_k, oracle.to_f32(g[f"{case.name}/key/{b}"], dtype), dtype, f"key[{b}]")
        np.testing.assert_array_equal(_pool_rows(value_pool, slot_list[b], bs), g[f"{case.name}/value/{b}"])
        offset += t
    # the layer output: attention over the pool with the fused query
    bt = torch.from_numpy(oracle.padded_block_tables(tables)).to(DEVICE, torch.int32)
    lens = torch.tensor(case.lens, dtype=torch.int32, device=DEVICE)
    pk, pv = lib.np_bits(key_pool), lib.np_bits(value_pool)
    if case.batched_decode:
        out = lib.as_f32(lib.np_bits(ops.paged_decode(q_out, key_pool, value_pool, bt, lens)), dtype)
        bound = oracle.decode_rounding_bound(got_q, pk, pv, tables, case.lens, dtype=dtype)
        for b in range(case.batch):
            ref = oracle.to_f32(g[f"{case.name}/out/{b}"], dtype)[0]
            lib.assert_close(out[b], ref, dtype, f"layer output[{b}]", extra=bound[b])
    else:
        cu = torch.tensor(np.concatenate([[0], np.cumsum(case.new_lens)]), dtype=torch.int32, device=DEVICE)
        out = lib.as_f32(lib.np_bits(ops.paged_prefill(q_out, cu, key_pool, value_pool, bt, lens)), dtype)
        offset = 0
        for b in range(case.batch):
            t = case.new_lens[b]
            q = got_q[offset : offset + t].transpose(1, 0, 2)
            bound = oracle.prefill_rounding_bound(q, pk, pv, tables[b], case.lens[b], dtype=dtype).transpose(1, 0, 2)
            ref = oracle.to_f32(g[f"{case.name}/out/{b}"], dtype)
            lib.assert_close(out[offset : offset + t], ref, dtype, f"layer output[{b}]", extra=bound)
            offset += t


@pytest.mark.parametrize(
    "dtype,head_dim,rotary_dim,hq,hkv,index_dtype,block_size",
    [
        (torch.bfloat16, 256, 64, 16, 2, torch.int32, 16),  # the model's layout
        (torch.float16, 128, 32, 8, 1, torch.int64, 16),
        (torch.float32, 64, 64, 4, 4, torch.int32, 16),  # rotary over the whole head
        (torch.bfloat16, 128, 0, 8, 2, torch.int64, 16),  # no rotary part
        (torch.float16, 512, 128, 4, 2, torch.int32, 16),
        (torch.bfloat16, 1024, 256, 2, 1, torch.int32, 16),
        (torch.bfloat16, 256, 64, 6, 3, torch.int64, 24),  # pages of 24 slots (not a power of two)
        (torch.bfloat16, 256, 192, 5, 1, torch.int32, 16),  # rotary pairs across lanes: via shared memory
        (torch.float16, 256, 256, 3, 2, torch.int64, 16),  # rotary over the whole head, odd query rows
        (torch.bfloat16, 128, 32, 0, 2, torch.int32, 16),  # no query rows: key/value append only
        (torch.float32, 256, 64, 4, 2, torch.int64, 16),  # fp32 rows of 16 elements per lane
        (torch.bfloat16, 64, 32, 6, 2, torch.int32, 16),  # 8-byte runs per lane
    ],
)
def test_fused_norm_rope_append_matches_oracle(dtype, head_dim, rotary_dim, hq, hkv, index_dtype, block_size) -> None:
    ops = _ops()
    name = cases.dtype_name(dtype)
    gen = torch.Generator().manual_seed(head_dim + rotary_dim + hq)
    tokens, num_pages, offset = 53, 12, 7
    query = torch.randn((tokens, hq, head_dim), generator=gen).to(dtype)
    key = torch.randn((tokens, hkv, head_dim), generator=gen).to(dtype)
    value = torch.randn((tokens, hkv, head_dim), generator=gen).to(dtype)
    q_weight = (0.2 * torch.randn((head_dim,), generator=gen)).to(dtype)
    k_weight = (0.2 * torch.randn((head_dim,), generator=gen)).to(dtype)
    positions = torch.randint(0, 4000, (tokens,), generator=gen)
    slots = torch.randperm(num_pages * block_size, generator=gen)[:tokens]
    slots[::9] = -1  # padding tokens: skipped
    table = ops.rope_cos_sin_table(4100, head_dim, rotary_dim / head_dim, 1e7, dtype)
    key_pool = torch.full((num_pages, hkv, block_size, head_dim), 7.0, dtype=dtype, device=DEVICE)
    value_pool = torch.full_like(key_pool, 7.0)
    flag = ops.new_error_flag(DEVICE)
    q_out = ops.qk_norm_rope_append(query.to(DEVICE), key.to(DEVICE), value.to(DEVICE), q_weight.to(DEVICE),
                                    k_weight.to(DEVICE), table.to(DEVICE), positions.to(DEVICE, index_dtype),
                                    slots.to(DEVICE), key_pool, value_pool, eps=1e-6, position_offset=offset,
                                    error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    f32 = lambda t: lib.as_f32(lib.np_bits(t), name)  # noqa: E731
    tab = f32(table)
    pos = positions.numpy() + offset
    cos, sin = tab[pos, :rotary_dim], tab[pos, rotary_dim:]
    exp_q, exp_k = oracle.qk_norm_rope(f32(query), f32(key), f32(q_weight), f32(k_weight), 1e-6, cos, sin, dtype=name)
    max_ulp, min_exact = (4, 0.5) if name == "float32" else (2, 0.99)
    lib.assert_ulp_close(f32(q_out), exp_q, name, "query", max_ulp=max_ulp, min_exact=min_exact)
    live = slots.numpy() >= 0
    got_k = lib.as_f32(_pool_rows(key_pool, slots.numpy()[live], block_size), name)
    lib.assert_ulp_close(got_k, exp_k[live], name, "key", max_ulp=max_ulp, min_exact=min_exact)
    np.testing.assert_array_equal(_pool_rows(value_pool, slots.numpy()[live], block_size), lib.np_bits(value)[live])
    # slots no token was mapped to (padding tokens included) keep the fill value
    used = set(slots.numpy()[live].tolist())
    pool_k = f32(key_pool).transpose(0, 2, 1, 3).reshape(num_pages * block_size, hkv, head_dim)  # slot-major
    untouched = [s for s in range(num_pages * block_size) if s not in used]
    assert np.all(pool_k[untouched] == 7.0)


def test_fused_norm_rope_append_reports_bad_slots_and_positions() -> None:
    ops = _ops()
    dtype = torch.bfloat16
    hq, hkv, d, bs, pages = 4, 2, 128, 16, 4
    tokens = 6
    query = torch.randn((tokens, hq, d), device=DEVICE).to(dtype)
    key = torch.randn((tokens, hkv, d), device=DEVICE).to(dtype)
    value = torch.randn((tokens, hkv, d), device=DEVICE).to(dtype)
    w = torch.zeros((d,), dtype=dtype, device=DEVICE)
    table = ops.rope_cos_sin_table(100, d, 0.25, 1e7, dtype, DEVICE)
    key_pool = torch.zeros((pages, hkv, bs, d), dtype=dtype, device=DEVICE)
    value_pool = torch.zeros_like(key_pool)
    positions = torch.tensor([0, 1, 2, 100, 4, 5], dtype=torch.int64, device=DEVICE)  # token 3: past the table
    slots = torch.tensor([0, 1, pages * bs, 3, -1, 5], dtype=torch.int64, device=DEVICE)  # token 2: past the pool
    q_out = torch.full((tokens, hq, d), 3.0, dtype=dtype, device=DEVICE)
    flag = ops.new_error_flag(DEVICE)
    ops.qk_norm_rope_append(query, key, value, w, w, table, positions, slots, key_pool, value_pool, eps=1e-6,
                            q_out=q_out, error_flag=flag)
    torch.cuda.synchronize()
    bits = int(flag.item())
    assert bits & ops.DEVERR_SLOT_OUT_OF_RANGE and bits & ops.DEVERR_BAD_SEQUENCE_LENGTH
    by_slot = lambda pool: pool.permute(0, 2, 1, 3).reshape(pages * bs, hkv, d)  # noqa: E731
    assert torch.all(q_out[3] == 3.0)  # the token with a bad position is not written at all
    assert torch.all(by_slot(key_pool)[3] == 0) and torch.all(by_slot(value_pool)[3] == 0)
    assert not torch.all(q_out[2] == 3.0)  # a bad slot still yields the query row
    assert not torch.all(by_slot(key_pool)[5] == 0)  # valid tokens are appended
    assert torch.equal(by_slot(value_pool)[5], value[5])
    with pytest.raises(RuntimeError, match="rotary_dim"):
        bad_table = torch.zeros((100, 2 * 36), dtype=dtype, device=DEVICE)
        ops.qk_norm_rope_append(query, key, value, w, w, bad_table, positions, slots, key_pool, value_pool, eps=1e-6)


def test_decode_step_from_projections_matches_oracle() -> None:
    """DecodeStepRunner.step_projected over 2 layers: slot mapping, fused norm/rotary/append and paged
    decode per layer equal the oracle's composition (norm + rotary of the projections at each request's
    position, append, dense decode attention)."""
    from tp_runtime import DecodeStepRunner

    ops = _ops()
    dtype, name = torch.bfloat16, "bfloat16"
    gen = torch.Generator().manual_seed(77)
    layers, batch, hq, hkv, d, bs = 2, 5, 16, 2, 256, 16
    lens0 = [3, 16, 40, 129, 700]
    pages_per = [(n + 1 + bs - 1) // bs for n in lens0]
    num_pages = sum(pages_per) + 4
    perm = torch.randperm(num_pages, generator=gen).tolist()
    tables, used = [], 0
    for n in pages_per:
        tables.append(perm[used : used + n])
        used += n
    key_pools = torch.randn((layers, num_pages, hkv, bs, d), generator=gen).to(dtype)
    value_pools = torch.randn((layers, num_pages, hkv, bs, d), generator=gen).to(dtype)
    max_blocks = max(pages_per)
    bt = torch.full((batch, max_blocks), -1, dtype=torch.int32)
    for b, t in enumerate(tables):
        bt[b, : len(t)] = torch.tensor(t, dtype=torch.int32)
    query = torch.randn((layers, batch, hq, 2 * d), generator=gen).to(dtype)  # query | gate halves
    key = torch.randn((layers, batch, hkv, d), generator=gen).to(dtype)
    value = torch.randn((layers, batch, hkv, d), generator=gen).to(dtype)
    q_norm = (0.1 * torch.randn((layers, d), generator=gen)).to(dtype)
    k_norm = (0.1 * torch.randn((layers, d), generator=gen)).to(dtype)
    table = ops.rope_cos_sin_table(1024, d, 0.25, 1e7, dtype)
    kp_dev, vp_dev = key_pools.to(DEVICE), value_pools.to(DEVICE)
    runner = DecodeStepRunner(kp_dev, vp_dev, bt.to(DEVICE), torch.tensor(lens0, dtype=torch.int32, device=DEVICE),
                              num_q_heads=hq)
    out = torch.empty((layers, batch, hq, d), dtype=dtype, device=DEVICE)
    q_dev = query.to(DEVICE)
    runner.step_projected(q_dev[..., :d], key.to(DEVICE), value.to(DEVICE), q_norm.to(DEVICE), k_norm.to(DEVICE),
                          table.to(DEVICE), 1e-6, out)
    torch.cuda.synchronize()
    assert runner.check_errors() == 0
    assert runner.seq_lens.tolist() == [n + 1 for n in lens0]
    f32 = lambda t: lib.as_f32(lib.np_bits(t), name)  # noqa: E731
    tab = f32(table)
    cos, sin = tab[lens0, :64], tab[lens0, 64:]
    lens = [n + 1 for n in lens0]
    got = f32(out)
    for layer in range(layers):
        q, k = oracle.qk_norm_rope(f32(query[layer, :, :, :d]), f32(key[layer]), f32(q_norm[layer]),
                                   f32(k_norm[layer]), 1e-6, cos, sin, dtype=name)
        slots = np.array([tables[b][lens0[b] // bs] * bs + lens0[b] % bs for b in range(batch)])
        # the kernel's rotated key may differ from the oracle's by a rounding: compare the stored pool
        # rows within that (and the value bit for bit), then attend over the kernel's own pool
        got_pk, got_pv = lib.np_bits(kp_dev[layer].cpu()), lib.np_bits(vp_dev[layer].cpu())
        lib.assert_ulp_close(lib.as_f32(got_pk[slots // bs, :, slots % bs], name), k, name, f"layer {layer} key")
        np.testing.assert_array_equal(got_pv[slots // bs, :, slots % bs], lib.np_bits(value[layer]))
        exp = oracle.decode_attention(q, got_pk, got_pv, tables, lens, dtype=name, round_probs=False)
        lib.assert_close(got[layer], exp, name, f"layer {layer} output")
