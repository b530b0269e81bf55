"""GPU parity of the FP8 (e4m3) page format: the quantising append bit for bit against the oracle, and
paged decode over fp8 pools against the oracle's exact attention over the dequantised cache."""

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


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("head_dim", [64, 128, 256])
def test_fp8_append_matches_oracle_bit_for_bit(dtype, head_dim) -> None:
    ops = _ops()
    name = cases.dtype_name(dtype)
    gen = torch.Generator().manual_seed(head_dim + (1 if dtype == torch.float16 else 0))
    tokens, hkv, bs, pages = 45, 2, 16, 8
    mag = torch.exp(4 * torch.randn((tokens, 1, 1), generator=gen))  # rows over several decades
    key = (torch.randn((tokens, hkv, head_dim), generator=gen) * mag).to(dtype)
    value = (torch.randn((tokens, hkv, head_dim), generator=gen) * mag).to(dtype)
    key[3] = 0  # rows of zeros: scale 0
    slots = torch.randperm(pages * bs, generator=gen)[:tokens]
    slots[7] = -1  # padding token
    kp, vp, ks, vs = ops.new_fp8_pools(pages, hkv, bs, head_dim, DEVICE)
    flag = ops.new_error_flag(DEVICE)
    ops.kv_append_fp8(key.to(DEVICE), value.to(DEVICE), slots.to(DEVICE), kp, vp, ks, vs, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    f32 = lambda t: lib.as_f32(lib.np_bits(t), name)  # noqa: E731
    for src, pool, scales in ((key, kp, ks), (value, vp, vs)):
        codes, sc = oracle.quantize_fp8_rows(f32(src))
        got_codes = pool.cpu().numpy()
        got_sc = scales.cpu().numpy()
        for t, slot in enumerate(slots.tolist()):
            if slot < 0:
                continue
            np.testing.assert_array_equal(got_codes[slot // bs, :, slot % bs], codes[t], err_msg=f"token {t}")
            np.testing.assert_array_equal(got_sc[slot // bs, :, slot % bs], sc[t], err_msg=f"scale {t}")


def _fp8_case(seed: int, lens: list[int], hq: int, hkv: int, head_dim: int, bs: int, dtype: torch.dtype):
    """Random K/V appended through kv_append_fp8 into shuffled pages; never-written slots of the last
    pages hold NaN codes (0x7f) and NaN scales."""
    ops = _ops()
    gen = torch.Generator().manual_seed(seed)
    need = [(n + bs - 1) // bs for n in lens]
    num_pages = sum(need) + 5
    perm = torch.randperm(num_pages, generator=gen).tolist()
    tables, used = [], 0
    for n in need:
        tables.append(perm[used : used + n])
        used += n
    kp, vp, ks, vs = ops.new_fp8_pools(num_pages, hkv, bs, head_dim, DEVICE)
    kp.fill_(0x7F)
    vp.fill_(0x7F)
    ks.fill_(float("nan"))
    vs.fill_(float("nan"))
    total = sum(lens)
    key = torch.randn((total, hkv, head_dim), generator=gen).to(dtype)
    value = torch.randn((total, hkv, head_dim), generator=gen).to(dtype)
    slots = np.concatenate([oracle.slot_mapping(tables[b], 0, lens[b], bs) for b in range(len(lens)) if lens[b]]
                           or [np.zeros(0, np.int64)])
    ops.kv_append_fp8(key.to(DEVICE), value.to(DEVICE), torch.from_numpy(slots).to(DEVICE), kp, vp, ks, vs)
    query = torch.randn((len(lens), hq, head_dim), generator=gen).to(dtype)
    return kp, vp, ks, vs, tables, query, key, value


def _dequant_pools(kp, vp, ks, vs):
    return (oracle.dequantize_fp8(kp.cpu().numpy(), ks.cpu().numpy()),
            oracle.dequantize_fp8(vp.cpu().numpy(), vs.cpu().numpy()))


@pytest.mark.parametrize(
    "dtype,head_dim,hq,hkv,bs,index_dtype,pps",
    [
        (torch.bfloat16, 256, 16, 2, 16, torch.int32, 0),  # the model's layout
        (torch.float16, 128, 16, 4, 32, torch.int64, 0),
        (torch.bfloat16, 128, 8, 8, 16, torch.int32, 1),  # one query head per KV head, many splits
        (torch.float16, 256, 8, 1, 16, torch.int32, 2),
    ],
)
def test_fp8_decode_matches_oracle_over_dequantised_cache(dtype, head_dim, hq, hkv, bs, index_dtype, pps) -> None:
    ops = _ops()
    name = cases.dtype_name(dtype)
    lens = [1, 15, 16, 17, 100, 333, 0, 1000]
    kp, vp, ks, vs, tables, query, _, _ = _fp8_case(hq * head_dim + bs, lens, hq, hkv, head_dim, bs, dtype)
    bt = torch.from_numpy(oracle.padded_block_tables(tables)).to(DEVICE, index_dtype)
    sl = torch.tensor(lens, dtype=index_dtype, device=DEVICE)
    flag = ops.new_error_flag(DEVICE)
    out = ops.paged_decode_fp8(query.to(DEVICE), kp, vp, ks, vs, bt, sl, pages_per_split=pps, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    pk, pv = _dequant_pools(kp, vp, ks, vs)
    q = lib.as_f32(lib.np_bits(query), name)
    exp = oracle.decode_attention(q, pk, pv, tables, lens, dtype="float32", round_probs=False)
    got = lib.as_f32(lib.np_bits(out), name)
    assert np.isfinite(got).all()
    lib.assert_close(got, oracle.round_to(exp, name), name, "fp8 decode")
    assert np.all(got[lens.index(0)] == 0)  # a request without tokens gives zeros
    # chained launches (and, after the first, page loads started before the previous call ends) change
    # nothing: the same outputs bit for bit over back-to-back calls sharing a workspace
    work = ops.new_decode_workspace(ops.paged_decode_workspace_size(len(lens), hq, hkv, head_dim, bt.shape[1], bs, pps),
                                    DEVICE)
    outs = [ops.paged_decode_fp8(query.to(DEVICE), kp, vp, ks, vs, bt, sl, pages_per_split=pps, workspace=work,
                                 chained=True, prefetch=i > 0) for i in range(3)]
    torch.cuda.synchronize()
    for o in outs:
        np.testing.assert_array_equal(lib.np_bits(o), lib.np_bits(out))


def test_fp8_decode_stays_close_to_the_unquantised_cache() -> None:
    """The format's own error (a property of e4m3, not parity): against attention over the original bf16
    K/V, every output of N(0, 1) data stays within one e4m3 step (2^-4) and the mean error is small."""
    ops = _ops()
    lens = [64, 500, 2000]
    kp, vp, ks, vs, tables, query, key, value = _fp8_case(91, lens, 16, 2, 256, 16, torch.bfloat16)
    bt = torch.from_numpy(oracle.padded_block_tables(tables)).to(DEVICE, torch.int32)
    out = ops.paged_decode_fp8(query.to(DEVICE), kp, vp, ks, vs, bt, torch.tensor(lens, dtype=torch.int32,
                                                                               device=DEVICE))
    torch.cuda.synchronize()
    got = lib.as_f32(lib.np_bits(out), "bfloat16")
    q = lib.as_f32(lib.np_bits(query), "bfloat16")
    k = lib.as_f32(lib.np_bits(key), "bfloat16")
    v = lib.as_f32(lib.np_bits(value), "bfloat16")
    start, errs = 0, []
    for b, n in enumerate(lens):
        kb, vb = k[start : start + n], v[start : start + n]  # (n, Hkv, D)
        for h in range(16):
            s = kb[:, h // 8] @ q[b, h] / 16.0
            p = np.exp(s - s.max())
            errs.append(np.abs(got[b, h] - (p / p.sum()) @ vb[:, h // 8]))
        start += n
    errs = np.stack(errs)
    assert errs.max() < 2.0 ** -4 and errs.mean() < 0.01, (errs.max(), errs.mean())


def test_fp8_decode_rejects_unsupported_shapes() -> None:
    ops = _ops()
    kp, vp, ks, vs = ops.new_fp8_pools(4, 2, 16, 64, DEVICE)
    query = torch.zeros((1, 16, 64), dtype=torch.bfloat16, device=DEVICE)
    bt = torch.zeros((1, 4), dtype=torch.int32, device=DEVICE)
    with pytest.raises(RuntimeError, match="head_dim must be 128 or 256"):
        ops.paged_decode_fp8(query, kp, vp, ks, vs, bt, torch.ones(1, dtype=torch.int32, device=DEVICE))
