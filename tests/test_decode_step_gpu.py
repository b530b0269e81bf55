"""GPU parity of the decode step (tp_runtime.DecodeStepRunner.step): device slot mapping for every
layer of the stacked pools, one append of every layer's new K/V, and the per-layer paged decode
launched as a chained sequence -- against the oracle's append + dense decode attention."""

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


def _setup(seed: int, layers: int, lens0: list[int], hkv: int, d: int, bs: int, dtype):
    gen = torch.Generator().manual_seed(seed)
    pages_per = [(n + 1 + bs - 1) // bs for n in lens0]
    num_pages = sum(pages_per) + 4
    perm = torch.randperm(num_pages, generator=gen).tolist()
    tables, used = [], 0
    for n in pages_per:
        tables.append(perm[used : used + n])
        used += n
    bt = torch.full((len(lens0), max(pages_per)), -1, dtype=torch.int32)
    for b, t in enumerate(tables):
        bt[b, : len(t)] = torch.tensor(t, dtype=torch.int32)
    pools = [torch.randn((layers, num_pages, hkv, bs, d), generator=gen).to(dtype) for _ in range(2)]
    return gen, tables, bt, num_pages, pools


def test_layered_slot_mapping_offsets_each_layer() -> None:
    ops = _ops()
    tables = torch.tensor([[3, 1, -1], [0, 2, 5]], dtype=torch.int32, device=DEVICE)
    lens = torch.tensor([17, 31], dtype=torch.int32, device=DEVICE)
    one = ops.decode_slot_mapping(tables, lens.clone(), 8, 16, advance=False)
    three = ops.decode_slot_mapping(tables, lens.clone(), 8, 16, advance=False, layers=3)
    assert one.tolist() == [1 * 16 + 1, 2 * 16 + 15]
    for layer in range(3):
        assert three[layer].tolist() == [s + layer * 8 * 16 for s in one.tolist()]
    lens[0] = 48  # past the table: slot -1 in every layer, flagged
    flag = ops.new_error_flag(DEVICE)
    three = ops.decode_slot_mapping(tables, lens, 8, 16, advance=True, layers=3, error_flag=flag)
    assert three[:, 0].tolist() == [-1, -1, -1] and int(flag.item()) & ops.DEVERR_TABLE_TOO_SHORT
    assert lens.tolist() == [48, 32]  # only rows that got a slot advance


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("strided_kv", [False, True])
def test_decode_step_matches_oracle(dtype, strided_kv) -> None:
    """Three layers, ragged contexts (including one that opens a new page): the appended rows are
    bit-exact in every layer's pool and each layer's output equals dense attention over its pages.
    strided_kv passes K/V as slices of a wider projection output (per-layer appends)."""
    from tp_runtime import DecodeStepRunner

    name = cases.dtype_name(dtype)
    layers, hq, hkv, d, bs = 3, 16, 2, 256, 16
    lens0 = [3, 15, 16, 130, 700]
    batch = len(lens0)
    gen, tables, bt, num_pages, (kp, vp) = _setup(11 + strided_kv, layers, lens0, hkv, d, bs, dtype)
    query = torch.randn((layers, batch, hq, d), generator=gen).to(dtype)
    if strided_kv:
        kv = torch.randn((layers, batch, 2 * hkv, d), generator=gen).to(dtype)
        key_h, value_h = kv[:, :, :hkv], kv[:, :, hkv:]
    else:
        key_h = torch.randn((layers, batch, hkv, d), generator=gen).to(dtype)
        value_h = torch.randn((layers, batch, hkv, d), generator=gen).to(dtype)
    kp_dev, vp_dev = kp.to(DEVICE), vp.to(DEVICE)
    runner = DecodeStepRunner(kp_dev, vp_dev, bt.to(DEVICE), torch.tensor(lens0, dtype=torch.int32, device=DEVICE),
                              num_q_heads=hq)
    if strided_kv:
        kv_dev = kv.to(DEVICE)
        key, value = kv_dev[:, :, :hkv], kv_dev[:, :, hkv:]
    else:
        key, value = key_h.to(DEVICE), value_h.to(DEVICE)
    out = torch.empty((layers, batch, hq, d), dtype=dtype, device=DEVICE)
    runner.step(query.to(DEVICE), key, value, out)
    torch.cuda.synchronize()
    assert runner.check_errors() == 0
    assert runner.seq_lens.tolist() == [n + 1 for n in lens0]
    lens = [n + 1 for n in lens0]
    slots = np.array([tables[b][lens0[b] // bs] * bs + lens0[b] % bs for b in range(batch)])
    got = lib.as_f32(lib.np_bits(out), name)
    for layer in range(layers):
        pk, pv = lib.np_bits(kp_dev[layer].cpu()), lib.np_bits(vp_dev[layer].cpu())
        np.testing.assert_array_equal(pk[slots // bs, :, slots % bs], lib.np_bits(key_h[layer].contiguous()))
        np.testing.assert_array_equal(pv[slots // bs, :, slots % bs], lib.np_bits(value_h[layer].contiguous()))
        # every other row of the pools is untouched
        mask = np.ones(pk.shape[0] * bs, dtype=bool)
        mask[slots] = False
        ref_k = lib.np_bits(kp[layer]).transpose(0, 2, 1, 3).reshape(-1, hkv, d)
        np.testing.assert_array_equal(pk.transpose(0, 2, 1, 3).reshape(-1, hkv, d)[mask], ref_k[mask])
        q = lib.as_f32(lib.np_bits(query[layer]), name)
        exp = oracle.decode_attention(q, pk, pv, tables, lens, dtype=name, round_probs=False)
        lib.assert_close(got[layer], exp, name, f"layer {layer}")


def test_decode_step_over_fp8_pages_matches_oracle() -> None:
    from tp_runtime import DecodeStepRunner

    ops = _ops()
    layers, hq, hkv, d, bs = 2, 16, 2, 256, 16
    lens0 = [5, 47, 300]
    batch = len(lens0)
    gen, tables, bt, num_pages, _ = _setup(21, layers, lens0, hkv, d, bs, torch.bfloat16)
    kp = torch.zeros((layers, num_pages, hkv, bs, d), dtype=torch.uint8, device=DEVICE)
    vp = torch.zeros_like(kp)
    ks = torch.zeros((layers, num_pages, hkv, bs), dtype=torch.float32, device=DEVICE)
    vs = torch.zeros_like(ks)
    # fill the existing context through the quantising append, one layer at a time
    for layer in range(layers):
        for b, n in enumerate(lens0):
            slots = torch.from_numpy(oracle.slot_mapping(tables[b], 0, n, bs)).to(DEVICE)
            k = torch.randn((n, hkv, d), generator=gen).to(torch.bfloat16).to(DEVICE)
            v = torch.randn((n, hkv, d), generator=gen).to(torch.bfloat16).to(DEVICE)
            ops.kv_append_fp8(k, v, slots, kp[layer], vp[layer], ks[layer], vs[layer])
    runner = DecodeStepRunner(kp, vp, bt.to(DEVICE), torch.tensor(lens0, dtype=torch.int32, device=DEVICE),
                              num_q_heads=hq, key_scales=ks, value_scales=vs)
    query = torch.randn((layers, batch, hq, d), generator=gen).to(torch.float16).to(DEVICE)
    key = torch.randn((layers, batch, hkv, d), generator=gen).to(torch.float16).to(DEVICE)
    value = torch.randn((layers, batch, hkv, d), generator=gen).to(torch.float16).to(DEVICE)
    out = torch.empty((layers, batch, hq, d), dtype=torch.float16, device=DEVICE)
    runner.step(query, key, value, out)
    torch.cuda.synchronize()
    assert runner.check_errors() == 0
    lens = [n + 1 for n in lens0]
    slots = np.array([tables[b][lens0[b] // bs] * bs + lens0[b] % bs for b in range(batch)])
    got = lib.as_f32(lib.np_bits(out), "float16")
    for layer in range(layers):
        codes, sc = oracle.quantize_fp8_rows(lib.as_f32(lib.np_bits(key[layer]), "float16"))
        np.testing.assert_array_equal(kp[layer].cpu().numpy()[slots // bs, :, slots % bs], codes)
        np.testing.assert_array_equal(ks[layer].cpu().numpy()[slots // bs, :, slots % bs], sc)
        pk = oracle.dequantize_fp8(kp[layer].cpu().numpy(), ks[layer].cpu().numpy())
        pv = oracle.dequantize_fp8(vp[layer].cpu().numpy(), vs[layer].cpu().numpy())
        q = lib.as_f32(lib.np_bits(query[layer]), "float16")
        exp = oracle.decode_attention(q, pk, pv, tables, lens, dtype="float32", round_probs=False)
        lib.assert_close(got[layer], oracle.round_to(exp, "float16"), "float16", f"fp8 layer {layer}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_chained_decode_is_bit_identical(dtype) -> None:
    """PKV_DECODE_CHAINED (and PKV_DECODE_PREFETCH) change only how the kernels are launched: outputs are
    bit for bit those of the plain launch, over several back-to-back calls on one stream sharing a
    workspace."""
    ops = _ops()
    gen = torch.Generator().manual_seed(5)
    lens = [1, 17, 200, 1500, 0, 64]
    hq, hkv, d, bs = 16, 2, 256, 16
    pages = sum((n + bs - 1) // bs for n in lens) + 3
    perm = torch.randperm(pages, generator=gen).tolist()
    tables, used = [], 0
    for n in lens:
        k = (n + bs - 1) // bs
        tables.append(perm[used : used + k])
        used += k
    bt = torch.from_numpy(oracle.padded_block_tables(tables)).to(DEVICE, torch.int32)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEVICE)
    kp = torch.randn((pages, hkv, bs, d), generator=gen).to(dtype).to(DEVICE)
    vp = torch.randn((pages, hkv, bs, d), generator=gen).to(dtype).to(DEVICE)
    qs = [torch.randn((len(lens), hq, d), generator=gen).to(dtype).to(DEVICE) for _ in range(4)]
    work = ops.new_decode_workspace(ops.paged_decode_workspace_size(len(lens), hq, hkv, d, bt.shape[1], bs, 0), DEVICE)
    plain = [ops.paged_decode(q, kp, vp, bt, sl, workspace=work) for q in qs]
    chained = [ops.paged_decode(q, kp, vp, bt, sl, workspace=work, chained=True) for q in qs]
    # PKV_DECODE_PREFETCH: the page loads of calls 2.. start before the previous call ends (the previous
    # call writes no pool, table or length); the query of each call is produced by the kernel right before
    # it (a copy), which the prefetching call must still wait for
    prefetched = []
    for i, q in enumerate(qs):
        qi = torch.empty_like(q)
        qi.copy_(q)
        prefetched.append(ops.paged_decode(qi, kp, vp, bt, sl, workspace=work, chained=True, prefetch=i > 0))
    torch.cuda.synchronize()
    for a, b, c in zip(plain, chained, prefetched):
        np.testing.assert_array_equal(lib.np_bits(a), lib.np_bits(b))
        np.testing.assert_array_equal(lib.np_bits(a), lib.np_bits(c))
