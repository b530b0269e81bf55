"""One process driving two GPUs: every kernel that needs more than 48 KB of dynamic shared memory (its
launch attribute is set per device) runs on cuda:0 and then on cuda:1 with the same inputs, and the
results are bit-identical. Skipped with fewer than two GPUs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import pkv_testlib as lib
from oracle import paged_kv_oracle as oracle

pytestmark = pytest.mark.gpu


def _need_two():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")


def _decode_inputs(gen, dtype):
    lens = [5, 70, 700, 1]
    hq, hkv, d, bs = 16, 2, 256, 16
    pages = sum((n + bs - 1) // bs for n in lens) + 2
    perm = torch.randperm(pages, generator=gen).tolist()
    tables, used = [], 0
    for n in lens:
        k = (n + bs - 1) // bs
        tables.append(perm[used : used + k])
        used += k
    bt = torch.from_numpy(oracle.padded_block_tables(tables)).to(torch.int32)
    return (torch.randn((len(lens), hq, d), generator=gen).to(dtype), torch.randn((pages, hkv, bs, d), generator=gen).to(dtype),
            torch.randn((pages, hkv, bs, d), generator=gen).to(dtype), bt, torch.tensor(lens, dtype=torch.int32))


def test_kernels_run_on_each_device_of_one_process() -> None:
    _need_two()
    import paged_kv_ops as ops

    gen = torch.Generator().manual_seed(3)
    dec = _decode_inputs(gen, torch.float16)
    # output stage inputs
    heads = torch.randn((8, 16, 1, 256), generator=gen).to(torch.bfloat16)
    gate = torch.randn((8, 1, 4096), generator=gen).to(torch.bfloat16)
    weight = (0.05 * torch.randn((256, 4096), generator=gen)).to(torch.float8_e4m3fn)
    scale = (0.5 + torch.rand((2, 32), generator=gen)).to(torch.bfloat16)
    # prefill inputs: one request, 40-token chunk on a 30-token prefix
    pq = torch.randn((40, 16, 256), generator=gen).to(torch.bfloat16)
    pk = torch.randn((8, 2, 16, 256), generator=gen).to(torch.bfloat16)
    pv = torch.randn((8, 2, 16, 256), generator=gen).to(torch.bfloat16)
    ptab = torch.tensor([[3, 0, 6, 1, 5]], dtype=torch.int32)
    results = []
    for dev in ("cuda:0", "cuda:1"):
        with torch.cuda.device(dev):
            q, kp, vp, bt, sl = (t.to(dev) for t in dec)
            out_dec = ops.paged_decode(q, kp, vp, bt, sl)
            kp8, vp8, ks, vs = ops.new_fp8_pools(kp.shape[0], 2, 16, 256, dev)
            slots = torch.arange(kp.shape[0] * 16, device=dev)
            ops.kv_append_fp8(kp.permute(0, 2, 1, 3).reshape(-1, 2, 256), vp.permute(0, 2, 1, 3).reshape(-1, 2, 256),
                              slots, kp8, vp8, ks, vs)
            out_f8 = ops.paged_decode_fp8(q, kp8, vp8, ks, vs, bt, sl)
            out_o = ops.gated_o_proj(heads.to(dev), gate.to(dev), weight.to(dev), scale.to(dev))
            cu = torch.tensor([0, 40], dtype=torch.int32, device=dev)
            out_p = ops.paged_prefill(pq.to(dev), cu, pk.to(dev), pv.to(dev), ptab.to(dev),
                                      torch.tensor([70], dtype=torch.int32, device=dev), max_q_len=40)
            torch.cuda.synchronize(dev)
            results.append([lib.np_bits(t) for t in (out_dec, out_f8, out_o, out_p)])
    for a, b in zip(*results):
        np.testing.assert_array_equal(a, b)
