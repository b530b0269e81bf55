"""Full-size long-context split-KV decode and continuous-batching churn with compaction, on the GPU.

long: 8 requests x 131072 tokens (bf16): sampled requests match the oracle; the output does not
depend on how the contexts are split (automatic vs 2048-token partitions).
churn: requests finish, arrive into staging pages and are compacted step after step; every request
always gathers exactly the tokens written for it (bit-exact page moves through pkv_copy_pages).
"""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch

import pkv_testlib as lib
from oracle import paged_kv_oracle as oracle

pytestmark = pytest.mark.gpu
DEVICE = "cuda:0"


def _ops():
    import paged_kv_ops

    return paged_kv_ops


def test_long_context_split_decode_matches_oracle_and_split_size() -> None:
    ops = _ops()
    B, L, hq, hkv, d, bs = 8, 131072, 16, 2, 256, 16
    pages = B * L // bs
    gen = torch.Generator(device=DEVICE).manual_seed(4)
    key_pool = torch.randn((pages + 3, hkv, bs, d), generator=gen, device=DEVICE).bfloat16()
    value_pool = torch.randn((pages + 3, hkv, bs, d), generator=gen, device=DEVICE).bfloat16()
    perm = torch.randperm(pages + 3, generator=torch.Generator().manual_seed(4))[:pages]
    tables = perm.view(B, L // bs).to(torch.int32).to(DEVICE)
    query = torch.randn((B, hq, d), generator=gen, device=DEVICE).bfloat16()
    lens = torch.full((B,), L, dtype=torch.int32, device=DEVICE)
    auto = ops.paged_decode(query, key_pool, value_pool, tables, lens)
    parts = ops.paged_decode(query, key_pool, value_pool, tables, lens, pages_per_split=128)  # 64 partitions
    a, p = lib.as_f32(lib.np_bits(auto), "bfloat16"), lib.as_f32(lib.np_bits(parts), "bfloat16")
    lib.assert_close(a, p, "bfloat16", "automatic vs 64 partitions")
    for b in (0, 5):
        table = tables[b].tolist()
        pk = lib.np_bits(key_pool[tables[b].long()])
        pv = lib.np_bits(value_pool[tables[b].long()])
        q = lib.as_f32(lib.np_bits(query[b : b + 1]), "bfloat16")
        exp = oracle.decode_attention(q, pk, pv, [list(range(len(table)))], [L], dtype="bfloat16", round_probs=False)
        lib.assert_close(a[b : b + 1], exp, "bfloat16", f"request {b}")


def _token_rows(rid: int, start: int, count: int, hkv: int, d: int) -> torch.Tensor:
    """Deterministic K rows of request `rid` at positions [start, start+count) (exact in fp16)."""
    pos = torch.arange(start, start + count, dtype=torch.float32)[:, None, None]
    head = torch.arange(hkv, dtype=torch.float32)[None, :, None]
    col = torch.arange(d, dtype=torch.float32)[None, None, :]
    return ((rid * 7 + pos * 3 + head * 5 + col) % 1021).to(torch.float16)


def test_churn_with_compaction_keeps_every_request_bit_exact() -> None:
    from scheduler import KVBlockManager

    ops = _ops()
    rng = random.Random(11)
    layers, bs, hkv, d, pages = 2, 16, 2, 64, 600
    mgr = KVBlockManager(pages, bs, max_blocks_per_request=64)
    pools_k = torch.zeros((layers, pages, hkv, bs, d), dtype=torch.float16, device=DEVICE)
    pools_v = torch.zeros_like(pools_k)
    live: dict[str, int] = {}
    counter = 0
    copies = 0
    for step in range(30):
        for rid in list(live):
            if rng.random() < 0.2:
                mgr.free_request(rid)
                del live[rid]
        while len(live) < 12:
            n = rng.randint(1, 600)
            rid = f"{counter}"
            mgr.add_request(rid, n, staging=True)
            rows = _token_rows(counter, 0, n, hkv, d).to(DEVICE)
            slots = torch.tensor(mgr.slots(rid, 0, n), dtype=torch.int64, device=DEVICE)
            for layer in range(layers):
                ops.kv_append(rows, rows + layer, slots, pools_k[layer], pools_v[layer])
            live[rid] = counter
            counter += 1
        src, dst = mgr.compact()
        if src:
            copies += len(src)
            ops.kv_copy_pages(pools_k, pools_v, torch.tensor(src, device=DEVICE), torch.tensor(dst, device=DEVICE))
        for rid, num in live.items():  # one decode token each
            slots = torch.tensor(mgr.slots_for_append(rid, 1), dtype=torch.int64, device=DEVICE)
            rows = _token_rows(num, mgr.requests[rid].length - 1, 1, hkv, d).to(DEVICE)
            for layer in range(layers):
                ops.kv_append(rows, rows + layer, slots, pools_k[layer], pools_v[layer])
        order = list(live)
        tables = torch.tensor(mgr.block_table_rows(order), dtype=torch.int32, device=DEVICE)
        lens = torch.tensor(mgr.lengths(order), dtype=torch.int32, device=DEVICE)
        for layer in range(layers):
            k, v = ops.kv_gather(pools_k[layer], pools_v[layer], tables, lens)
            for i, rid in enumerate(order):
                n = mgr.requests[rid].length
                expect = _token_rows(live[rid], 0, n, hkv, d).to(DEVICE).transpose(0, 1)
                assert torch.equal(k[i, :, :n], expect), (step, rid, layer)
                assert torch.equal(v[i, :, :n], expect + layer), (step, rid, layer)
    assert copies > 0
