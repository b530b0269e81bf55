"""The drop-ins for the reference's attention dispatch, driven the way the reference's own tests drive it.

* tests/unit/test_tp_runtime.py:760-827 of the reference: batched native paged decode over caches with
  their own pools (seeds 0 and 7, pools of uneven sizes) equals the dense fp32 reference of every row
  (rtol = atol = 1e-4) and makes no dense view of the cache. Here also over one shared pool.
* tests/unit/test_engine.py:299-442 of the reference (batched step == sequential step): several
  requests decode several steps through _tp_full_attention_batch_paged_or_dense and, on an identical
  copy of their caches, one at a time through _tp_full_attention_paged_or_dense; the greedy tokens of a
  fixed vocabulary projection are identical, the outputs agree within the path's tolerance and match
  the oracle, each step appends once per cache and no dense view is ever made.
* a prefill chunk through _tp_full_attention_paged_or_dense (the reference's dense causal path) matches
  the oracle's causal attention.

The reference's config / weights / runtime are stood in for as its tests and make_golden.py do: the
o_proj is the identity, the gate is +100 (sigmoid == 1), the all-reduce is the identity.
"""

from __future__ import annotations

import contextlib
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import pkv_testlib as lib
from oracle import paged_kv_oracle as oracle

pytestmark = pytest.mark.gpu
DEVICE = "cuda:0"


def _fakes():
    from tp_runtime import PagedAttentionDispatchStats

    runtime = SimpleNamespace(config=SimpleNamespace(world_size=1, rank=0), paged_attention_stats=PagedAttentionDispatchStats(),
                              profile_scope=lambda _name: contextlib.nullcontext(), all_reduce_sum=lambda t: t)
    weights = SimpleNamespace(linear=lambda hidden, _name: hidden)
    return SimpleNamespace(), weights, runtime, SimpleNamespace(o_proj=None)


def _dense_decode_fp32(query, key, value):
    scores = torch.matmul(query.float(), key.float().transpose(2, 3)) * (query.shape[-1] ** -0.5)
    return torch.matmul(torch.softmax(scores, dim=-1, dtype=torch.float32), value.float())


@pytest.mark.parametrize("seed,seqs,shared", [(0, (3, 5), False), (7, (1, 9, 4), False), (0, (3, 5), True),
                                              (7, (1, 9, 4), True)])
def test_batched_native_decode_matches_dense_reference_without_dense_views(seed, seqs, shared) -> None:
    from decode_state import FullAttentionCache, PagedKVBlockPool, batch_page_tables
    from tp_runtime import _tp_full_attention_batch_native_paged_decode

    torch.manual_seed(seed)
    pool = PagedKVBlockPool.shared(64, 2, 4, block_size=2, dtype=torch.float32, device=DEVICE) if shared else None
    caches, keys, values = [], [], []
    for row, seq in enumerate(seqs):
        cache = FullAttentionCache(block_size=2, pool=pool)
        key = torch.randn((1, 2, seq, 4), device=DEVICE) + row
        value = torch.randn((1, 2, seq, 4), device=DEVICE) - row
        cache.append_blocks(key, value)
        caches.append(cache)
        keys.append(key)
        values.append(value)
    if not shared:
        assert len({cache.key_blocks.shape[0] for cache in caches}) > 1 or len(seqs) == 2
    query = torch.randn((len(seqs), 2, 1, 4), device=DEVICE)
    page_tables = batch_page_tables(caches)
    actual = _tp_full_attention_batch_native_paged_decode(query, page_tables, caches)
    expected = torch.cat([_dense_decode_fp32(query[r:r + 1], keys[r], values[r]) for r in range(len(seqs))])
    torch.testing.assert_close(actual, expected, rtol=1e-4, atol=1e-4)
    assert all(c.stats().contiguous_view_calls == 0 and c.stats().gather_view_calls == 0 for c in caches)


def _copy_caches(caches, pool):
    """Caches on `pool` holding the same tokens at the same page ids (the pools are bit-identical copies)."""
    from decode_state import FullAttentionCache

    pool.key_blocks.copy_(caches[0].pool.key_blocks)
    pool.value_blocks.copy_(caches[0].pool.value_blocks)
    out = []
    for c in caches:
        twin = FullAttentionCache(block_size=c.block_size, pool=pool)
        twin.block_table = list(c.block_table)
        twin.valid = c.valid
        out.append(twin)
    pool.allocator.take([p for c in caches for p in c.block_table])
    return out


def test_batched_step_produces_the_same_tokens_as_sequential_steps() -> None:
    from decode_state import FullAttentionCache, PagedKVBlockPool
    from tp_runtime import _tp_full_attention_batch_paged_or_dense, _tp_full_attention_paged_or_dense

    gen = torch.Generator().manual_seed(299)
    hq, hkv, d, bs, vocab = 16, 2, 256, 16, 512
    prompts = [37, 300, 5]
    steps = 4
    config, weights, runtime_b, mapping = _fakes()
    _, _, runtime_s, _ = _fakes()
    pool_b = PagedKVBlockPool.shared(256, hkv, d, block_size=bs, dtype=torch.float16, device=DEVICE)
    pool_s = PagedKVBlockPool.shared(256, hkv, d, block_size=bs, dtype=torch.float16, device=DEVICE)
    batched = []
    for n in prompts:
        cache = FullAttentionCache(capacity_hint=n + steps, block_size=bs, pool=pool_b)
        cache.append_blocks(torch.randn((1, hkv, n, d), generator=gen).to(torch.float16).to(DEVICE),
                            torch.randn((1, hkv, n, d), generator=gen).to(torch.float16).to(DEVICE))
        batched.append(cache)
    sequential = _copy_caches(batched, pool_s)
    lm_head = torch.randn((vocab, hq * d), generator=gen).to(DEVICE)
    tokens_b, tokens_s = [], []
    for step in range(steps):
        q = torch.randn((len(prompts), hq, 1, d), generator=gen).to(torch.float16).to(DEVICE)
        k = torch.randn((len(prompts), hkv, 1, d), generator=gen).to(torch.float16).to(DEVICE)
        v = torch.randn((len(prompts), hkv, 1, d), generator=gen).to(torch.float16).to(DEVICE)
        gate = torch.full((len(prompts), 1, hq * d), 100.0, dtype=torch.float16, device=DEVICE)
        before = [c.stats() for c in batched]
        for r, cache in enumerate(batched):  # the reference's per-row append loop (src/tp_runtime.py:2481-2483)
            cache.append_blocks(k[r:r + 1], v[r:r + 1])
        hidden = torch.zeros((len(prompts), 1, hq * d), dtype=torch.float16, device=DEVICE)
        positions = torch.tensor([c.valid - 1 for c in batched], device=DEVICE)
        out_b = _tp_full_attention_batch_paged_or_dense(q, gate, hidden, mapping, config, weights, runtime_b,
                                                        caches=batched, position_offsets=positions)
        outs_s = []
        for r, cache in enumerate(sequential):
            cache.append_blocks(k[r:r + 1], v[r:r + 1])
            outs_s.append(_tp_full_attention_paged_or_dense(q[r:r + 1], gate[r:r + 1], hidden[r:r + 1], mapping,
                                                            config, weights, runtime_s, cache=cache,
                                                            position_offset=cache.valid - 1))
        out_s = torch.cat(outs_s)
        assert out_b.shape == (len(prompts), 1, hq * d)
        tokens_b.append((out_b[:, 0].float() @ lm_head.T).argmax(-1).tolist())
        tokens_s.append((out_s[:, 0].float() @ lm_head.T).argmax(-1).tolist())
        got_b = lib.as_f32(lib.np_bits(out_b[:, 0].view(len(prompts), hq, d)), "float16")
        got_s = lib.as_f32(lib.np_bits(out_s[:, 0].view(len(prompts), hq, d)), "float16")
        lib.assert_close(got_b, got_s, "float16", f"batched vs sequential, step {step}")
        tables = [c.block_table for c in batched]
        lens = [c.valid for c in batched]
        pk, pv = lib.np_bits(pool_b.key_blocks), lib.np_bits(pool_b.value_blocks)
        expected = oracle.decode_attention(lib.as_f32(lib.np_bits(q[:, :, 0]), "float16"), pk, pv, tables, lens,
                                           dtype="float16", round_probs=False)
        lib.assert_close(got_b, expected, "float16", f"batched vs oracle, step {step}")
        for b0, c in zip(before, batched):
            after = c.stats()
            assert after.append_calls == b0.append_calls + 1
            assert after.contiguous_view_calls + after.gather_view_calls == 0
    assert tokens_b == tokens_s
    assert runtime_b.paged_attention_stats.native_hits == steps
    assert runtime_s.paged_attention_stats.native_hits == steps * len(prompts)
    assert runtime_b.paged_attention_stats.dense_fallbacks == 0


def test_prefill_chunk_through_the_single_dispatch_matches_oracle() -> None:
    from decode_state import FullAttentionCache, PagedKVBlockPool
    from tp_runtime import _tp_full_attention_paged_or_dense

    gen = torch.Generator().manual_seed(606)
    hq, hkv, d, bs = 16, 2, 256, 16
    prefix, chunk = 70, 129
    config, weights, runtime, mapping = _fakes()
    pool = PagedKVBlockPool.shared(64, hkv, d, block_size=bs, dtype=torch.bfloat16, device=DEVICE)
    cache = FullAttentionCache(block_size=bs, pool=pool)
    cache.append_blocks(torch.randn((1, hkv, prefix, d), generator=gen).to(torch.bfloat16).to(DEVICE),
                        torch.randn((1, hkv, prefix, d), generator=gen).to(torch.bfloat16).to(DEVICE))
    cache.append_blocks(torch.randn((1, hkv, chunk, d), generator=gen).to(torch.bfloat16).to(DEVICE),
                        torch.randn((1, hkv, chunk, d), generator=gen).to(torch.bfloat16).to(DEVICE))
    q = torch.randn((1, hq, chunk, d), generator=gen).to(torch.bfloat16).to(DEVICE)
    gate = torch.full((1, chunk, hq * d), 100.0, dtype=torch.bfloat16, device=DEVICE)
    hidden = torch.zeros((1, chunk, hq * d), dtype=torch.bfloat16, device=DEVICE)
    out = _tp_full_attention_paged_or_dense(q, gate, hidden, mapping, config, weights, runtime, cache=cache,
                                            position_offset=prefix)
    got = lib.as_f32(lib.np_bits(out[0].view(chunk, hq, d)), "bfloat16")
    pk, pv = lib.np_bits(pool.key_blocks), lib.np_bits(pool.value_blocks)
    qf = lib.as_f32(lib.np_bits(q[0]), "bfloat16")  # (hq, chunk, d)
    expected = oracle.prefill_attention(qf, pk, pv, cache.block_table, cache.valid, dtype="bfloat16",
                                        round_probs=False).transpose(1, 0, 2)
    lib.assert_close(got, expected, "bfloat16", "prefill chunk through the dispatch")
    assert cache.stats().gather_view_calls == 0 and runtime.paged_attention_stats.native_hits == 1
    with pytest.raises(ValueError, match="must end at"):
        _tp_full_attention_paged_or_dense(q, gate, hidden, mapping, config, weights, runtime, cache=cache,
                                          position_offset=prefix - 1)


def test_append_blocks_flags_a_table_entry_outside_the_pool() -> None:
    """The table-addressed append skips (and flags) a token whose page id is outside the pool."""
    import paged_kv_ops as ops

    pool_k = torch.zeros((4, 2, 16, 64), dtype=torch.float16, device=DEVICE)
    pool_v = torch.zeros_like(pool_k)
    table = torch.tensor([2, 9], dtype=torch.int64, device=DEVICE)  # page 9 is outside the pool
    rows = torch.randn((20, 2, 64), device=DEVICE).to(torch.float16)
    flag = ops.new_error_flag(DEVICE)
    ops.kv_append_positions(rows, rows, table, 0, pool_k, pool_v, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) & ops.DEVERR_PAGE_OUT_OF_RANGE
    assert torch.equal(pool_k[2].transpose(0, 1), rows[:16])
    assert int(torch.count_nonzero(pool_k[[0, 1, 3]])) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_steps_match_prefill_rows(dtype) -> None:
    """tests/unit/test_reference_ops.py:298-350 of the reference (decode steps == prefill logits), for the
    attention alone: a 21-token chunk through _tp_full_attention_paged_or_dense as one prefill call gives,
    row for row, what the same tokens give appended and decoded one at a time through the same dispatch
    (prefill kernel against decode kernel, both fp32-accurate in P), and both match the oracle."""
    from decode_state import FullAttentionCache, PagedKVBlockPool
    from tp_runtime import _tp_full_attention_paged_or_dense

    gen = torch.Generator().manual_seed(298)
    hq, hkv, d, bs = 16, 2, 256, 16
    prefix, chunk = 37, 21
    name = "bfloat16" if dtype == torch.bfloat16 else "float16"
    keys = torch.randn((1, hkv, prefix + chunk, d), generator=gen).to(dtype).to(DEVICE)
    values = torch.randn((1, hkv, prefix + chunk, d), generator=gen).to(dtype).to(DEVICE)
    q = torch.randn((1, hq, chunk, d), generator=gen).to(dtype).to(DEVICE)
    config, weights, runtime_p, mapping = _fakes()
    _, _, runtime_d, _ = _fakes()
    caches = []
    for _ in range(2):
        pool = PagedKVBlockPool.shared(16, hkv, d, block_size=bs, dtype=dtype, device=DEVICE)
        cache = FullAttentionCache(block_size=bs, pool=pool)
        cache.append_blocks(keys[:, :, :prefix], values[:, :, :prefix])
        caches.append(cache)
    prefill_cache, decode_cache = caches
    prefill_cache.append_blocks(keys[:, :, prefix:], values[:, :, prefix:])
    gate = torch.full((1, chunk, hq * d), 100.0, dtype=dtype, device=DEVICE)
    hidden = torch.zeros((1, chunk, hq * d), dtype=dtype, device=DEVICE)
    rows = _tp_full_attention_paged_or_dense(q, gate, hidden, mapping, config, weights, runtime_p,
                                             cache=prefill_cache, position_offset=prefix)
    steps = []
    for t in range(chunk):
        decode_cache.append_blocks(keys[:, :, prefix + t:prefix + t + 1], values[:, :, prefix + t:prefix + t + 1])
        steps.append(_tp_full_attention_paged_or_dense(q[:, :, t:t + 1], gate[:, t:t + 1], hidden[:, t:t + 1], mapping,
                                                       config, weights, runtime_d, cache=decode_cache,
                                                       position_offset=prefix + t))
    stepped = torch.cat(steps, dim=1)
    assert rows.shape == stepped.shape == (1, chunk, hq * d)
    got_rows = lib.as_f32(lib.np_bits(rows[0].view(chunk, hq, d)), name)
    got_steps = lib.as_f32(lib.np_bits(stepped[0].view(chunk, hq, d)), name)
    lib.assert_close(got_steps, got_rows, name, "decode steps vs prefill rows")
    pk, pv = lib.np_bits(prefill_cache.pool.key_blocks), lib.np_bits(prefill_cache.pool.value_blocks)
    expected = oracle.prefill_attention(lib.as_f32(lib.np_bits(q[0]), name), pk, pv, prefill_cache.block_table,
                                        prefill_cache.valid, dtype=name, round_probs=False).transpose(1, 0, 2)
    lib.assert_close(got_rows, expected, name, "prefill rows vs oracle")
    lib.assert_close(got_steps, expected, name, "decode steps vs oracle")
    assert runtime_p.paged_attention_stats.native_hits == 1
    assert runtime_d.paged_attention_stats.native_hits == chunk
    assert runtime_d.paged_attention_stats.dense_fallbacks == 0
