"""Host-side behaviour of the dispatch drop-ins (no GPU): the reference's dispatch counters keep their
meaning (tests/unit/test_tp_runtime.py:713-724 of the reference), and a CPU cache raises instead of
falling back to dense attention."""

from __future__ import annotations

import contextlib
from types import SimpleNamespace

import pytest
import torch


def _runtime():
    from tp_runtime import PagedAttentionDispatchStats

    return SimpleNamespace(paged_attention_stats=PagedAttentionDispatchStats(),
                           profile_scope=lambda _name: contextlib.nullcontext(), all_reduce_sum=lambda t: t)


def test_dispatch_records_native_hit_like_the_reference() -> None:
    from tp_runtime import _record_native_paged_dispatch

    runtime = _runtime()
    _record_native_paged_dispatch(runtime, "no_kernel", native=True)
    stats = runtime.paged_attention_stats
    assert (stats.calls, stats.eligible, stats.native_hits, stats.dense_fallbacks, stats.fallback_no_kernel) == (
        1, 1, 1, 0, 0)
    _record_native_paged_dispatch(runtime, "per_request_pools", native=False)
    assert (stats.calls, stats.dense_fallbacks, stats.fallback_per_request_pools, stats.eligible) == (2, 1, 1, 1)
    _record_native_paged_dispatch(SimpleNamespace(), "no_kernel", native=True)  # no stats: nothing to count


def test_dispatch_on_a_cpu_cache_raises_instead_of_falling_back() -> None:
    from decode_state import FullAttentionCache, PagedKVBlockPool
    from tp_runtime import _tp_full_attention_paged_or_dense

    pool = PagedKVBlockPool.shared(8, 2, 16, block_size=4, dtype=torch.float32, device="cpu")
    cache = FullAttentionCache(block_size=4, pool=pool)
    cache.block_table = pool.allocate(2)
    cache.valid = 5
    query = torch.zeros((1, 2, 1, 16))
    hidden = torch.zeros((1, 1, 32))
    weights = SimpleNamespace(linear=lambda h, _n: h)
    with pytest.raises(RuntimeError, match="must be CUDA"):
        _tp_full_attention_paged_or_dense(query, torch.zeros((1, 1, 32)), hidden, SimpleNamespace(o_proj=None),
                                          SimpleNamespace(), weights, _runtime(), cache=cache, position_offset=4)
