"""Pins the torch restatement of the reference's CPU decode composition (oracle/reference_torch.py, the
timed CPU baseline) against the fixtures made by running the reference itself: the per-request pools
it fills are bit-identical (sha256 of every request's K and V pool) and so is the attention output."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
import pkv_testlib as lib
from oracle import reference_torch as ref


@pytest.mark.parametrize("make", [cases.config1, cases.decode_fp16, cases.decode_bf16], ids=lambda m: m.__name__)
def test_reference_torch_decode_step_reproduces_the_reference(make) -> None:
    case = make()
    group = case.num_q_heads // case.num_kv_heads
    caches = []
    for b in range(case.batch):
        cache = ref.RequestCache(case.num_q_heads, case.head_dim, case.pages_per_request, case.block_size,
                                 case.dtype, case.tables()[b])
        if case.prefix_lens[b]:
            k = ref.repeat_kv(case.prefix_k[b].permute(1, 0, 2)[None], group)
            v = ref.repeat_kv(case.prefix_v[b].permute(1, 0, 2)[None], group)
            cache.append_blocks(k, v)
        caches.append(cache)
    out = ref.decode_step_layer(case.query[:, :, None, :], case.new_k[:, :, None, :], case.new_v[:, :, None, :],
                                caches, case.num_kv_heads)
    g = lib.golden()
    for b, cache in enumerate(caches):
        assert lib.sha(lib.np_bits(cache.key_blocks)) == g[f"{case.name}/pool_k_sha/{b}"].tobytes().hex(), b
        assert lib.sha(lib.np_bits(cache.value_blocks)) == g[f"{case.name}/pool_v_sha/{b}"].tobytes().hex(), b
    got = lib.np_bits(out[:, :, 0, :])
    np.testing.assert_array_equal(got, g[f"{case.name}/out"])


def test_reference_torch_gather_views_match_the_table_order() -> None:
    cache = ref.RequestCache(2, 4, 4, 2, torch.float32, [2, 0, 3])
    rows = torch.arange(5 * 2 * 4, dtype=torch.float32).view(1, 2, 5, 4)
    cache.append_blocks(rows, -rows)
    k, v = cache.as_tensors()
    assert torch.equal(k, rows) and torch.equal(v, -rows)
    contiguous = ref.RequestCache(2, 4, 4, 2, torch.float32, [1, 2, 3])
    contiguous.append_blocks(rows, rows)
    k, _ = contiguous.as_tensors()
    assert torch.equal(k, rows) and k.data_ptr() == contiguous.key_blocks[0, 0, 1].data_ptr()
