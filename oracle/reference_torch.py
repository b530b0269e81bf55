"""The reference's CPU composition for a batched decode step, restated in torch -- TEST INFRASTRUCTURE ONLY.

Used as the timed CPU baseline (bench.py's `cpu_baseline` leg and `--impl reference`) and checked by
tests/ against the fixtures that tests/golden/make_golden.py made by running the reference itself.
It performs the same torch operations, in the same order and on the same layouts, as the reference's
dense path for one full-attention layer (paths relative to the reference project root):

  per-request pools (1, H, pages, block_size, D) of REPEATED heads   src/decode_state.py:13-84
  FullAttentionCache.append_blocks: slice assignment per block span    src/decode_state.py:271-293
  the per-row append loop of the batched step                          src/tp_runtime.py:2481-2483
  _repeat_kv of the new K/V before the append                          src/tp_runtime.py:2736-2741
  as_tensors: as_strided view of a contiguous table, else index_select src/decode_state.py:295-303, 382-404
  batch_kv_tensors: zero-padded stack + valid mask                     src/decode_state.py:501-542
  masked dense attention, fp32 scores and softmax, probs cast to the   src/tp_runtime.py:2558-2605
  query dtype, probs @ V in that dtype

The gate, o_proj and all-reduce around it are left out (the same identity stand-ins make_golden.py
uses), since they are not part of the paged KV path. Nothing in the product imports this module.
"""

from __future__ import annotations

from typing import Sequence

import torch


class RequestCache:
    """One request's pages of one layer in the reference's layout: a private pool holding the
    Hq/TP repeated heads, a block table (list of page ids) and the number of valid tokens."""

    def __init__(self, num_heads: int, head_dim: int, num_pages: int, block_size: int, dtype: torch.dtype,
                 block_table: Sequence[int]) -> None:
        self.block_size = block_size
        self.key_blocks = torch.zeros((1, num_heads, num_pages, block_size, head_dim), dtype=dtype)
        self.value_blocks = torch.zeros_like(self.key_blocks)
        self.block_table = list(block_table)
        self.valid = 0

    def append_blocks(self, key: torch.Tensor, value: torch.Tensor) -> None:
        """key/value (1, H, T, D): written span by span into the table's pages (decode_state.py:271-293)."""
        seq = key.shape[2]
        done = 0
        while done < seq:
            pos = self.valid + done
            page = self.block_table[pos // self.block_size]
            off = pos % self.block_size
            take = min(seq - done, self.block_size - off)
            self.key_blocks[:, :, page, off:off + take] = key[:, :, done:done + take]
            self.value_blocks[:, :, page, off:off + take] = value[:, :, done:done + take]
            done += take
        self.valid += seq

    def _dense(self, blocks: torch.Tensor) -> torch.Tensor:
        table = self.block_table
        n = len(table)
        if table == list(range(table[0], table[0] + n)):  # contiguous: a strided view, no copy
            view = blocks.as_strided((1, blocks.shape[1], n * self.block_size, blocks.shape[4]),
                                     (blocks.stride(0), blocks.stride(1), blocks.stride(3), blocks.stride(4)),
                                     storage_offset=blocks.storage_offset() + table[0] * blocks.stride(2))
        else:
            view = blocks.index_select(2, torch.tensor(table, dtype=torch.long)).reshape(
                1, blocks.shape[1], n * self.block_size, blocks.shape[4])
        return view[:, :, :self.valid]

    def as_tensors(self) -> tuple[torch.Tensor, torch.Tensor]:
        return self._dense(self.key_blocks), self._dense(self.value_blocks)


def repeat_kv(x: torch.Tensor, repeats: int) -> torch.Tensor:
    """(B, Hkv, T, D) -> (B, Hkv*repeats, T, D), each KV head repeated for its query heads."""
    if repeats == 1:
        return x
    b, h, t, d = x.shape
    return x[:, :, None].expand(b, h, repeats, t, d).reshape(b, h * repeats, t, d)


def batch_kv_tensors(caches: Sequence[RequestCache]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Zero-padded (B, H, max_valid, D) keys and values and the (B, max_valid) valid mask."""
    max_valid = max(c.valid for c in caches)
    first_k, first_v = caches[0].as_tensors()
    batch, heads, dim = len(caches), first_k.shape[1], first_k.shape[3]
    keys = torch.zeros(batch, heads, max_valid, dim, dtype=first_k.dtype)
    values = torch.zeros_like(keys)
    mask = torch.zeros(batch, max_valid, dtype=torch.bool)
    for i, cache in enumerate(caches):
        k, v = (first_k, first_v) if i == 0 else cache.as_tensors()
        keys[i:i + 1, :, :cache.valid] = k
        values[i:i + 1, :, :cache.valid] = v
        mask[i, :cache.valid] = True
    return keys, values, mask


def decode_step_layer(query: torch.Tensor, new_key: torch.Tensor, new_value: torch.Tensor,
                      caches: Sequence[RequestCache], num_kv_heads: int) -> torch.Tensor:
    """One layer of the reference's batched decode step on the host: query (B, Hq, 1, D); new_key /
    new_value (B, Hkv, 1, D) -> attention output (B, Hq, 1, D) in the query dtype.

    Appends each row's token (repeated to Hq heads) into its cache, gathers every request's K/V dense
    and padded, and runs the masked dense attention with the reference's rounding points."""
    batch, hq, _, dim = query.shape
    repeats = hq // num_kv_heads
    key = repeat_kv(new_key, repeats)
    value = repeat_kv(new_value, repeats)
    for r in range(batch):
        caches[r].append_blocks(key[r:r + 1], value[r:r + 1])
    keys, values, valid = batch_kv_tensors(caches)
    positions = torch.tensor([c.valid - 1 for c in caches], dtype=torch.long)
    scores = torch.matmul(query.float(), keys.float().transpose(2, 3)) * (dim ** -0.5)
    key_pos = torch.arange(keys.shape[2])
    masked = ((key_pos[None, :] > positions[:, None]) | ~valid)[:, None, None, :]
    scores = scores.masked_fill(masked, torch.finfo(scores.dtype).min)
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32).to(query.dtype)
    return torch.matmul(probs, values)
