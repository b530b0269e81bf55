"""Generates tests/golden/golden.npz by running the REFERENCE's own Python code on seeded inputs.

Run where the reference checkout is importable (pass its src/ directory with --reference-src). The GPU box never runs this file; tests only read the .npz it writes. The
reference code paths exercised (paths relative to the reference project root):

  FullAttentionCache.append_blocks / as_tensors      src/decode_state.py:271-303
  batch_kv_tensors                                   src/decode_state.py:501-542
  PagedKVBlockPool.allocate / release                src/decode_state.py:72-84
  _repeat_kv (GQA head repetition before append)     src/tp_runtime.py:2736-2741
  _tp_full_attention_batch_dense_from_kv (decode)    src/tp_runtime.py:2558-2609
  _tp_full_attention_dense_from_kv (causal prefill)  src/tp_runtime.py:698-730
  tp_full_attention (norm, RoPE, repeat, append)     src/tp_runtime.py:499-548
  _tp_full_attention_batch (batched decode)          src/tp_runtime.py:2437-2490
  rms_norm / rotary_embeddings / apply_rotary_pos_emb  src/reference_ops.py:166-169, :203-224
  _tp_full_attention_finish_from_heads (gate, o_proj)  src/tp_runtime.py:672-695
  linear / dequantize_fp8_weight (FP8 block scales)   src/reference_ops.py:436-506

The dense attention functions are driven with stand-ins for the parts around attention: o_proj is
the identity, the output gate is +100 (sigmoid == 1 exactly in every dtype), the all-reduce is the
identity and world_size is 1, so their result is the attention output itself. Request pools are
zero-filled after allocation so that pool hashes do not depend on uninitialised memory.

    python tests/golden/make_golden.py [--reference-src PATH]
"""

from __future__ import annotations

import argparse
import contextlib
import os
import hashlib
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import cases  # noqa: E402


def _fakes(num_heads: int, head_dim: int, dtype: torch.dtype):
    config = SimpleNamespace(full_attention=SimpleNamespace(num_heads=num_heads, head_dim=head_dim))
    runtime = SimpleNamespace(
        config=SimpleNamespace(world_size=1, rank=0),
        profile_scope=lambda _name: contextlib.nullcontext(),
        all_reduce_sum=lambda tensor: tensor,
    )
    weights = SimpleNamespace(linear=lambda hidden, _tensor: hidden)
    mapping = SimpleNamespace(o_proj=None)
    return config, runtime, weights, mapping


def _sha(tensor: torch.Tensor) -> str:
    return hashlib.sha256(cases.to_bits(tensor).tobytes()).hexdigest()


def _build_caches(ds, tp, case, lens_prefix, new_k=None, new_v=None, chunk_k=None, chunk_v=None):
    group = case.num_q_heads // case.num_kv_heads
    caches = []
    for b in range(case.batch):
        cache = ds.FullAttentionCache(block_size=case.block_size)
        dummy = torch.zeros((1, case.num_q_heads, 1, case.head_dim), dtype=case.dtype)
        cache.pool.ensure_initialized(dummy, dummy, case.pages_per_request)
        cache.pool.key_blocks.zero_()
        cache.pool.value_blocks.zero_()
        table = case.tables()[b]
        cache.block_table = list(table)
        used = set(table)
        cache.pool.free_blocks = [p for p in range(case.pages_per_request) if p not in used]
        if lens_prefix[b] > 0:
            k = tp._repeat_kv(case.prefix_k[b].permute(1, 0, 2)[None], group)
            v = tp._repeat_kv(case.prefix_v[b].permute(1, 0, 2)[None], group)
            cache.append_blocks(k, v)
        if new_k is not None:
            cache.append_blocks(tp._repeat_kv(new_k[b][:, None, :][None], group),
                                tp._repeat_kv(new_v[b][:, None, :][None], group))
        if chunk_k is not None:
            cache.append_blocks(tp._repeat_kv(chunk_k[b].permute(1, 0, 2)[None], group),
                                tp._repeat_kv(chunk_v[b].permute(1, 0, 2)[None], group))
        caches.append(cache)
    return caches


def decode_golden(ds, tp, case: cases.DecodeCase, out: dict) -> None:
    new_k = case.new_k if case.append_new else None
    new_v = case.new_v if case.append_new else None
    caches = _build_caches(ds, tp, case, case.prefix_lens, new_k=new_k, new_v=new_v)
    lens = case.lens
    live = [b for b in range(case.batch) if lens[b] > 0]
    config, runtime, weights, mapping = _fakes(case.num_q_heads, case.head_dim, case.dtype)
    hq, d = case.num_q_heads, case.head_dim
    query = case.query[live][:, :, None, :]
    gate = torch.full((len(live), 1, hq * d), 100.0, dtype=case.dtype)
    hidden = torch.zeros((len(live), 1, hq * d), dtype=case.dtype)
    positions = torch.tensor([lens[b] - 1 for b in live], dtype=torch.long)
    res = tp._tp_full_attention_batch_dense_from_kv(
        query, gate, hidden, mapping, config, weights, runtime,
        caches=[caches[b] for b in live], position_offsets=positions,
    )
    full = torch.zeros((case.batch, hq, d), dtype=case.dtype)  # empty rows: zeros (fp8_linear_cuda.cu:987-991)
    full[live] = res.reshape(len(live), hq, d)
    out[f"{case.name}/out"] = cases.to_bits(full)
    for b in range(case.batch):
        out[f"{case.name}/pool_k_sha/{b}"] = np.frombuffer(bytes.fromhex(_sha(caches[b].key_blocks)), dtype=np.uint8)
        out[f"{case.name}/pool_v_sha/{b}"] = np.frombuffer(bytes.fromhex(_sha(caches[b].value_blocks)), dtype=np.uint8)


def prefill_golden(ds, tp, case: cases.PrefillCase, out: dict) -> None:
    caches = _build_caches(ds, tp, case, case.prefix_lens, chunk_k=case.chunk_k, chunk_v=case.chunk_v)
    config, runtime, weights, mapping = _fakes(case.num_q_heads, case.head_dim, case.dtype)
    hq, d = case.num_q_heads, case.head_dim
    for b in range(case.batch):
        t = case.chunk_lens[b]
        key, value = caches[b].as_tensors()
        query = case.query[b].permute(1, 0, 2)[None]
        gate = torch.full((1, t, hq * d), 100.0, dtype=case.dtype)
        hidden = torch.zeros((1, t, hq * d), dtype=case.dtype)
        res = tp._tp_full_attention_dense_from_kv(
            query, gate, key, value, hidden, mapping, config, weights, runtime, position_offset=case.prefix_lens[b]
        )
        out[f"{case.name}/out/{b}"] = cases.to_bits(res.reshape(t, hq, d))
        out[f"{case.name}/pool_k_sha/{b}"] = np.frombuffer(bytes.fromhex(_sha(caches[b].key_blocks)), dtype=np.uint8)
        out[f"{case.name}/pool_v_sha/{b}"] = np.frombuffer(bytes.fromhex(_sha(caches[b].value_blocks)), dtype=np.uint8)


def norm_rope_golden(ds, tp, ro, case: cases.NormRopeCase, out: dict) -> None:
    """Runs the reference's full-attention layer entry (tp_full_attention, or _tp_full_attention_batch for
    the decode case) on the case's projections with a cache holding the prefix, and records what the
    fused kernel must reproduce: the normalised + rotated query (the composition of
    src/tp_runtime.py:510-517 applied with the reference's own functions), the new tokens' K and V as
    the cache stores them, the cos/sin rows, and the layer output (the attention, as the gate is +100)."""
    d, hq_local = case.head_dim, case.local_q_heads
    group = case.num_q_heads // case.num_kv_heads
    head_start = case.rank * hq_local
    full = SimpleNamespace(num_heads=case.num_q_heads, num_key_value_heads=case.num_kv_heads, head_dim=d,
                           paged_kv_metadata=False, native_paged_attention=False)
    config = SimpleNamespace(full_attention=full, rms_norm_eps=case.eps, rope_theta=case.rope_theta,
                             partial_rotary_factor=case.partial_rotary_factor)
    runtime = SimpleNamespace(
        config=SimpleNamespace(world_size=case.world_size, rank=case.rank),
        profile_scope=lambda _name: contextlib.nullcontext(),
        all_reduce_sum=lambda tensor: tensor,
        paged_attention_stats=tp.PagedAttentionDispatchStats(),
    )
    mapping = SimpleNamespace(q_proj="q", k_proj="k", v_proj="v", q_norm="qn", k_norm="kn", o_proj="o")
    norms = {"qn": case.q_norm, "kn": case.k_norm}

    def weights_for(tensors):
        return SimpleNamespace(linear=lambda hidden, name: hidden if name == "o" else tensors[name],
                               tensor=lambda name: norms[name])

    caches = []
    for b in range(case.batch):
        cache = ds.FullAttentionCache(block_size=case.block_size)
        dummy = torch.zeros((1, hq_local, 1, d), dtype=case.dtype)
        cache.pool.ensure_initialized(dummy, dummy, case.pages_per_request)
        cache.pool.key_blocks.zero_()
        cache.pool.value_blocks.zero_()
        table = case.tables()[b]
        cache.block_table = list(table)
        cache.pool.free_blocks = [p for p in range(case.pages_per_request) if p not in set(table)]
        if case.prefix_lens[b] > 0:
            k = tp._repeat_kv(case.prefix_k[b].permute(1, 0, 2)[None], group)[:, head_start : head_start + hq_local]
            v = tp._repeat_kv(case.prefix_v[b].permute(1, 0, 2)[None], group)[:, head_start : head_start + hq_local]
            cache.append_blocks(k, v)
        caches.append(cache)
    if case.batched_decode:
        tensors = {
            "q": torch.stack([q.reshape(1, hq_local * 2 * d) for q in case.q_proj]),
            "k": torch.stack([k.reshape(1, case.num_kv_heads * d) for k in case.key]),
            "v": torch.stack([v.reshape(1, case.num_kv_heads * d) for v in case.value]),
        }
        hidden = torch.zeros((case.batch, 1, 8), dtype=case.dtype)
        res = tp._tp_full_attention_batch(hidden, mapping, config, weights_for(tensors), runtime, caches=caches,
                                          position_offsets=torch.tensor(case.prefix_lens, dtype=torch.long))
        outs = [res[b].reshape(1, hq_local, d) for b in range(case.batch)]
    else:
        outs = []
        for b in range(case.batch):
            t = case.new_lens[b]
            tensors = {"q": case.q_proj[b].reshape(1, t, hq_local * 2 * d),
                       "k": case.key[b].reshape(1, t, case.num_kv_heads * d),
                       "v": case.value[b].reshape(1, t, case.num_kv_heads * d)}
            hidden = torch.zeros((1, t, 8), dtype=case.dtype)
            res = tp.tp_full_attention(hidden, mapping, config, weights_for(tensors), runtime, cache=caches[b],
                                       position_offset=case.prefix_lens[b])
            outs.append(res.reshape(t, hq_local, d))
    for b in range(case.batch):
        t, p0 = case.new_lens[b], case.prefix_lens[b]
        query = case.q_proj[b][None].chunk(2, dim=-1)[0]  # (1, t, Hq_local, D)
        query = ro.rms_norm(query, case.q_norm, case.eps).transpose(1, 2)
        key = ro.rms_norm(case.key[b][None], case.k_norm, case.eps).transpose(1, 2)
        positions = torch.arange(p0, p0 + t).expand(1, t)
        cos, sin = ro.rotary_embeddings(positions, config, dtype=query.dtype)
        query, _ = ro.apply_rotary_pos_emb(query, key, cos, sin)
        k_dense, v_dense = caches[b].as_tensors()
        heads = [kl * group for kl in range(case.local_kv_heads)]  # first repeated copy of each stored KV head
        out[f"{case.name}/query/{b}"] = cases.to_bits(query[0].transpose(0, 1))
        out[f"{case.name}/key/{b}"] = cases.to_bits(k_dense[0, heads, p0 : p0 + t].transpose(0, 1))
        out[f"{case.name}/value/{b}"] = cases.to_bits(v_dense[0, heads, p0 : p0 + t].transpose(0, 1))
        out[f"{case.name}/cos/{b}"] = cases.to_bits(cos[0])
        out[f"{case.name}/sin/{b}"] = cases.to_bits(sin[0])
        out[f"{case.name}/out/{b}"] = cases.to_bits(outs[b])


def oproj_golden(tp, ro, case: cases.OProjCase, out: dict) -> None:
    """Runs the reference's output stage _tp_full_attention_finish_from_heads (src/tp_runtime.py:672-695)
    once per rank with that rank's row-parallel o_proj shard, through reference_ops.linear (the
    dequantise + float32 F.linear path, src/reference_ops.py:436-506), and records each rank's partial
    (the all-reduce input) and their sum as NCCL's SUM of two tensors of the hidden dtype computes it."""
    config = SimpleNamespace(full_attention=SimpleNamespace(num_heads=case.num_heads, head_dim=case.head_dim))
    batch, seq = case.heads.shape[0], case.heads.shape[2]
    hidden_states = torch.zeros((batch, seq, 8), dtype=case.hidden_dtype)
    mapping = SimpleNamespace(o_proj="o")
    partials = []
    for rank in range(case.world_size):
        heads, gate, weight, scale = case.rank_inputs(rank)
        captured = []

        def capture(tensor, captured=captured):
            captured.append(tensor.clone())
            return tensor

        runtime = SimpleNamespace(config=SimpleNamespace(world_size=case.world_size, rank=rank),
                                  profile_scope=lambda _name: contextlib.nullcontext(), all_reduce_sum=capture)
        weights = SimpleNamespace(linear=lambda x, _name, w=weight, s=scale: ro.linear(x, w, s))
        tp._tp_full_attention_finish_from_heads(heads, gate, hidden_states, mapping, config, weights, runtime,
                                                scope_prefix="oproj")
        partials.append(captured[0])
    total = partials[0]
    for p in partials[1:]:
        total = total + p
    n = case.name
    out[f"{n}/heads"] = cases.to_bits(case.heads)
    out[f"{n}/gate"] = cases.to_bits(case.gate)
    out[f"{n}/weight"] = case.weight.view(torch.uint8).numpy()
    out[f"{n}/scale_inv"] = cases.to_bits(case.scale_inv)
    for rank, p in enumerate(partials):
        out[f"{n}/partial{rank}"] = cases.to_bits(p.reshape(batch * seq, -1))
    out[f"{n}/out"] = cases.to_bits(total.reshape(batch * seq, -1))


def decode_state_golden(ds, out: dict) -> None:
    """The reference test's arange data (tests/unit/test_decode_state.py:18-23, :47-64): a 3-token
    prefill then 3 single-token appends with block_size 2, growing the table by doubling."""

    def kv(step: int, seq: int):
        count = 2 * seq * 4
        base = float(step * 1000)
        key = (base + torch.arange(count, dtype=torch.float32)).reshape(1, 2, seq, 4)
        value = (base + 0.5 + torch.arange(count, dtype=torch.float32)).reshape(1, 2, seq, 4)
        return key, value

    cache = ds.FullAttentionCache(block_size=2)
    appended = []
    for step, seq in ((0, 3), (1, 1), (2, 1), (3, 1)):
        key, value = kv(step, seq)
        appended.append((key, value))
        cache.append_blocks(key, value)
    k_dense, v_dense = cache.as_tensors()
    out["decode_state/block_table"] = np.asarray(cache.block_table, dtype=np.int64)
    out["decode_state/valid"] = np.asarray([cache.valid], dtype=np.int64)
    out["decode_state/k_dense"] = k_dense.numpy().copy()
    out["decode_state/v_dense"] = v_dense.numpy().copy()
    out["decode_state/growth_events"] = np.asarray([cache.growth_events], dtype=np.int64)
    # reordered table (tests/unit/test_decode_state.py:194-219)
    cache2 = ds.FullAttentionCache(capacity_hint=6, block_size=2)
    parts = [kv(i, 2) for i in range(3)]
    for key, value in parts:
        cache2.append(key, value)
    cache2.block_table = [2, 0, 1]
    for page, (key, value) in zip((2, 0, 1), parts):
        cache2.pool.key_blocks[:, :, page] = key
        cache2.pool.value_blocks[:, :, page] = value
    k2, v2 = cache2.as_tensors()
    out["decode_state/reordered_k"] = k2.numpy().copy()
    out["decode_state/reordered_v"] = v2.numpy().copy()


def allocator_golden(ds, out: dict) -> None:
    pool = ds.PagedKVBlockPool(block_size=2)
    dummy = torch.zeros((1, 1, 1, 1))
    results = []
    for op, arg in cases.allocator_script():
        if op == "init":
            pool.ensure_initialized(dummy, dummy, arg)
        elif op == "allocate":
            results.extend(pool.allocate(arg, dummy, dummy))
            results.append(-1)
        else:
            pool.release(list(arg))
    out["allocator/results"] = np.asarray(results, dtype=np.int64)
    out["allocator/free"] = np.asarray(pool.free_blocks, dtype=np.int64)


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference-src", default=os.environ.get("QWEN36_REFERENCE_SRC", ""), required=not os.environ.get("QWEN36_REFERENCE_SRC"))
    parser.add_argument("--out", default=str(HERE / "golden.npz"))
    args = parser.parse_args(argv)
    sys.path.insert(0, args.reference_src)
    import decode_state as ds  # reference module
    import reference_ops as ro  # reference module
    import tp_runtime as tp  # reference module

    out: dict[str, np.ndarray] = {}
    for make in cases.DECODE_CASES:
        decode_golden(ds, tp, make(), out)
    for make in cases.PREFILL_CASES:
        prefill_golden(ds, tp, make(), out)
    for make in cases.NORM_ROPE_CASES:
        norm_rope_golden(ds, tp, ro, make(), out)
    for make in cases.OPROJ_CASES:
        oproj_golden(tp, ro, make(), out)
    decode_state_golden(ds, out)
    allocator_golden(ds, out)
    np.savez_compressed(args.out, **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {len(out)} arrays ({total} bytes raw) to {args.out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
