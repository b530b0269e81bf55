"""Attention dispatch of the paged KV path: one native path, no dense fallback.

Host-side mirror of the reference's full-attention dispatch (src/tp_runtime.py:499-669, 2437-2609)
for the part this library owns: append the step's new K/V through a slot mapping, then run paged GQA
decode over the pages; optionally the fused q/k norm + RoPE + append before it and the output stage
after it (gate, FP8 o_proj, tensor-parallel all-reduce: finish_from_heads). The projections before
attention and the MoE stay with the caller. Tensor parallelism follows the reference's head split (src/tp_runtime.py:504-522,
src/tensor_parallel.py:20-25) without repeating KV heads: rank r of a TP group of size tp stores KV
heads [r*Hkv/tp, (r+1)*Hkv/tp) and serves query heads [r*Hq/tp, (r+1)*Hq/tp).

Names kept from the reference: PagedAttentionDispatchStats (src/tp_runtime.py:90-107) counts calls
and native hits; the fallback counters stay in the record (always zero) so existing readers work.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import paged_kv_ops as ops


@dataclass
class PagedAttentionDispatchStats:
    calls: int = 0
    eligible: int = 0
    dense_fallbacks: int = 0
    native_hits: int = 0
    fallback_disabled: int = 0
    fallback_no_kernel: int = 0
    fallback_prefill_or_multitoken: int = 0
    fallback_cpu: int = 0
    fallback_per_request_pools: int = 0
    fallback_shape: int = 0

    def snapshot(self) -> PagedAttentionDispatchStats:
        return PagedAttentionDispatchStats(**vars(self))

    def to_dict(self) -> dict[str, int]:
        return dict(vars(self))


def tp_head_range(num_heads: int, world_size: int, rank: int) -> tuple[int, int]:
    """[start, start + count) of the heads rank `rank` owns (TensorParallel.shard_range,
    src/tensor_parallel.py:20-25): heads must divide evenly across ranks."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} out of range for world_size {world_size}")
    if num_heads % world_size != 0:
        raise ValueError(f"size {num_heads} not divisible by world_size {world_size}")
    count = num_heads // world_size
    return rank * count, count


@dataclass(frozen=True)
class DecodeShape:
    num_layers: int
    batch: int
    num_q_heads: int  # per rank
    num_kv_heads: int  # per rank
    head_dim: int
    block_size: int
    num_pages: int
    max_blocks: int


class DecodeStepRunner:
    """Runs the paged part of one batched decode step over all full-attention layers (16-bit pools, or
    e4m3 pools with per-slot scales when key_scales / value_scales are given).

    Owns the device-resident state of the step: the per-layer K/V pools stacked as
    (num_layers, num_pages, num_kv_heads, block_size, head_dim), the int32 block tables
    (batch, max_blocks) shared by every layer, the int32 context lengths, one decode workspace
    reused by every layer (calls are stream-ordered) and the slot-mapping buffer. A step is:

      1. pkv_decode_slot_mapping_layers: the slot of each request's new token in every layer's pool
         (the pools are addressed as one stacked pool), seq_lens += 1;
      2. one pkv_kv_append of every layer's new K/V;
      3. per layer: pkv_paged_decode (attention + split merge), launched as a chain with
         programmatic dependent launch so each kernel is resident before its predecessor ends (and,
         from the second layer on, starts its page loads before it ends: PKV_DECODE_PREFETCH).

    That is 2 + 2 * num_layers kernel launches and no host synchronisation, so the step can also be
    captured in a CUDA graph.
    """

    def __init__(
        self,
        key_pools: Any,
        value_pools: Any,
        block_tables: Any,
        seq_lens: Any,
        *,
        num_q_heads: int,
        pages_per_split: int = 0,
        key_scales: Any = None,
        value_scales: Any = None,
        cuda_cores: bool = False,
    ) -> None:
        torch = _torch()
        self.cuda_cores = cuda_cores  # decode on the CUDA-core formulation (16-bit pools; for comparison)
        if key_pools.dim() != 5 or key_pools.shape != value_pools.shape:
            raise ValueError("pools must be (num_layers, num_pages, num_kv_heads, block_size, head_dim)")
        # FP8 pages: uint8 e4m3 pools plus (num_layers, num_pages, num_kv_heads, block_size) fp32 scales
        self.fp8 = key_scales is not None
        if self.fp8 and (value_scales is None or key_pools.dtype != torch.uint8
                         or key_scales.shape != key_pools.shape[:4] or value_scales.shape != key_scales.shape):
            raise ValueError("fp8 pools are uint8 with (layers, pages, kv heads, block_size) key/value scales")
        self.key_scales = key_scales
        self.value_scales = value_scales
        if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
            raise ValueError("block_tables and seq_lens must be int32")
        layers, pages, kv_heads, block_size, head_dim = key_pools.shape
        batch, max_blocks = block_tables.shape
        if num_q_heads % kv_heads != 0:
            raise ValueError("num_q_heads must be a multiple of the pool's KV heads")
        self.shape = DecodeShape(layers, batch, num_q_heads, kv_heads, head_dim, block_size, pages, max_blocks)
        self.key_pools = key_pools
        self.value_pools = value_pools
        self.block_tables = block_tables
        self.seq_lens = seq_lens
        self.pages_per_split = pages_per_split
        device = key_pools.device
        size = ops.paged_decode_workspace_size(batch, num_q_heads, kv_heads, head_dim, max_blocks, block_size,
                                               pages_per_split)
        self.workspace = ops.new_decode_workspace(size, device)
        self.slots = torch.empty((layers, batch), dtype=torch.int64, device=device)
        # every layer's pool as pages of one stacked pool (slots carry the layer offset)
        for t in (key_pools, value_pools) + ((key_scales, value_scales) if self.fp8 else ()):
            if t.stride(0) != pages * t.stride(1):
                raise ValueError("the layers' pools (and scales) must be stacked contiguously along the layer axis")
        self.key_stack = key_pools.view((layers * pages,) + tuple(key_pools.shape[2:]))
        self.value_stack = value_pools.view((layers * pages,) + tuple(value_pools.shape[2:]))
        if self.fp8:
            self.key_scale_stack = key_scales.view((layers * pages,) + tuple(key_scales.shape[2:]))
            self.value_scale_stack = value_scales.view((layers * pages,) + tuple(value_scales.shape[2:]))
        self.error_flag = ops.new_error_flag(device)
        self.stats = PagedAttentionDispatchStats()

    @property
    def launches_per_step(self) -> int:
        return 2 + 2 * self.shape.num_layers

    def _append(self, key: Any, value: Any, slots: Any) -> None:
        if self.fp8:
            ops.kv_append_fp8(key, value, slots, self.key_stack, self.value_stack, self.key_scale_stack,
                              self.value_scale_stack, error_flag=self.error_flag)
        else:
            ops.kv_append(key, value, slots, self.key_stack, self.value_stack, error_flag=self.error_flag)

    def step(self, query: Any, key: Any, value: Any, out: Any, gather: HeadGather | None = None,
             after_layer: Any = None) -> Any:
        """query/out (layers, batch, Hq, D); key/value (layers, batch, Hkv, D); all on the device.

        With a HeadGather (tensor-parallel ranks), `out` is ``gather.local_out`` and every layer's head
        outputs are exchanged right after that layer's decode, overlapping the next layer's.
        `after_layer(layer)` is called after each layer's decode is enqueued, e.g. to enqueue that
        layer's output stage (finish_from_heads with chained=True) right behind it."""
        s = self.shape
        ops.decode_slot_mapping(self.block_tables, self.seq_lens, s.num_pages, s.block_size, advance=True,
                                layers=s.num_layers, out=self.slots, error_flag=self.error_flag)
        if key.stride(0) == s.batch * key.stride(1) and value.stride(0) == s.batch * value.stride(1):
            # (layers, batch) flattens into one token axis: every layer's new K/V in one launch
            self._append(key.flatten(0, 1), value.flatten(0, 1), self.slots.view(-1))
        else:
            for layer in range(s.num_layers):
                self._append(key[layer], value[layer], self.slots[layer])
        for layer in range(s.num_layers):
            if self.fp8:
                ops.paged_decode_fp8(query[layer], self.key_pools[layer], self.value_pools[layer],
                                     self.key_scales[layer], self.value_scales[layer], self.block_tables,
                                     self.seq_lens, pages_per_split=self.pages_per_split, workspace=self.workspace,
                                     out=out[layer], error_flag=self.error_flag, chained=True, prefetch=layer > 0)
            else:
                # layers after the first: the kernel before is the previous layer's decode (or a hook's
                # output stage), which writes no pool, table or length, so the page loads start early
                ops.paged_decode(query[layer], self.key_pools[layer], self.value_pools[layer], self.block_tables,
                                 self.seq_lens, pages_per_split=self.pages_per_split, workspace=self.workspace,
                                 out=out[layer], error_flag=self.error_flag, chained=True,
                                 cuda_cores=self.cuda_cores, prefetch=layer > 0)
            if gather is not None:
                gather.launch(layer)
            if after_layer is not None:
                after_layer(layer)
            self.stats.calls += 1
            self.stats.eligible += 1
            self.stats.native_hits += 1
        if gather is not None:
            gather.join()
        return out

    def step_projected(self, query: Any, key: Any, value: Any, q_norm: Any, k_norm: Any, cos_sin: Any, eps: float,
                       out: Any) -> Any:
        """The step from the projections instead of the rotated q/k: per layer one fused launch normalises
        and rotates the query and key and appends K/V (pkv_qk_norm_rope_append), then paged decode.

        query (layers, batch, Hq, D) pre-norm, any token/head strides (e.g. the query half of q_proj);
        key/value (layers, batch, Hkv, D) pre-norm, the pool's KV heads; q_norm/k_norm (layers, D);
        cos_sin from paged_kv_ops.rope_cos_sin_table; out (layers, batch, Hq, D). Each request's new
        token sits at position = its length before the step (the reference's position_offsets,
        src/tp_runtime.py:2466). 1 + 3 * num_layers launches.
        """
        torch = _torch()
        s = self.shape
        if getattr(self, "_q_rot", None) is None or self._q_rot.dtype != query.dtype:
            self._q_rot = torch.empty((s.batch, s.num_q_heads, s.head_dim), dtype=query.dtype,
                                      device=self.key_pools.device)
        ops.decode_slot_mapping(self.block_tables, self.seq_lens, s.num_pages, s.block_size, advance=True,
                                layers=s.num_layers, out=self.slots, error_flag=self.error_flag)
        for layer in range(s.num_layers):
            # seq_lens already counts the new token: its position is seq_len - 1; the slots address the
            # stacked pools
            ops.qk_norm_rope_append(query[layer], key[layer], value[layer], q_norm[layer], k_norm[layer], cos_sin,
                                    self.seq_lens, self.slots[layer], self.key_stack, self.value_stack,
                                    eps=eps, position_offset=-1, q_out=self._q_rot, error_flag=self.error_flag)
            ops.paged_decode(self._q_rot, self.key_pools[layer], self.value_pools[layer], self.block_tables,
                             self.seq_lens, pages_per_split=self.pages_per_split, workspace=self.workspace,
                             out=out[layer], error_flag=self.error_flag)
            self.stats.calls += 1
            self.stats.eligible += 1
            self.stats.native_hits += 1
        return out

    def check_errors(self) -> int:
        """Reads (synchronously) and clears the device error word; returns the PKV_DEVERR_* bits seen."""
        bits = int(self.error_flag.item())
        if bits:
            self.error_flag.zero_()
        return bits


class DecodePipeline:
    """Host-fed decode steps with transfers overlapped: step i's query / new K/V are copied from pinned
    host memory on an upload stream while step i-1 computes, and step i's output goes back to the host
    on a download stream while step i+1 computes. Two device buffer sets alternate; events order the
    three streams without host synchronisation.

    submit(host_q, host_k, host_v, host_out) enqueues one step (host_out is filled when the returned
    event completes); finish() waits for everything enqueued. With `use_graph` the step's kernels
    are captured once per buffer set into a CUDA graph and replayed, so a step costs the host one
    replay and four copy calls; the runner must have run one step before (the library's one-time
    kernel set-up happens outside capture).

    Tensor-parallel ranks pass `gathers`, one HeadGather per buffer set: the step then exchanges every
    layer's head outputs inside the replayed graph and host_out receives the gathered
    (layers, world, batch, H_local, head_dim) buffer (HeadGather.full gives the reference's head order).
    """

    def __init__(self, runner: DecodeStepRunner, dtype: Any, *, use_graph: bool = True,
                 gathers: tuple[HeadGather, HeadGather] | None = None) -> None:
        torch = _torch()
        s = runner.shape
        device = runner.key_pools.device
        self.runner = runner
        self.compute = torch.cuda.Stream(device)
        self.copy = torch.cuda.Stream(device)  # uploads
        self.download = torch.cuda.Stream(device)
        if gathers is not None and len(gathers) != 2:
            raise ValueError("gathers: one HeadGather per buffer set (2)")
        self.bufs = []
        for i in range(2):
            gather = None if gathers is None else gathers[i]
            out = (torch.empty((s.num_layers, s.batch, s.num_q_heads, s.head_dim), dtype=dtype, device=device)
                   if gather is None else gather.local_out)
            self.bufs.append({
                "q": torch.empty((s.num_layers, s.batch, s.num_q_heads, s.head_dim), dtype=dtype, device=device),
                "k": torch.empty((s.num_layers, s.batch, s.num_kv_heads, s.head_dim), dtype=dtype, device=device),
                "v": torch.empty((s.num_layers, s.batch, s.num_kv_heads, s.head_dim), dtype=dtype, device=device),
                "out": out,
                "result": out if gather is None else gather.buffer,  # what goes back to the host
                "gather": gather,
                "inputs_free": None,  # event: compute finished reading the inputs
                "out_free": None,  # event: the output reached the host
                "graph": None,
            })
        self.i = 0
        if use_graph:
            for b in self.bufs:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.stream(self.compute):
                    with torch.cuda.graph(graph, stream=self.compute):
                        runner.step(b["q"], b["k"], b["v"], b["out"], gather=b["gather"])
                b["graph"] = graph

    @property
    def h2d_bytes(self) -> int:
        b = self.bufs[0]
        return (b["q"].numel() + b["k"].numel() + b["v"].numel()) * b["q"].element_size()

    @property
    def d2h_bytes(self) -> int:
        return self.bufs[0]["result"].numel() * self.bufs[0]["result"].element_size()

    def release(self) -> None:
        """Drops the captured graphs (a graph that holds NCCL calls must go before the process group)."""
        for b in self.bufs:
            b["graph"] = None

    def submit(self, host_q: Any, host_k: Any, host_v: Any, host_out: Any) -> Any:
        torch = _torch()
        b = self.bufs[self.i % 2]
        self.i += 1
        with torch.cuda.stream(self.copy):
            if b["inputs_free"] is not None:
                self.copy.wait_event(b["inputs_free"])
            b["q"].copy_(host_q, non_blocking=True)
            b["k"].copy_(host_k, non_blocking=True)
            b["v"].copy_(host_v, non_blocking=True)
            loaded = torch.cuda.Event()
            loaded.record(self.copy)
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(loaded)
            if b["out_free"] is not None:
                self.compute.wait_event(b["out_free"])
            if b["graph"] is not None:
                b["graph"].replay()
            else:
                self.runner.step(b["q"], b["k"], b["v"], b["out"], gather=b["gather"])
            done = torch.cuda.Event()
            done.record(self.compute)
            b["inputs_free"] = done
        with torch.cuda.stream(self.download):
            self.download.wait_event(done)
            host_out.copy_(b["result"], non_blocking=True)
            delivered = torch.cuda.Event()
            delivered.record(self.download)
            b["out_free"] = delivered
        return delivered

    def finish(self) -> None:
        self.compute.synchronize()
        self.copy.synchronize()
        self.download.synchronize()


def paged_decode_caches(query: Any, caches: Any, stats: PagedAttentionDispatchStats | None = None,
                        **kwargs: Any) -> Any:
    """Batched decode over decode_state caches: query (B, Hq, 1, D) or (B, Hq, D) -> the same shape.
    Replaces _tp_full_attention_batch_native_paged_decode and its dense fallback (src/tp_runtime.py:626-643,
    2498-2609): one native path for every dtype and shape (a shared pool, or one pool per request)."""
    from decode_state import batch_page_tables

    meta = batch_page_tables(caches)
    squeeze = query.dim() == 4
    q = query[:, :, 0, :] if squeeze else query
    out = _decode_over_page_tables(q, meta, **kwargs)
    if stats is not None:
        stats.calls += 1
        stats.eligible += 1
        stats.native_hits += 1
    return out[:, :, None, :] if squeeze else out


def _decode_over_page_tables(q: Any, meta: Any, **kwargs: Any) -> Any:
    pool = meta.key_blocks[0]
    if all(k is pool for k in meta.key_blocks):
        return ops.paged_decode(q, pool, meta.value_blocks[0], meta.block_tables, meta.sequence_lengths, **kwargs)
    # one CTA per (request, KV head) over each request's own pool: no split, so no workspace
    kept = {k: v for k, v in kwargs.items() if k in ("scale", "out", "error_flag")}
    return ops.paged_decode_request_pools(q, meta.block_tables, list(meta.key_blocks), list(meta.value_blocks),
                                          meta.sequence_lengths, **kept)


# ---- drop-ins for the reference's attention dispatch (src/tp_runtime.py:551-669, 747-767, 2498-2555) --------
# Same names, arguments and results as the reference's functions, so an unchanged caller
# (tp_full_attention / _tp_full_attention_batch) runs the native path: the cache's pages are read in
# place by the paged kernels, decode and chunked prefill alike, and nothing falls back to a dense
# gather (a CPU tensor or a missing library raises instead). `config`, `weights`, `runtime` and
# `mapping` are the caller's objects; only weights.linear, runtime.all_reduce_sum,
# runtime.profile_scope and runtime.paged_attention_stats are used, as the reference uses them.

def _scope(runtime: Any, name: str) -> Any:
    import contextlib

    scope = getattr(runtime, "profile_scope", None)
    return contextlib.nullcontext() if scope is None else scope(name)


def _record_native_paged_dispatch(runtime: Any, reason: str, *, native: bool) -> None:
    """Counts one dispatch in runtime.paged_attention_stats with the reference's counter semantics
    (src/tp_runtime.py:747-767): `reason` "no_kernel" means eligible; a native call is a hit."""
    stats = getattr(runtime, "paged_attention_stats", None)
    if stats is None:
        return
    stats.calls += 1
    if reason == "no_kernel":
        stats.eligible += 1
    if native:
        stats.native_hits += 1
        return
    stats.dense_fallbacks += 1
    counter = {"disabled": "fallback_disabled", "cpu": "fallback_cpu",
               "prefill_or_multitoken": "fallback_prefill_or_multitoken",
               "per_request_pools": "fallback_per_request_pools", "shape": "fallback_shape"}.get(reason,
                                                                                             "fallback_no_kernel")
    setattr(stats, counter, getattr(stats, counter) + 1)


def _tp_full_attention_native_paged_decode(query: Any, page_table: Any) -> Any:
    """query (1, H, 1, D) over one cache's pages (page_table from FullAttentionCache.page_metadata)
    -> (1, H, 1, D). Replaces src/tp_runtime.py:613-623; any dtype, GQA by the pool's KV heads."""
    torch = _torch()
    table = page_table.block_table
    lens = torch.full((1,), int(page_table.sequence_length), dtype=table.dtype, device=table.device)
    out = ops.paged_decode(query[:, :, 0, :], page_table.key_blocks, page_table.value_blocks, table[None], lens)
    return out[:, :, None, :]


def _tp_full_attention_native_paged_prefill(query: Any, page_table: Any, position_offset: int) -> Any:
    """query (1, H, S, D): the chunk at positions [position_offset, position_offset + S), already appended,
    attending causally over the cache's pages -> (1, H, S, D). Replaces the reference's dense prefill
    (src/tp_runtime.py:597-610 with the causal mask of :716-721)."""
    torch = _torch()
    seq = query.shape[2]
    valid = int(page_table.sequence_length)
    if position_offset + seq != valid:
        raise ValueError(f"prefill chunk at positions [{position_offset}, {position_offset + seq}) must end at "
                         f"the cache's {valid} tokens (append it before the attention)")
    table = page_table.block_table
    device = table.device
    lens = torch.full((1,), valid, dtype=table.dtype, device=device)
    cu = torch.tensor([0, seq], dtype=torch.int32).to(device, non_blocking=True)
    out = ops.paged_prefill(query[0].transpose(0, 1), cu, page_table.key_blocks, page_table.value_blocks,
                            table[None], lens, max_q_len=seq)
    return out.transpose(0, 1)[None]


def _tp_full_attention_batch_native_paged_decode(query: Any, page_tables: Any, caches: Any) -> Any:
    """query (B, H, 1, D) over the caches' pages (page_tables from batch_page_tables) -> (B, H, 1, D).
    Replaces src/tp_runtime.py:626-643: one launch over a shared pool, or over the per-request pools."""
    for cache in caches:
        if cache.key_blocks is None or cache.value_blocks is None:
            raise RuntimeError("native batched paged attention requires allocated block storage")
    return _decode_over_page_tables(query[:, :, 0, :], page_tables)[:, :, None, :]


def _tp_full_attention_finish_from_heads(heads: Any, gate: Any, hidden_states: Any, mapping: Any, config: Any,
                                         weights: Any, runtime: Any, *, scope_prefix: str) -> Any:
    """The output stage after attention with the caller's weights and runtime (src/tp_runtime.py:672-695):
    gate the heads, project with weights.linear(., mapping.o_proj), all-reduce. Callers holding the
    e4m3 o_proj shard can use finish_from_heads instead (the same math in native kernels, the all-reduce
    over NVLink inside them)."""
    torch = _torch()
    batch, seq_len, _ = hidden_states.shape
    with _scope(runtime, f"{scope_prefix}.value"):
        out = heads.transpose(1, 2).reshape(batch, seq_len, heads.shape[1] * heads.shape[3])
        out = out * torch.sigmoid(gate)
    with _scope(runtime, f"{scope_prefix}.output_proj"):
        partial = weights.linear(out, mapping.o_proj).to(hidden_states.dtype)
    with _scope(runtime, f"{scope_prefix}.all_reduce"):
        return runtime.all_reduce_sum(partial)


def _tp_full_attention_paged_or_dense(query: Any, gate: Any, hidden_states: Any, mapping: Any, config: Any,
                                      weights: Any, runtime: Any, *, cache: Any, position_offset: int) -> Any:
    """Drop-in for src/tp_runtime.py:551-610: one request's attention over its cache's pages -- decode
    (query length 1) or a prefill chunk (longer queries, causal) -- then the output stage. Always native."""
    with _scope(runtime, "full_attention.page_metadata"):
        page_table = cache.page_metadata()
    with _scope(runtime, "full_attention.native_paged"):
        if int(query.shape[2]) == 1:
            heads = _tp_full_attention_native_paged_decode(query, page_table)
        else:
            heads = _tp_full_attention_native_paged_prefill(query, page_table, position_offset)
    with _scope(runtime, "full_attention.paged_dispatch"):
        _record_native_paged_dispatch(runtime, "no_kernel", native=True)
    return _tp_full_attention_finish_from_heads(heads, gate, hidden_states, mapping, config, weights, runtime,
                                                scope_prefix="full_attention")


def _tp_full_attention_batch_paged_or_dense(query: Any, gate: Any, hidden_states: Any, mapping: Any, config: Any,
                                            weights: Any, runtime: Any, *, caches: Any, position_offsets: Any) -> Any:
    """Drop-in for src/tp_runtime.py:2498-2555: the batched decode step's attention over every row's
    cache (one query token per row, at the row's last position, as _tp_full_attention_batch appends it),
    then the output stage. Always native."""
    from decode_state import batch_page_tables

    del position_offsets  # each row's query is its cache's last token: the kernels attend to all of them
    if int(query.shape[2]) != 1:
        raise ValueError("the batched dispatch is for decode steps (one query token per row)")
    with _scope(runtime, "batch.full_attention.page_metadata"):
        page_tables = batch_page_tables(caches)
    with _scope(runtime, "batch.full_attention.native_paged"):
        heads = _tp_full_attention_batch_native_paged_decode(query, page_tables, caches)
    with _scope(runtime, "batch.full_attention.paged_dispatch"):
        _record_native_paged_dispatch(runtime, "no_kernel", native=True)
    return _tp_full_attention_finish_from_heads(heads, gate, hidden_states, mapping, config, weights, runtime,
                                                scope_prefix="batch.full_attention")


class HeadGather:
    """The per-layer head-output exchange of a tensor-parallel group, preallocated and overlapped.

    Rank r of a group of `world` ranks serves query heads [r*H_local, (r+1)*H_local). The gather buffer
    is (layers, world, batch, H_local, head_dim); rank r's decode writes its heads straight into slot
    [layer, r] (``local_out`` -- pass it as DecodeStepRunner.step's `out`), and ``launch(layer)`` gathers
    that layer in place (one NCCL all_gather_into_tensor whose input is the rank's own chunk of the output,
    so nothing is copied locally) on a side stream that waits only for that layer's decode: layer l's
    exchange overlaps layer l+1's decode. ``join()`` makes the caller's stream wait for every gather.
    Allocates nothing per call, so a step with its gathers can be captured in one CUDA graph.

    Replaces the reference's per-layer collective after attention (src/tp_runtime.py:694-695, where the
    o_proj partials are all-reduced) for an attention-only step: the exchange that the TP head split
    (src/tp_runtime.py:504-522, src/tensor_parallel.py:20-25) requires to rebuild all heads.
    """

    def __init__(self, num_layers: int, batch: int, local_heads: int, head_dim: int, dtype: Any, device: Any,
                 group: Any = None) -> None:
        torch = _torch()
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.buffer = torch.empty((num_layers, self.world, batch, local_heads, head_dim), dtype=dtype, device=device)
        self.local_out = self.buffer[:, self.rank]
        # host tensors (gloo process groups on CPU) gather synchronously, without streams
        self.on_device = self.buffer.is_cuda
        self.stream = torch.cuda.Stream(self.buffer.device) if self.on_device else None
        self.ready = [torch.cuda.Event() for _ in range(num_layers)] if self.on_device else []

    def launch(self, layer: int) -> None:
        """Starts the gather of `layer` once the current stream's work so far (its decode) is done."""
        torch = _torch()
        import torch.distributed as dist

        out, mine = self.buffer[layer].view(-1), self.buffer[layer, self.rank].view(-1)
        if not self.on_device:
            dist.all_gather_into_tensor(out, mine.clone(), group=self.group)
            return
        self.ready[layer].record(torch.cuda.current_stream())
        self.stream.wait_event(self.ready[layer])
        with torch.cuda.stream(self.stream):
            dist.all_gather_into_tensor(out, mine, group=self.group)

    def join(self) -> None:
        if self.on_device:
            _torch().cuda.current_stream().wait_stream(self.stream)

    def full(self, layer: int | None = None) -> Any:
        """(batch, world * H_local, head_dim) heads of one layer (or (layers, batch, heads, head_dim)), in
        the reference's head order; a copy (the buffer keeps the rank-major layout the collective needs)."""
        buf = self.buffer if layer is None else self.buffer[layer][None]
        layers, world, batch, heads, dim = buf.shape
        out = buf.permute(0, 2, 1, 3, 4).reshape(layers, batch, world * heads, dim)
        return out if layer is None else out[0]


def all_gather_heads(local_out: Any, group: Any = None) -> Any:
    """Gathers the per-rank query-head outputs (batch, Hq/tp, D) of a TP group into (batch, Hq, D).

    The only collective of the path: where the reference all-reduces o_proj partials after
    attention (src/tp_runtime.py:694-695), a TP=2 attention-only step exchanges head outputs into a
    local buffer with one NCCL all-gather.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    parts = [torch.empty_like(local_out) for _ in range(world)]
    dist.all_gather(parts, local_out.contiguous(), group=group)
    return torch.cat(parts, dim=1)


def create_output_exchange(capacity_tokens: int, hidden: int, out_dtype: Any, device: Any,
                           group: Any = None) -> ops.OutputExchange:
    """The exchange buffers of this rank's tensor-parallel group for finish_from_heads: every rank
    allocates its buffer, the IPC handles travel through the process group (any backend) and each rank
    maps its peers'. Collective: every rank of `group` calls it with the same arguments. Close it
    (after a barrier, so no peer still writes into it) with ``exchange.close()``."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    exchange = ops.OutputExchange(rank, world, capacity_tokens, hidden, out_dtype, device)
    handles = [None] * world
    dist.all_gather_object(handles, exchange.allocate(), group=group)
    exchange.attach(handles)
    dist.barrier(group=group)
    return exchange


def finish_from_heads(heads: Any, gate: Any, o_weight: Any, o_scale_inv: Any, hidden_dtype: Any,
                      exchange: ops.OutputExchange | None = None, *, out: Any | None = None,
                      workspace: Any | None = None, error_flag: Any | None = None, chained: bool = False) -> Any:
    """The attention layer's output stage, as _tp_full_attention_finish_from_heads
    (src/tp_runtime.py:672-695) computes it: ``all_reduce_sum((heads.transpose(1, 2).reshape(B, S,
    H*D) * sigmoid(gate)) @ dequant(o_proj)^T).to(hidden_dtype)`` with heads (B, H_local, S, D), gate
    (B, S, H_local*D) and this rank's row-parallel e4m3 o_proj shard with its bf16 block scales.

    One native call: the gate, the FP8 block-scaled projection on tensor cores, and -- with an
    exchange of a TP group -- the all-reduce over NVLink inside the same kernels (no NCCL call).
    Returns (B, S, hidden) of hidden_dtype, identical on every rank."""
    return ops.gated_o_proj(heads, gate, o_weight, o_scale_inv, out_dtype=hidden_dtype, exchange=exchange, out=out,
                            workspace=workspace, error_flag=error_flag, chained=chained)


def _torch() -> Any:
    import torch

    return torch
