"""Torch-facing wrappers of the paged KV-cache C ABI (include/qwen36_paged_kv.h).

Every function validates shapes, dtypes and devices the way the reference's pybind layer does
(src/csrc/fp8_linear_cuda.cu:1199-1240, 1276-1330), raising ``RuntimeError`` with the same
messages where the same check exists, then calls the C ABI with raw pointers and element strides on
the current CUDA stream. There is no CPU or dense fallback: a CPU tensor or a missing library is an
error. The caller owns every buffer; these wrappers only allocate outputs and the decode workspace
when the caller did not pass them.

Tensor layouts:
  pool         (num_pages, num_kv_heads, block_size, head_dim), head_dim contiguous; any strided
               view of that logical shape works (e.g. the reference's per-request pool
               ``key_blocks[0].permute(1, 0, 2, 3)``).
  block_tables (batch, max_blocks) int32 or int64, -1 padded.
  seq_lens     (batch,) same dtype as block_tables.
"""

from __future__ import annotations

import ctypes
from typing import Any, Sequence

from cuda_loader import check, load_paged_kv_library

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
INDEX_I32, INDEX_I64 = 0, 1
PREFILL_ROUND_PROBS = 1  # PKV_PREFILL_ROUND_PROBS
DECODE_CHAINED = 1  # PKV_DECODE_CHAINED
DECODE_CUDA_CORES = 2  # PKV_DECODE_CUDA_CORES
OPROJ_CHAINED = 4  # PKV_OPROJ_CHAINED
DECODE_PREFETCH = 4  # PKV_DECODE_PREFETCH
# device error bits (PKV_DEVERR_*), ORed into an error_flag word
DEVERR_PAGE_OUT_OF_RANGE, DEVERR_SLOT_OUT_OF_RANGE, DEVERR_WAIT_TIMEOUT = 1, 2, 4
DEVERR_TABLE_TOO_SHORT, DEVERR_BAD_SEQUENCE_LENGTH = 8, 16

STAT_NAMES = (
    "append_calls",
    "copy_pages_calls",
    "gather_calls",
    "decode_tensor_core_calls",
    "decode_generic_calls",
    "decode_splits_merged",
    "reference_single_decode_calls",
    "reference_batched_decode_calls",
    "prefill_calls",
    "lse_merge_calls",
    "qk_norm_rope_append_calls",
    "append_fp8_calls",
    "decode_fp8_calls",
    "gated_o_proj_calls",
)


def _torch() -> Any:
    import torch

    return torch


def dtype_code(dtype: Any) -> int:
    torch = _torch()
    codes = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}
    if dtype not in codes:
        raise RuntimeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16")
    return codes[dtype]


def index_code(dtype: Any) -> int:
    torch = _torch()
    if dtype == torch.int32:
        return INDEX_I32
    if dtype == torch.int64:
        return INDEX_I64
    raise RuntimeError(f"index tensors must be int32 or int64, got {dtype}")


def _ptr(tensor: Any | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def _stream(device: Any) -> int:
    return _torch().cuda.current_stream(device).cuda_stream


def _require_cuda(tensor: Any, name: str) -> None:
    if not getattr(tensor, "is_cuda", False):
        raise RuntimeError(f"{name} must be CUDA")


def _same_device(tensor: Any, ref: Any, name: str, ref_name: str) -> None:
    if tensor.device != ref.device:
        raise RuntimeError(f"{name} must be on same CUDA device as {ref_name}")


def _check_pool(pool: Any, name: str) -> None:
    _require_cuda(pool, name)
    if pool.dim() != 4:
        raise RuntimeError(f"{name} must have shape [num_pages, num_kv_heads, block_size, head_dim]")
    if pool.stride(3) != 1:
        raise RuntimeError(f"{name} must have a contiguous head_dim")


def native_stats() -> dict[str, int]:
    """Call counters of the native entry points (replaces fp8_native_stats, src/fp8_cuda.py:8-9)."""
    lib = load_paged_kv_library()
    n = lib.pkv_stats(None, 0)
    buf = (ctypes.c_int64 * n)()
    lib.pkv_stats(buf, n)
    return {STAT_NAMES[i] if i < len(STAT_NAMES) else f"stat_{i}": int(buf[i]) for i in range(n)}


def reset_native_stats() -> None:
    load_paged_kv_library().pkv_reset_stats()


def new_error_flag(device: Any) -> Any:
    """A zeroed int32 device word for the kernels' PKV_DEVERR_* bits."""
    torch = _torch()
    return torch.zeros(1, dtype=torch.int32, device=device)


# ---- a1: slot-mapped append ----------------------------------------------------------------------------
def kv_append(
    key: Any,
    value: Any,
    slot_mapping: Any,
    key_pool: Any,
    value_pool: Any,
    *,
    error_flag: Any | None = None,
) -> None:
    """Writes token i of key/value (T, num_kv_heads, head_dim) into slot slot_mapping[i] of the pools.

    Bit-exact replacement for FullAttentionCache.append_blocks (src/decode_state.py:271-293) applied
    to all requests of a step at once; negative slots are skipped.
    """
    torch = _torch()
    for tensor, name in ((key, "key"), (value, "value"), (slot_mapping, "slot_mapping")):
        _require_cuda(tensor, name)
    _check_pool(key_pool, "key_pool")
    _check_pool(value_pool, "value_pool")
    if key.dim() != 3 or value.shape != key.shape:
        raise RuntimeError("key/value must have shape [num_tokens, num_kv_heads, head_dim]")
    if key.stride(2) != 1 or value.stride(2) != 1:
        raise RuntimeError("key/value must have a contiguous head_dim")
    if key_pool.shape != value_pool.shape or key_pool.stride() != value_pool.stride():
        raise RuntimeError("key_pool and value_pool must have the same shape and strides")
    num_pages, heads, block_size, head_dim = key_pool.shape
    if key.shape[1] != heads or key.shape[2] != head_dim:
        raise RuntimeError("key/value heads and head_dim must match the pool")
    if key.dtype != key_pool.dtype or value.dtype != key_pool.dtype or value_pool.dtype != key_pool.dtype:
        raise RuntimeError("key/value must have the pool dtype")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or slot_mapping.shape[0] != key.shape[0]:
        raise RuntimeError("slot_mapping must be int64 of shape [num_tokens]")
    slot_mapping = slot_mapping.contiguous()
    lib = load_paged_kv_library()
    status = lib.pkv_kv_append(
        key.data_ptr(), key.stride(0), key.stride(1),
        value.data_ptr(), value.stride(0), value.stride(1),
        slot_mapping.data_ptr(), key.shape[0],
        key_pool.data_ptr(), value_pool.data_ptr(),
        num_pages, heads, block_size, head_dim,
        key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        dtype_code(key_pool.dtype), _ptr(error_flag), _stream(key.device),
    )
    check(status, "kv_append")


def kv_append_positions(
    key: Any,
    value: Any,
    block_table: Any,
    start: int,
    key_pool: Any,
    value_pool: Any,
    *,
    error_flag: Any | None = None,
) -> None:
    """Writes token i of key/value (T, num_kv_heads, head_dim) to logical position start + i of the
    request whose pages are listed in `block_table` (int64 device tensor of page ids).

    FullAttentionCache.append_blocks (src/decode_state.py:271-293) in one launch: the kernel derives
    each token's slot from the device table, so no slot list is built on the host or copied per call.
    """
    torch = _torch()
    for tensor, name in ((key, "key"), (value, "value"), (block_table, "block_table")):
        _require_cuda(tensor, name)
    _check_pool(key_pool, "key_pool")
    _check_pool(value_pool, "value_pool")
    if key.dim() != 3 or value.shape != key.shape:
        raise RuntimeError("key/value must have shape [num_tokens, num_kv_heads, head_dim]")
    if key.stride(2) != 1 or value.stride(2) != 1:
        raise RuntimeError("key/value must have a contiguous head_dim")
    if key_pool.shape != value_pool.shape or key_pool.stride() != value_pool.stride():
        raise RuntimeError("key_pool and value_pool must have the same shape and strides")
    num_pages, heads, block_size, head_dim = key_pool.shape
    if key.shape[1] != heads or key.shape[2] != head_dim:
        raise RuntimeError("key/value heads and head_dim must match the pool")
    if key.dtype != key_pool.dtype or value.dtype != key_pool.dtype or value_pool.dtype != key_pool.dtype:
        raise RuntimeError("key/value must have the pool dtype")
    if block_table.dtype != torch.int64 or block_table.dim() != 1 or not block_table.is_contiguous():
        raise RuntimeError("block_table must be a contiguous int64 vector")
    status = load_paged_kv_library().pkv_kv_append_positions(
        key.data_ptr(), key.stride(0), key.stride(1),
        value.data_ptr(), value.stride(0), value.stride(1),
        block_table.data_ptr(), block_table.shape[0], int(start), key.shape[0],
        key_pool.data_ptr(), value_pool.data_ptr(),
        num_pages, heads, block_size, head_dim,
        key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        dtype_code(key_pool.dtype), _ptr(error_flag), _stream(key.device),
    )
    check(status, "kv_append_positions")


def decode_slot_mapping(
    block_tables: Any,
    seq_lens: Any,
    num_pages: int,
    block_size: int,
    *,
    advance: bool = True,
    layers: int = 1,
    out: Any | None = None,
    error_flag: Any | None = None,
) -> Any:
    """Slots of one new token per request at position seq_lens[b] (int64, -1 for skipped rows); with
    `advance` the device seq_lens are incremented in place. Computed on the device from the persistent
    block tables, so a decode step needs no host round trip. With layers > 1 the result is
    (layers, batch): the slots in the layers' stacked pools (layer l's pages start at l * num_pages),
    for one kv_append over all layers."""
    torch = _torch()
    _require_cuda(block_tables, "block_tables")
    _require_cuda(seq_lens, "seq_lens")
    if block_tables.dtype != seq_lens.dtype or block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise RuntimeError("block_tables must be [batch, max_blocks] with contiguous rows, same dtype as seq_lens")
    if not seq_lens.is_contiguous():
        raise RuntimeError("seq_lens must be contiguous (it is updated in place)")
    batch = block_tables.shape[0]
    if out is None:
        shape = (batch,) if layers == 1 else (layers, batch)
        out = torch.empty(shape, dtype=torch.int64, device=block_tables.device)
    if not out.is_contiguous() or out.numel() != layers * batch or out.dtype != torch.int64:
        raise RuntimeError("out must be a contiguous int64 tensor of layers * batch slots")
    status = load_paged_kv_library().pkv_decode_slot_mapping_layers(
        block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1], seq_lens.data_ptr(),
        index_code(seq_lens.dtype), batch, int(block_size), int(num_pages), int(layers), out.data_ptr(),
        int(bool(advance)), _ptr(error_flag), _stream(block_tables.device),
    )
    check(status, "decode_slot_mapping")
    return out


# ---- a3: gather ---------------------------------------------------------------------------------------
def kv_gather(
    key_pool: Any,
    value_pool: Any,
    block_tables: Any,
    seq_lens: Any,
    max_len: int | None = None,
    *,
    error_flag: Any | None = None,
) -> tuple[Any, Any]:
    """Dense logical-order K/V (batch, num_kv_heads, max_len, head_dim), zero padded.

    Same values as batch_kv_tensors / as_tensors (src/decode_state.py:501-542, 295-303); a debug and
    oracle aid, never used by the attention path.
    """
    torch = _torch()
    _check_pool(key_pool, "key_pool")
    _check_pool(value_pool, "value_pool")
    _require_cuda(block_tables, "block_tables")
    _require_cuda(seq_lens, "seq_lens")
    if block_tables.dtype != seq_lens.dtype:
        raise RuntimeError("block_tables and seq_lens must have the same dtype")
    if block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise RuntimeError("block_tables must be [batch, max_blocks] with contiguous rows")
    batch = block_tables.shape[0]
    num_pages, heads, block_size, head_dim = key_pool.shape
    if max_len is None:
        max_len = int(seq_lens.max().item()) if batch else 0
    k_out = torch.empty((batch, heads, max_len, head_dim), dtype=key_pool.dtype, device=key_pool.device)
    v_out = torch.empty_like(k_out)
    lib = load_paged_kv_library()
    status = lib.pkv_gather_kv(
        key_pool.data_ptr(), value_pool.data_ptr(), num_pages, heads, block_size, head_dim,
        key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
        seq_lens.contiguous().data_ptr(), index_code(seq_lens.dtype), batch, max_len,
        k_out.data_ptr(), v_out.data_ptr(), k_out.stride(0), k_out.stride(1), k_out.stride(2),
        dtype_code(key_pool.dtype), _ptr(error_flag), _stream(key_pool.device),
    )
    check(status, "kv_gather")
    return k_out, v_out


# ---- a10: page copy -------------------------------------------------------------------------------------
def kv_copy_pages(
    key_pools: Any,
    value_pools: Any,
    src_pages: Any,
    dst_pages: Any,
    *,
    error_flag: Any | None = None,
) -> None:
    """Copies page src_pages[i] to dst_pages[i] in every layer of both pools, bit for bit.

    Pools are one layer (num_pages, heads, block_size, head_dim) or a stack of layers
    (num_layers, num_pages, heads, block_size, head_dim) whose page dimension holds whole contiguous
    pages. src and dst must be disjoint (the compaction planner guarantees it).
    """
    torch = _torch()
    _require_cuda(src_pages, "src_pages")
    _require_cuda(dst_pages, "dst_pages")
    if key_pools.shape != value_pools.shape or key_pools.stride() != value_pools.stride():
        raise RuntimeError("key and value pools must have the same shape and strides")
    pools = key_pools if key_pools.dim() == 5 else key_pools.unsqueeze(0)
    if pools.dim() != 5:
        raise RuntimeError("pools must be [pages, heads, block_size, head_dim] or with a leading layer dim")
    num_layers, num_pages = pools.shape[0], pools.shape[1]
    page_elems = pools.shape[2] * pools.shape[3] * pools.shape[4]
    if not pools[0, 0].is_contiguous():
        raise RuntimeError("kv_copy_pages needs contiguous pages (native pool layout)")
    es = pools.element_size()
    src = src_pages.to(torch.int32).contiguous()
    dst = dst_pages.to(torch.int32).contiguous()
    if src.shape != dst.shape or src.dim() != 1:
        raise RuntimeError("src_pages and dst_pages must be 1-D of equal length")
    lib = load_paged_kv_library()
    status = lib.pkv_copy_pages(
        key_pools.data_ptr(), value_pools.data_ptr(), num_layers, pools.stride(0) * es,
        num_pages, pools.stride(1) * es, 1, page_elems * es, page_elems * es,
        src.data_ptr(), dst.data_ptr(), src.shape[0], _ptr(error_flag), _stream(src.device),
    )
    check(status, "kv_copy_pages")


# ---- a4-a6: GQA paged decode -------------------------------------------------------------------------------
def paged_decode_workspace_size(
    batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int, max_blocks: int, block_size: int,
    pages_per_split: int = 0,
) -> int:
    size = load_paged_kv_library().pkv_paged_decode_workspace_size(
        batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, pages_per_split
    )
    if size < 0:
        raise RuntimeError("paged_decode_workspace_size: invalid sizes")
    return int(size)


def new_decode_workspace(size: int, device: Any) -> Any:
    """A decode workspace of `size` bytes. It must start zero-filled: the kernels keep per-(request,
    KV head) merge counters in it and leave them at zero when a call completes."""
    torch = _torch()
    return torch.zeros(size, dtype=torch.uint8, device=device)


def paged_decode(
    query: Any,
    key_pool: Any,
    value_pool: Any,
    block_tables: Any,
    seq_lens: Any,
    *,
    scale: float | None = None,
    pages_per_split: int = 0,
    workspace: Any | None = None,
    out: Any | None = None,
    error_flag: Any | None = None,
    chained: bool = False,
    cuda_cores: bool = False,
    prefetch: bool = False,
) -> Any:
    """GQA decode attention of one query token per request over its pages.

    query (batch, num_q_heads, head_dim) -> (batch, num_q_heads, head_dim) in the pool dtype; query
    head h reads KV head h // (num_q_heads // num_kv_heads). scale defaults to head_dim ** -0.5 as in
    the reference (src/tp_runtime.py:712, src/reference_ops.py:353). `chained` launches the kernels
    with programmatic dependent launch (PKV_DECODE_CHAINED): same results, less latency between
    consecutive kernels of a step. `cuda_cores` runs the CUDA-core formulation even where the
    tensor-core path applies (PKV_DECODE_CUDA_CORES), for comparing the two. `prefetch` (with
    `chained`; PKV_DECODE_PREFETCH) promises that the kernel before this call in the stream writes none of
    the pools, tables or lengths read here, so the page loads start before that kernel completes.
    """
    torch = _torch()
    _require_cuda(query, "query")
    _check_pool(key_pool, "key_pool")
    _check_pool(value_pool, "value_pool")
    _require_cuda(block_tables, "block_tables")
    _require_cuda(seq_lens, "seq_lens")
    if query.dim() != 3 or query.stride(2) != 1:
        raise RuntimeError("query must have shape [batch, num_q_heads, head_dim] with contiguous head_dim")
    if key_pool.shape != value_pool.shape or key_pool.stride() != value_pool.stride():
        raise RuntimeError("key_pool and value_pool must have the same shape and strides")
    if query.dtype != key_pool.dtype or value_pool.dtype != key_pool.dtype:
        raise RuntimeError(f"query must be {key_pool.dtype} (same dtype as key_pool/value_pool)")
    if block_tables.dtype != seq_lens.dtype:
        raise RuntimeError("block_tables and seq_lens must have the same dtype")
    if block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise RuntimeError("block_tables must be [batch, max_blocks] with contiguous rows")
    for tensor, name in ((key_pool, "key_pool"), (value_pool, "value_pool"), (block_tables, "block_tables"),
                         (seq_lens, "seq_lens")):
        _same_device(tensor, query, name, "query")
    batch, num_q_heads, head_dim = query.shape
    num_pages, num_kv_heads, block_size, pool_head_dim = key_pool.shape
    if pool_head_dim != head_dim:
        raise RuntimeError("KV head_dim must match query")
    if block_tables.shape[0] != batch or seq_lens.shape != (batch,):
        raise RuntimeError("block_tables/seq_lens batch must match query")
    max_blocks = block_tables.shape[1]
    if scale is None:
        scale = head_dim ** -0.5
    seq_lens = seq_lens.contiguous()
    size = paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size,
                                       pages_per_split)
    if workspace is None:
        workspace = new_decode_workspace(size, query.device)
    if out is None:
        out = torch.empty((batch, num_q_heads, head_dim), dtype=query.dtype, device=query.device)
    elif out.shape != query.shape or out.dtype != query.dtype or out.stride(2) != 1:
        raise RuntimeError("out must match query's shape and dtype with contiguous head_dim")
    lib = load_paged_kv_library()
    status = lib.pkv_paged_decode_ex(
        query.data_ptr(), query.stride(0), query.stride(1),
        key_pool.data_ptr(), value_pool.data_ptr(), num_pages, num_kv_heads, block_size, head_dim,
        key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        block_tables.data_ptr(), block_tables.stride(0), max_blocks, seq_lens.data_ptr(),
        index_code(seq_lens.dtype), batch, num_q_heads, float(scale), int(pages_per_split),
        workspace.data_ptr(), workspace.numel() * workspace.element_size(),
        out.data_ptr(), out.stride(0), out.stride(1),
        dtype_code(query.dtype),
        (DECODE_CHAINED if chained else 0) | (DECODE_CUDA_CORES if cuda_cores else 0)
        | (DECODE_PREFETCH if prefetch else 0),
        _ptr(error_flag), _stream(query.device),
    )
    check(status, "paged_decode")
    return out


def paged_decode_request_pools(
    query: Any,
    block_tables: Any,
    key_pools: Sequence[Any],
    value_pools: Sequence[Any],
    seq_lens: Any,
    *,
    scale: float | None = None,
    out: Any | None = None,
    error_flag: Any | None = None,
) -> Any:
    """Batched GQA decode where request b owns its private pools key_pools[b] / value_pools[b]
    (pages_b, num_kv_heads, block_size, head_dim): the per-request-pool form of the reference's
    paged_attention_decode_batched (src/csrc/fp8_linear_cuda.cu:1269-1365), without repeated heads.

    query (batch, num_q_heads, head_dim); block_tables int64 (batch, max_blocks), -1 padded; seq_lens
    int64 (batch,). The pools' addresses and page counts go to the device in one pinned copy."""
    torch = _torch()
    for tensor, name in ((query, "query"), (block_tables, "block_tables"), (seq_lens, "seq_lens")):
        _require_cuda(tensor, name)
    if query.dim() != 3 or query.stride(2) != 1:
        raise RuntimeError("query must have shape [batch, num_q_heads, head_dim] with contiguous head_dim")
    batch, num_q_heads, head_dim = query.shape
    if block_tables.dtype != torch.int64 or block_tables.dim() != 2 or block_tables.shape[0] != batch:
        raise RuntimeError("block_tables must be int64 of shape [batch, max_blocks]")
    if seq_lens.dtype != torch.int64 or seq_lens.shape != (batch,):
        raise RuntimeError("seq_lens must be int64 of shape [batch]")
    if len(key_pools) != batch or len(value_pools) != batch:
        raise RuntimeError("key_blocks list length must match batch")
    if batch == 0:
        return torch.empty_like(query) if out is None else out
    ref = key_pools[0]
    _, num_kv_heads, block_size, pool_dim = ref.shape
    meta = torch.empty((3, batch), dtype=torch.int64, pin_memory=True)
    for row, (k, v) in enumerate(zip(key_pools, value_pools)):
        _check_pool(k, "key_pool")
        _check_pool(v, "value_pool")
        _same_device(k, query, "key/value blocks", "query")
        _same_device(v, query, "key/value blocks", "query")
        if k.shape != v.shape or k.shape[1:] != ref.shape[1:] or not (k.is_contiguous() and v.is_contiguous()):
            raise RuntimeError("per-request pools must be contiguous (pages, num_kv_heads, block_size, head_dim) "
                               "with matching heads, block_size and head_dim")
        if k.dtype != query.dtype or v.dtype != query.dtype:
            raise RuntimeError(f"key/value blocks must be {_dtype_name(query.dtype)} (same dtype as query)")
        meta[0, row] = k.data_ptr()
        meta[1, row] = v.data_ptr()
        meta[2, row] = k.shape[0]
    if pool_dim != head_dim or num_q_heads % num_kv_heads:
        raise RuntimeError("KV head_dim must match query and num_q_heads must be a multiple of num_kv_heads")
    meta_dev = meta.to(query.device, non_blocking=True)
    block_tables = block_tables.contiguous()
    seq_lens = seq_lens.contiguous()
    if out is None:
        out = torch.empty_like(query)
    if scale is None:
        scale = head_dim ** -0.5
    status = load_paged_kv_library().pkv_paged_decode_request_pools(
        query.data_ptr(), query.stride(0), query.stride(1), meta_dev[0].data_ptr(), meta_dev[1].data_ptr(),
        meta_dev[2].data_ptr(), num_kv_heads, block_size, head_dim, block_tables.data_ptr(), block_tables.shape[1],
        seq_lens.data_ptr(), batch, num_q_heads, float(scale), out.data_ptr(), out.stride(0), out.stride(1),
        dtype_code(query.dtype), _ptr(error_flag), _stream(query.device),
    )
    check(status, "paged_decode_request_pools")
    return out


def lse_merge(partial_out: Any, partial_lse: Any, out_dtype: Any | None = None) -> tuple[Any, Any]:
    """Merges S normalised partial attention results (S, rows, D) with their LSEs (S, rows)."""
    torch = _torch()
    _require_cuda(partial_out, "partial_out")
    _require_cuda(partial_lse, "partial_lse")
    if partial_out.dtype != torch.float32 or partial_lse.dtype != torch.float32:
        raise RuntimeError("partial_out and partial_lse must be float32")
    parts, rows, head_dim = partial_out.shape
    if partial_lse.shape != (parts, rows):
        raise RuntimeError("partial_lse must have shape [parts, rows]")
    out_dtype = out_dtype or torch.float32
    partial_out = partial_out.contiguous()
    partial_lse = partial_lse.contiguous()
    out = torch.empty((rows, head_dim), dtype=out_dtype, device=partial_out.device)
    lse = torch.empty((rows,), dtype=torch.float32, device=partial_out.device)
    status = load_paged_kv_library().pkv_lse_merge(
        partial_out.data_ptr(), partial_lse.data_ptr(), parts, rows, head_dim, out.data_ptr(), out.stride(0),
        lse.data_ptr(), dtype_code(out_dtype), _stream(partial_out.device),
    )
    check(status, "lse_merge")
    return out, lse


# ---- a11: chunked prefill ------------------------------------------------------------------------------------
def paged_prefill(
    query: Any,
    cu_q_lens: Any,
    key_pool: Any,
    value_pool: Any,
    block_tables: Any,
    seq_lens: Any,
    *,
    max_q_len: int | None = None,
    scale: float | None = None,
    out: Any | None = None,
    error_flag: Any | None = None,
    round_probs: bool = False,
) -> Any:
    """Causal attention of each request's new chunk over its pages (prefix + the chunk itself).

    query (total_q, num_q_heads, head_dim) packed by request with int32 offsets cu_q_lens
    (batch + 1); seq_lens (batch,) are the context lengths INCLUDING the chunk, whose K/V must
    already be appended. Replaces the dense prefill fallback (src/tp_runtime.py:597-610, :716-721).
    round_probs lets the kernel round the probabilities once to the compute dtype before P.V, as the
    reference's probs.to(query.dtype) does (src/tp_runtime.py:723); by default they stay fp32-accurate.
    """
    torch = _torch()
    for tensor, name in ((query, "query"), (cu_q_lens, "cu_q_lens"), (block_tables, "block_tables"),
                         (seq_lens, "seq_lens")):
        _require_cuda(tensor, name)
    _check_pool(key_pool, "key_pool")
    _check_pool(value_pool, "value_pool")
    if query.dim() != 3 or query.stride(2) != 1:
        raise RuntimeError("query must have shape [total_q, num_q_heads, head_dim] with contiguous head_dim")
    if query.dtype != key_pool.dtype or value_pool.dtype != key_pool.dtype:
        raise RuntimeError(f"query must be {key_pool.dtype} (same dtype as key_pool/value_pool)")
    if cu_q_lens.dtype != torch.int32:
        raise RuntimeError("cu_q_lens must be int32")
    if block_tables.dtype != seq_lens.dtype or block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise RuntimeError("block_tables must be [batch, max_blocks] with contiguous rows, same dtype as seq_lens")
    total_q, num_q_heads, head_dim = query.shape
    num_pages, num_kv_heads, block_size, _ = key_pool.shape
    batch = block_tables.shape[0]
    if cu_q_lens.shape != (batch + 1,):
        raise RuntimeError("cu_q_lens must have batch + 1 entries")
    if max_q_len is None:
        max_q_len = int((cu_q_lens[1:] - cu_q_lens[:-1]).max().item()) if batch else 0
    if scale is None:
        scale = head_dim ** -0.5
    if out is None:
        out = torch.empty_like(query)
    status = load_paged_kv_library().pkv_paged_prefill_ex(
        query.data_ptr(), query.stride(0), query.stride(1), cu_q_lens.contiguous().data_ptr(), total_q, max_q_len,
        key_pool.data_ptr(), value_pool.data_ptr(), num_pages, num_kv_heads, block_size, head_dim,
        key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1], seq_lens.contiguous().data_ptr(),
        index_code(seq_lens.dtype), batch, num_q_heads, float(scale), out.data_ptr(), out.stride(0), out.stride(1),
        dtype_code(query.dtype), PREFILL_ROUND_PROBS if round_probs else 0, _ptr(error_flag), _stream(query.device),
    )
    check(status, "paged_prefill")
    return out


# ---- fused q/k RMSNorm + partial rotary embedding + K/V append -----------------------------------------------
def rope_cos_sin_table(max_position: int, head_dim: int, partial_rotary_factor: float, rope_theta: float,
                       dtype: Any, device: Any = None) -> Any:
    """(max_position, 2 * rotary_dim) rows of [cos | sin] in `dtype` for positions 0 .. max_position - 1.

    Computed on the CPU in float32 with the arithmetic of rotary_embeddings (src/reference_ops.py:203-212):
    rotary_dim = int(head_dim * partial_rotary_factor), inv_freq = 1 / theta^(2i / rotary_dim), angles
    position * inv_freq over both halves, cos/sin cast to dtype -- so the rows equal the reference's bit
    for bit. Built once per model; the fused kernel reads its rows by position.
    """
    torch = _torch()
    rotary_dim = int(head_dim * partial_rotary_factor)
    inv_freq = 1.0 / (float(rope_theta) ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim))
    freqs = torch.outer(torch.arange(max_position, dtype=torch.float32), inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    table = torch.cat((emb.cos().to(dtype), emb.sin().to(dtype)), dim=-1).contiguous()
    return table if device is None else table.to(device)


def qk_norm_rope_append(
    query: Any,
    key: Any,
    value: Any,
    q_weight: Any,
    k_weight: Any,
    cos_sin: Any,
    positions: Any,
    slot_mapping: Any,
    key_pool: Any,
    value_pool: Any,
    *,
    eps: float,
    position_offset: int = 0,
    q_out: Any | None = None,
    error_flag: Any | None = None,
) -> Any:
    """RMSNorm + rotary embedding of a step's query and key, and the K/V append, in one launch.

    query (T, Hq, D) -- e.g. the query half of q_proj viewed per head, any token/head strides --,
    key/value (T, Hkv, D) holding exactly the pool's KV heads (a TP rank passes its slice, no repeated
    heads), q_weight/k_weight (D,), cos_sin from rope_cos_sin_table, positions (T,) int32/int64 plus
    position_offset, slot_mapping (T,) int64 (negative = padding). Returns q_out (T, Hq, D): the
    normalised, rotated query for the attention kernels; the rotated key and the value land in their
    slots. Replaces src/tp_runtime.py:510-525 (and :2461-2483 for batched decode).
    """
    torch = _torch()
    for tensor, name in ((query, "query"), (key, "key"), (value, "value"), (q_weight, "q_weight"),
                         (k_weight, "k_weight"), (cos_sin, "cos_sin"), (positions, "positions"),
                         (slot_mapping, "slot_mapping")):
        _require_cuda(tensor, name)
    _check_pool(key_pool, "key_pool")
    _check_pool(value_pool, "value_pool")
    if key_pool.shape != value_pool.shape or key_pool.stride() != value_pool.stride():
        raise RuntimeError("key_pool and value_pool must have the same shape and strides")
    num_pages, kv_heads, block_size, head_dim = key_pool.shape
    if query.dim() != 3 or query.shape[2] != head_dim or query.stride(2) != 1:
        raise RuntimeError("query must have shape [num_tokens, num_q_heads, head_dim] with contiguous head_dim")
    tokens = query.shape[0]
    for tensor, name in ((key, "key"), (value, "value")):
        if tensor.shape != (tokens, kv_heads, head_dim) or tensor.stride(2) != 1:
            raise RuntimeError(f"{name} must have shape [num_tokens, pool kv heads, head_dim] with contiguous head_dim")
    dtype = key_pool.dtype
    for tensor, name in ((query, "query"), (key, "key"), (value, "value"), (q_weight, "q_weight"),
                         (k_weight, "k_weight"), (cos_sin, "cos_sin"), (value_pool, "value_pool")):
        if tensor.dtype != dtype:
            raise RuntimeError(f"{name} must be {dtype} (the pool dtype)")
    if q_weight.shape != (head_dim,) or k_weight.shape != (head_dim,):
        raise RuntimeError("q_weight/k_weight must have shape [head_dim]")
    if cos_sin.dim() != 2 or cos_sin.shape[1] % 2 != 0:
        raise RuntimeError("cos_sin must be [max_position, 2 * rotary_dim] (see rope_cos_sin_table)")
    if positions.dim() != 1 or positions.shape[0] != tokens or positions.dtype not in (torch.int32, torch.int64):
        raise RuntimeError("positions must be int32/int64 of shape [num_tokens]")
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (tokens,):
        raise RuntimeError("slot_mapping must be int64 of shape [num_tokens]")
    if q_out is None:
        q_out = torch.empty((tokens, query.shape[1], head_dim), dtype=dtype, device=query.device)
    cos_sin = cos_sin.contiguous()
    status = load_paged_kv_library().pkv_qk_norm_rope_append(
        query.data_ptr(), query.stride(0), query.stride(1),
        key.data_ptr(), key.stride(0), key.stride(1),
        value.data_ptr(), value.stride(0), value.stride(1),
        q_weight.contiguous().data_ptr(), k_weight.contiguous().data_ptr(), float(eps),
        cos_sin.data_ptr(), cos_sin.shape[0], cos_sin.shape[1] // 2,
        positions.contiguous().data_ptr(), int(position_offset), index_code(positions.dtype),
        slot_mapping.contiguous().data_ptr(),
        key_pool.data_ptr(), value_pool.data_ptr(), num_pages, kv_heads, block_size, head_dim,
        key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
        tokens, query.shape[1], dtype_code(dtype), _ptr(error_flag), _stream(query.device),
    )
    check(status, "qk_norm_rope_append")
    return q_out


# ---- FP8 (e4m3) KV pages ------------------------------------------------------------------------------------
def new_fp8_pools(num_pages: int, num_kv_heads: int, block_size: int, head_dim: int, device: Any) -> tuple:
    """Zeroed e4m3 K/V pools (uint8, (pages, kv heads, block_size, head_dim)) and their fp32 scale pools
    ((pages, kv heads, block_size)): (key_pool, value_pool, key_scales, value_scales)."""
    torch = _torch()
    shape = (num_pages, num_kv_heads, block_size, head_dim)
    return (torch.zeros(shape, dtype=torch.uint8, device=device), torch.zeros(shape, dtype=torch.uint8, device=device),
            torch.zeros(shape[:3], dtype=torch.float32, device=device),
            torch.zeros(shape[:3], dtype=torch.float32, device=device))


def _check_fp8_pools(key_pool: Any, value_pool: Any, key_scales: Any, value_scales: Any) -> None:
    torch = _torch()
    for pool, name in ((key_pool, "key_pool"), (value_pool, "value_pool")):
        _check_pool(pool, name)
        if pool.dtype != torch.uint8:
            raise RuntimeError(f"{name} must be uint8 (e4m3 codes)")
    if key_pool.shape != value_pool.shape or key_pool.stride() != value_pool.stride():
        raise RuntimeError("key_pool and value_pool must have the same shape and strides")
    for sc, name in ((key_scales, "key_scales"), (value_scales, "value_scales")):
        _require_cuda(sc, name)
        if sc.dtype != torch.float32 or sc.shape != key_pool.shape[:3] or sc.stride(2) != 1:
            raise RuntimeError(f"{name} must be float32 of shape [num_pages, num_kv_heads, block_size], slots contiguous")
    if key_scales.stride() != value_scales.stride():
        raise RuntimeError("key_scales and value_scales must have the same strides")


def kv_append_fp8(key: Any, value: Any, slot_mapping: Any, key_pool: Any, value_pool: Any, key_scales: Any,
                  value_scales: Any, *, error_flag: Any | None = None) -> None:
    """Quantising append into e4m3 pools: per (slot, KV head) row, scale = max|x| / 448 and codes =
    e4m3(x * 448 / max|x|) (round to nearest even, saturating)."""
    torch = _torch()
    for tensor, name in ((key, "key"), (value, "value"), (slot_mapping, "slot_mapping")):
        _require_cuda(tensor, name)
    _check_fp8_pools(key_pool, value_pool, key_scales, value_scales)
    num_pages, heads, block_size, head_dim = key_pool.shape
    if key.dim() != 3 or value.shape != key.shape or key.shape[1:] != (heads, head_dim):
        raise RuntimeError("key/value must have shape [num_tokens, pool kv heads, head_dim]")
    if key.stride(2) != 1 or value.stride(2) != 1 or value.dtype != key.dtype:
        raise RuntimeError("key/value must share a dtype and have a contiguous head_dim")
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (key.shape[0],):
        raise RuntimeError("slot_mapping must be int64 of shape [num_tokens]")
    status = load_paged_kv_library().pkv_kv_append_fp8(
        key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(), value.stride(0), value.stride(1),
        slot_mapping.contiguous().data_ptr(), key.shape[0], key_pool.data_ptr(), value_pool.data_ptr(),
        key_scales.data_ptr(), value_scales.data_ptr(), key_scales.stride(0), key_scales.stride(1),
        num_pages, heads, block_size, head_dim, key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        dtype_code(key.dtype), _ptr(error_flag), _stream(key.device),
    )
    check(status, "kv_append_fp8")


def paged_decode_fp8(query: Any, key_pool: Any, value_pool: Any, key_scales: Any, value_scales: Any,
                     block_tables: Any, seq_lens: Any, *, scale: float | None = None, pages_per_split: int = 0,
                     workspace: Any | None = None, out: Any | None = None, error_flag: Any | None = None,
                     chained: bool = False, prefetch: bool = False) -> Any:
    """paged_decode over e4m3 pools (see kv_append_fp8): query (B, Hq, D) fp16/bf16 -> (B, Hq, D)."""
    torch = _torch()
    _require_cuda(query, "query")
    _check_fp8_pools(key_pool, value_pool, key_scales, value_scales)
    num_pages, kv_heads, block_size, head_dim = key_pool.shape
    if query.dim() != 3 or query.shape[2] != head_dim or query.stride(2) != 1:
        raise RuntimeError("query must have shape [batch, num_q_heads, head_dim] with contiguous head_dim")
    if block_tables.dtype != seq_lens.dtype or block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise RuntimeError("block_tables must be [batch, max_blocks] with contiguous rows, same dtype as seq_lens")
    batch, num_q_heads, _ = query.shape
    if scale is None:
        scale = head_dim ** -0.5
    if workspace is None:
        size = paged_decode_workspace_size(batch, num_q_heads, kv_heads, head_dim, block_tables.shape[1], block_size,
                                           pages_per_split)
        workspace = new_decode_workspace(size, query.device)
    if out is None:
        out = torch.empty_like(query)
    status = load_paged_kv_library().pkv_paged_decode_fp8_ex(
        query.data_ptr(), query.stride(0), query.stride(1), key_pool.data_ptr(), value_pool.data_ptr(),
        key_scales.data_ptr(), value_scales.data_ptr(), key_scales.stride(0), key_scales.stride(1),
        num_pages, kv_heads, block_size, head_dim, key_pool.stride(0), key_pool.stride(1), key_pool.stride(2),
        block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1], seq_lens.contiguous().data_ptr(),
        index_code(seq_lens.dtype), batch, num_q_heads, float(scale), int(pages_per_split), workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), out.data_ptr(), out.stride(0), out.stride(1),
        dtype_code(query.dtype), (DECODE_CHAINED if chained else 0) | (DECODE_PREFETCH if prefetch else 0),
        _ptr(error_flag), _stream(query.device),
    )
    check(status, "paged_decode_fp8")
    return out


# ---- attention output stage: gate, FP8 o_proj, tensor-parallel all-reduce (src/tp_runtime.py:672-695) ----
class OutputExchange:
    """The exchange buffers of one tensor-parallel group for gated_o_proj: ``pointers[p]`` is rank p's
    buffer as mapped in this process (``pointers[rank]`` this rank's own). All ranks of a group use
    buffers of the same world, capacity (tokens per call), hidden size and output dtype, and make the
    same sequence of gated_o_proj calls with them.

    ``allocate`` makes this rank's buffer and returns its IPC handle; ``attach`` maps the peers'
    handles (one process per GPU). ``local_group`` builds every rank's view inside ONE process over
    buffers on one device (the ranks' kernels then run one after another on one stream: a test of the
    data path, not of concurrency)."""

    def __init__(self, rank: int, world: int, capacity: int, hidden: int, out_dtype: Any, device: Any) -> None:
        torch = _torch()
        self.rank, self.world, self.capacity, self.hidden = int(rank), int(world), int(capacity), int(hidden)
        self.out_dtype = out_dtype
        self.device = torch.device(device)
        self.nbytes = int(load_paged_kv_library().pkv_o_proj_comm_bytes(self.world, self.capacity, self.hidden,
                                                                         dtype_code(out_dtype)))
        if self.nbytes <= 0:
            raise RuntimeError("invalid exchange shape: world in [1, 8], capacity >= 1, hidden a multiple of 128")
        self.pointers: list[int] = [0] * self.world
        self._owned: list[int] = []
        self._opened: list[int] = []

    def allocate(self) -> bytes:
        lib = load_paged_kv_library()
        handle = ctypes.create_string_buffer(int(lib.pkv_ipc_handle_bytes()))
        ptr = ctypes.c_void_p()
        with _torch().cuda.device(self.device):
            check(lib.pkv_ipc_alloc(self.nbytes, ctypes.byref(ptr), handle), "exchange buffer")
        self.pointers[self.rank] = int(ptr.value)
        self._owned.append(int(ptr.value))
        return handle.raw

    def attach(self, handles: Sequence[bytes]) -> None:
        lib = load_paged_kv_library()
        with _torch().cuda.device(self.device):
            for p, handle in enumerate(handles):
                if p == self.rank:
                    continue
                ptr = ctypes.c_void_p()
                check(lib.pkv_ipc_open(ctypes.create_string_buffer(bytes(handle), len(handle)), ctypes.byref(ptr)),
                      "exchange buffer of a peer")
                self.pointers[p] = int(ptr.value)
                self._opened.append(int(ptr.value))

    @classmethod
    def local_group(cls, world: int, capacity: int, hidden: int, out_dtype: Any, device: Any) -> list["OutputExchange"]:
        ranks = [cls(r, world, capacity, hidden, out_dtype, device) for r in range(world)]
        for r in ranks:
            r.allocate()
        pointers = [r.pointers[r.rank] for r in ranks]
        for r in ranks:
            r.pointers = list(pointers)
        return ranks

    def close(self) -> None:
        lib = load_paged_kv_library()
        with _torch().cuda.device(self.device):
            for ptr in self._opened:
                lib.pkv_ipc_close(ptr)
            for ptr in self._owned:
                lib.pkv_ipc_free(ptr)
        self._opened, self._owned = [], []


def o_proj_workspace_size(num_tokens: int, k_local: int, hidden: int) -> int:
    return int(load_paged_kv_library().pkv_o_proj_workspace_size(int(num_tokens), int(k_local), int(hidden)))


def gated_o_proj(heads: Any, gate: Any, weight: Any, scale_inv: Any, *, out_dtype: Any | None = None,
                 exchange: OutputExchange | None = None, out: Any | None = None, workspace: Any | None = None,
                 phases: int = 3, error_flag: Any | None = None, chained: bool = False) -> Any:
    """The output stage of a full-attention layer on this rank (src/tp_runtime.py:672-695):
    ``all_reduce_sum(((heads.transpose(1, 2).reshape(B, S, H*D) * sigmoid(gate)) @ dequant(W)^T).to(out_dtype))``.

    heads (B, H, S, D) -- or (B, H, D) for one token per request -- this rank's heads; gate (B, S, H*D)
    (or (B, H*D)); weight this rank's row-parallel o_proj shard, float8_e4m3fn (or its uint8 bytes)
    (hidden, H*D); scale_inv bfloat16 (hidden / 128, H*D / 128). With an ``exchange`` of world > 1 the
    result is summed over the group's ranks. Returns (B, S, hidden) (or (B, hidden)) of out_dtype
    (default: the exchange's, else bfloat16). `chained` (PKV_OPROJ_CHAINED) makes the stage resident
    while the kernel before it (the layer's decode) drains, its weight loads starting at once."""
    torch = _torch()
    for tensor, name in ((heads, "heads"), (gate, "gate"), (weight, "weight"), (scale_inv, "scale_inv")):
        _require_cuda(tensor, name)
    squeeze = heads.dim() == 3
    if squeeze:
        heads = heads.unsqueeze(2)
        gate = gate.unsqueeze(1)
    if heads.dim() != 4 or heads.stride(3) != 1:
        raise RuntimeError("heads must have shape [batch, num_heads, seq_len, head_dim] with contiguous head_dim")
    batch, num_heads, seq_len, head_dim = heads.shape
    k = num_heads * head_dim
    if gate.dim() != 3 or tuple(gate.shape) != (batch, seq_len, k) or gate.stride(2) != 1:
        raise RuntimeError("gate must have shape [batch, seq_len, num_heads * head_dim] with a contiguous last axis")
    if weight.dtype == torch.float8_e4m3fn:
        weight = weight.view(torch.uint8)
    if weight.dtype != torch.uint8 or weight.dim() != 2 or weight.shape[1] != k or weight.stride(1) != 1:
        raise RuntimeError("weight must be float8_e4m3fn [hidden, num_heads * head_dim] with contiguous rows")
    hidden = weight.shape[0]
    if scale_inv.dtype != torch.bfloat16 or tuple(scale_inv.shape) != ((hidden + 127) // 128, (k + 127) // 128):
        raise RuntimeError("scale_inv must be bfloat16 [hidden / 128, num_heads * head_dim / 128]")
    if out_dtype is None:
        out_dtype = exchange.out_dtype if exchange is not None else torch.bfloat16
    world, rank, pointers, capacity = 1, 0, None, 0
    if exchange is not None and exchange.world > 1:
        if exchange.out_dtype != out_dtype or exchange.hidden != hidden:
            raise RuntimeError("the exchange buffers were made for another output dtype or hidden size")
        world, rank, capacity = exchange.world, exchange.rank, exchange.capacity
        pointers = (ctypes.c_void_p * world)(*exchange.pointers)
    tokens = batch * seq_len
    if workspace is None:
        workspace = torch.empty(max(o_proj_workspace_size(tokens, k, hidden), 256), dtype=torch.uint8,
                                device=heads.device)
    if out is None:
        out = torch.empty((batch, seq_len, hidden), dtype=out_dtype, device=heads.device)
    if out.dtype != out_dtype or out.numel() != tokens * hidden or out.stride(-1) != 1 or out.dim() < 2:
        raise RuntimeError("out must hold [batch * seq_len, hidden] of out_dtype with a contiguous last axis")
    o_stride = out.stride(-2)
    if out.dim() == 3 and out.shape[1] > 1 and out.stride(0) != out.shape[1] * o_stride:
        raise RuntimeError("out must space its token rows evenly")
    status = load_paged_kv_library().pkv_gated_o_proj(
        heads.data_ptr(), heads.stride(0), heads.stride(1), heads.stride(2), dtype_code(heads.dtype),
        gate.data_ptr(), gate.stride(0), gate.stride(1), dtype_code(gate.dtype), batch, seq_len, num_heads, head_dim,
        weight.data_ptr(), weight.stride(0), scale_inv.data_ptr(), scale_inv.stride(0), scale_inv.stride(1), hidden,
        out.data_ptr(), o_stride, dtype_code(out_dtype), workspace.data_ptr(), workspace.numel(), rank, world,
        pointers, capacity, int(phases) | (OPROJ_CHAINED if chained else 0), _ptr(error_flag), _stream(heads.device),
    )
    check(status, "gated_o_proj")
    return out.view(batch, hidden) if squeeze and out.dim() == 3 else out


# ---- reference-named entry points (src/fp8_cuda.py:217-250) ----------------------------------------------------
def paged_attention_decode(
    query: Any,
    block_table: Any,
    key_blocks: Any,
    value_blocks: Any,
    sequence_length: int,
    block_size: int,
) -> Any:
    """Reference-layout decode: query (B, H, 1, D), KV (B, H, P, block_size, D), 1-D int64 table.

    Same contract as the reference's paged_attention_decode (src/csrc/fp8_linear_cuda.cu:1192-1266);
    additionally accepts fp16/bf16 when query and KV share the dtype.
    """
    torch = _torch()
    for tensor, name in ((query, "query"), (block_table, "block_table"), (key_blocks, "key_blocks"),
                         (value_blocks, "value_blocks")):
        _require_cuda(tensor, name)
    if not key_blocks.is_contiguous():
        raise RuntimeError("key_blocks must be contiguous")
    if not value_blocks.is_contiguous():
        raise RuntimeError("value_blocks must be contiguous")
    if query.dtype != key_blocks.dtype or value_blocks.dtype != key_blocks.dtype:
        raise RuntimeError(f"query must be {_dtype_name(key_blocks.dtype)} (same dtype as key_blocks/value_blocks)")
    if block_table.dtype != torch.int64:
        raise RuntimeError("block_table must be int64/torch.long")
    if query.dim() != 4:
        raise RuntimeError("query must have shape [batch, heads, 1, head_dim]")
    if key_blocks.dim() != 5:
        raise RuntimeError("key_blocks must have shape [batch, heads, blocks, block_size, head_dim]")
    if value_blocks.dim() != 5:
        raise RuntimeError("value_blocks must have shape [batch, heads, blocks, block_size, head_dim]")
    if block_table.dim() != 1:
        raise RuntimeError("block_table must be rank-1")
    if query.shape[2] != 1:
        raise RuntimeError("query seq_len must be 1 for paged decode")
    batch, heads, _, head_dim = query.shape
    if key_blocks.shape[0] != batch or value_blocks.shape[0] != batch:
        raise RuntimeError("KV batch must match query")
    if key_blocks.shape[1] != heads or value_blocks.shape[1] != heads:
        raise RuntimeError("KV heads must match query")
    if key_blocks.shape[2] != value_blocks.shape[2]:
        raise RuntimeError("key/value physical block count must match")
    if key_blocks.shape[3] != block_size or value_blocks.shape[3] != block_size:
        raise RuntimeError("KV block_size mismatch")
    if key_blocks.shape[4] != head_dim or value_blocks.shape[4] != head_dim:
        raise RuntimeError("KV head_dim must match query")
    for tensor, name in ((block_table, "block_table"), (key_blocks, "key_blocks"), (value_blocks, "value_blocks")):
        _same_device(tensor, query, name, "query")
    query = query.contiguous()
    block_table = block_table.contiguous()
    out = torch.empty_like(query)
    status = load_paged_kv_library().pkv_paged_attention_decode(
        query.data_ptr(), block_table.data_ptr(), block_table.shape[0], key_blocks.data_ptr(),
        value_blocks.data_ptr(), batch, heads, key_blocks.shape[2], int(block_size), head_dim,
        int(sequence_length), out.data_ptr(), dtype_code(query.dtype), None, _stream(query.device),
    )
    check(status, "paged_attention_decode")
    return out


def paged_attention_decode_batched(
    query: Any,
    block_tables: Any,
    key_blocks: Sequence[Any],
    value_blocks: Sequence[Any],
    sequence_lengths: Any,
    block_size: int,
) -> Any:
    """Reference-layout batched decode over per-request pools (1, H, P_b, block_size, D).

    Same contract as the reference's paged_attention_decode_batched
    (src/csrc/fp8_linear_cuda.cu:1269-1365); the per-row pool pointers and page counts go to the
    device in one pinned host->device copy.
    """
    torch = _torch()
    for tensor, name in ((query, "query"), (block_tables, "block_tables"), (sequence_lengths, "sequence_lengths")):
        _require_cuda(tensor, name)
    if block_tables.dtype != torch.int64:
        raise RuntimeError("block_tables must be int64/torch.long")
    if sequence_lengths.dtype != torch.int64:
        raise RuntimeError("sequence_lengths must be int64/torch.long")
    if query.dim() != 4:
        raise RuntimeError("query must have shape [batch, heads, 1, head_dim]")
    if block_tables.dim() != 2:
        raise RuntimeError("block_tables must have shape [batch, max_blocks]")
    if sequence_lengths.dim() != 1:
        raise RuntimeError("sequence_lengths must be rank-1")
    if query.shape[2] != 1:
        raise RuntimeError("query seq_len must be 1 for paged decode")
    batch, heads, _, head_dim = query.shape
    if block_tables.shape[0] != batch:
        raise RuntimeError("block_tables batch must match query")
    if sequence_lengths.shape[0] != batch:
        raise RuntimeError("sequence_lengths batch must match query")
    if len(key_blocks) != batch:
        raise RuntimeError("key_blocks list length must match batch")
    if len(value_blocks) != batch:
        raise RuntimeError("value_blocks list length must match batch")
    meta = torch.empty((3, batch), dtype=torch.int64, pin_memory=True)
    for row, (key, value) in enumerate(zip(key_blocks, value_blocks)):
        if not (key.is_cuda and value.is_cuda):
            raise RuntimeError("key/value blocks must be CUDA")
        if key.device != query.device or value.device != query.device:
            raise RuntimeError("key/value blocks must be on same CUDA device as query")
        if not (key.is_contiguous() and value.is_contiguous()):
            raise RuntimeError("key/value blocks must be contiguous")
        if key.dtype != query.dtype or value.dtype != query.dtype:
            raise RuntimeError(f"key/value blocks must be {_dtype_name(query.dtype)} (same dtype as query)")
        if key.dim() != 5 or value.dim() != 5:
            raise RuntimeError("key/value blocks must have shape [1, heads, blocks, block_size, head_dim]")
        if key.shape[0] != 1 or value.shape[0] != 1:
            raise RuntimeError("per-request KV pools must have batch dim 1")
        if key.shape[1] != heads or value.shape[1] != heads:
            raise RuntimeError("KV heads must match query")
        if key.shape[2] != value.shape[2]:
            raise RuntimeError("key/value physical block count must match")
        if key.shape[3] != block_size or value.shape[3] != block_size:
            raise RuntimeError("KV block_size mismatch")
        if key.shape[4] != head_dim or value.shape[4] != head_dim:
            raise RuntimeError("KV head_dim must match query")
        meta[0, row] = key.data_ptr()
        meta[1, row] = value.data_ptr()
        meta[2, row] = key.shape[2]
    meta_dev = meta.to(query.device, non_blocking=True)
    query = query.contiguous()
    block_tables = block_tables.contiguous()
    sequence_lengths = sequence_lengths.contiguous()
    out = torch.empty_like(query)
    status = load_paged_kv_library().pkv_paged_attention_decode_batched(
        query.data_ptr(), block_tables.data_ptr(), block_tables.shape[1], meta_dev[0].data_ptr(),
        meta_dev[1].data_ptr(), meta_dev[2].data_ptr(), sequence_lengths.data_ptr(), batch, heads, int(block_size),
        head_dim, out.data_ptr(), dtype_code(query.dtype), None, _stream(query.device),
    )
    check(status, "paged_attention_decode_batched")
    # torch's pinned-memory allocator records the copy on the stream, so `meta` may be freed now
    return out


def _dtype_name(dtype: Any) -> str:
    return str(dtype).replace("torch.", "")
