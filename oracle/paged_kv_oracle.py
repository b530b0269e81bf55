"""CPU oracle of the paged KV-cache hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference runtime's algorithm for this path, used as the checker by
tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg. Nothing in the product path
imports it. Every function names the reference code it restates (paths are relative to the
reference project root).

Pinning: tests/test_oracle_golden.py checks every function here against fixtures that
tests/golden/make_golden.py produced by running the reference's own Python code
(src/decode_state.py, src/tp_runtime.py, src/reference_ops.py) on the same seeded inputs.

Dtypes: float32 and float16 are numpy dtypes; bfloat16 values travel as uint16 bit patterns and
are widened with bf16_to_f32 / narrowed with f32_to_bf16 (round to nearest even), so the oracle can
emulate the reference's ``probs.to(query.dtype)`` rounding for every dtype.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np

# ---- dtype helpers --------------------------------------------------------------------------------------


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, np.uint16(0x7FC0), out)
    return out


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Rounds float32 values to `dtype` ("float32", "float16", "bfloat16") and returns float32."""
    if dtype == "float32":
        return x.astype(np.float32)
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_to_f32(f32_to_bf16(x))
    raise ValueError(dtype)


def to_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    return bf16_to_f32(x) if dtype == "bfloat16" else x.astype(np.float32)


# ---- a1: append ---------------------------------------------------------------------------------------------


def slot_mapping(block_table: Sequence[int], start: int, count: int, block_size: int) -> np.ndarray:
    """Slots written when `count` tokens are appended at logical positions [start, start+count).

    The same physical_block / block_offset walk as FullAttentionCache.append_blocks
    (src/decode_state.py:278-284): slot = block_table[pos // block_size] * block_size + pos % block_size.
    """
    pos = np.arange(start, start + count, dtype=np.int64)
    table = np.asarray(block_table, dtype=np.int64)
    return table[pos // block_size] * block_size + pos % block_size


def append_slots(pool: np.ndarray, slots: np.ndarray, rows: np.ndarray) -> None:
    """pool (P, H, bs, D), rows (T, H, D): pool[slot // bs, :, slot % bs] = rows[i] for slot >= 0.

    The slice assignment of src/decode_state.py:285-290, one token at a time; a bit-exact copy.
    """
    block_size = pool.shape[2]
    for i, slot in enumerate(np.asarray(slots, dtype=np.int64)):
        if slot < 0:
            continue
        pool[slot // block_size, :, slot % block_size] = rows[i]


def append_blocks_reference_layout(
    pool: np.ndarray, block_table: Sequence[int], valid: int, new: np.ndarray
) -> int:
    """Reference-layout append (src/decode_state.py:271-293).

    pool (B, H, P, bs, D) and new (B, H, T, D): walks the logical positions valid..valid+T-1 block span
    by block span exactly like append_blocks and returns the new valid length.
    """
    block_size = pool.shape[3]
    seq = new.shape[2]
    src = 0
    pos = valid
    while src < seq:
        logical = pos // block_size
        off = pos % block_size
        take = min(seq - src, block_size - off)
        phys = block_table[logical]
        pool[:, :, phys, off : off + take] = new[:, :, src : src + take]
        src += take
        pos += take
    return valid + seq


# ---- a2/a3: tables and gather -------------------------------------------------------------------------------


def padded_block_tables(tables: Sequence[Sequence[int]]) -> np.ndarray:
    """-1 padded (B, max_blocks) int64, as batch_page_tables builds it (src/decode_state.py:570-590)."""
    max_blocks = max((len(t) for t in tables), default=0)
    out = np.full((len(tables), max_blocks), -1, dtype=np.int64)
    for i, table in enumerate(tables):
        out[i, : len(table)] = table
    return out


def gather_blocks(pool: np.ndarray, block_table: Sequence[int], valid: int) -> np.ndarray:
    """pool (P, H, bs, D) -> logical-order (H, valid, D).

    _gather_blocks (src/decode_state.py:395-404): index_select of the table's pages, flatten the
    (block, slot) axes, keep the first `valid` tokens.
    """
    table = np.asarray(block_table, dtype=np.int64)
    pages = pool[table]  # (n, H, bs, D)
    n, heads, bs, dim = pages.shape
    flat = pages.transpose(1, 0, 2, 3).reshape(heads, n * bs, dim)
    return flat[:, :valid]


def batch_kv(pool: np.ndarray, tables: Sequence[Sequence[int]], lens: Sequence[int]) -> tuple[np.ndarray, np.ndarray]:
    """Zero-padded (B, H, max_len, D) and the valid mask (B, max_len): batch_kv_tensors
    (src/decode_state.py:501-542) over one shared pool."""
    max_len = max(lens)
    heads, dim = pool.shape[1], pool.shape[3]
    out = np.zeros((len(lens), heads, max_len, dim), dtype=pool.dtype)
    mask = np.zeros((len(lens), max_len), dtype=bool)
    for i, (table, length) in enumerate(zip(tables, lens)):
        if length > 0:
            out[i, :, :length] = gather_blocks(pool, table, length)
            mask[i, :length] = True
    return out, mask


# ---- a4-a8: dense attention ----------------------------------------------------------------------------------


def repeat_kv(kv: np.ndarray, repeats: int) -> np.ndarray:
    """(B, Hkv, L, D) -> (B, Hkv*repeats, L, D), KV head i serving query heads i*repeats.. (i+1)*repeats-1
    (src/reference_ops.py:414-419, src/tp_runtime.py:2736-2741)."""
    return np.repeat(kv, repeats, axis=1)


def dense_attention(
    query: np.ndarray,
    key: np.ndarray,
    value: np.ndarray,
    *,
    dtype: str,
    query_positions: np.ndarray,
    valid_mask: np.ndarray | None = None,
    scale: float | None = None,
    round_probs: bool = True,
) -> np.ndarray:
    """Masked dense attention with the reference's rounding points, returned as float32.

    query (B, Hq, Tq, D); key/value (B, Hkv, L, D), all float32 holding `dtype` values. Query head h
    reads KV head h // (Hq // Hkv). Restates src/tp_runtime.py:2586-2605 (and reference_ops.py:353-359):
      scores = (q . k^T) * D**-0.5 in fp32; masked where key_pos > query_pos or the key is padding;
      probs = softmax(scores) in fp32, then rounded to `dtype` (``.to(query.dtype)``);
      out = probs @ v, rounded to `dtype`.
    query_positions is (B, Tq) absolute positions of the query tokens. round_probs=False skips the
    rounding of the probabilities (the "exact" mode: fp32 softmax and fp32 P.V, as the sm_100a kernels
    compute it); the output is rounded to `dtype` in both modes.
    """
    batch, hq, tq, dim = query.shape
    hkv = key.shape[1]
    group = hq // hkv
    if scale is None:
        scale = dim ** -0.5
    k = repeat_kv(key, group).astype(np.float32)
    v = repeat_kv(value, group).astype(np.float32)
    scores = np.matmul(query.astype(np.float32), k.transpose(0, 1, 3, 2)) * np.float32(scale)
    key_pos = np.arange(k.shape[2])
    mask = key_pos[None, None, :] > query_positions[:, :, None]  # (B, Tq, L)
    if valid_mask is not None:
        mask = mask | ~valid_mask[:, None, :]
    scores = np.where(mask[:, None, :, :], np.float32(np.finfo(np.float32).min), scores)
    scores = scores - scores.max(axis=-1, keepdims=True)
    e = np.exp(scores, dtype=np.float32)
    probs = e / e.sum(axis=-1, keepdims=True)
    if round_probs:
        probs = round_to(probs, dtype)
    out = np.matmul(probs, v)
    return round_to(out, dtype)


# relative rounding error bound (unit roundoff) of each dtype
UNIT_ROUNDOFF = {"float32": 2.0 ** -24, "float16": 2.0 ** -11, "bfloat16": 2.0 ** -8}


def prob_rounding_bound(
    query: np.ndarray,
    key: np.ndarray,
    value: np.ndarray,
    *,
    dtype: str,
    query_positions: np.ndarray,
    valid_mask: np.ndarray | None = None,
    scale: float | None = None,
) -> np.ndarray:
    """Bound on how far the reference's ``probs.to(query.dtype)`` (src/tp_runtime.py:2601) can move an
    attention output: each probability is rounded with relative error <= u, so the output moves by at
    most u * sum_j p_j |v_j|. Same arguments as dense_attention; returns that bound, float32."""
    batch, hq, tq, dim = query.shape
    group = hq // key.shape[1]
    if scale is None:
        scale = dim ** -0.5
    k = repeat_kv(key, group).astype(np.float32)
    v = repeat_kv(value, group).astype(np.float32)
    scores = np.matmul(query.astype(np.float32), k.transpose(0, 1, 3, 2)) * np.float32(scale)
    mask = np.arange(k.shape[2])[None, None, :] > query_positions[:, :, None]
    if valid_mask is not None:
        mask = mask | ~valid_mask[:, None, :]
    scores = np.where(mask[:, None, :, :], -np.inf, scores)
    scores = scores - scores.max(axis=-1, keepdims=True)
    e = np.exp(scores)
    probs = e / e.sum(axis=-1, keepdims=True)
    return (UNIT_ROUNDOFF[dtype] * np.matmul(probs, np.abs(v))).astype(np.float32)


def decode_attention(
    query: np.ndarray,
    pool_k: np.ndarray,
    pool_v: np.ndarray,
    tables: Sequence[Sequence[int]],
    lens: Sequence[int],
    *,
    dtype: str,
    scale: float | None = None,
    round_probs: bool = True,
) -> np.ndarray:
    """Batched paged decode: query (B, Hq, D) at position lens[b]-1 over each request's pages.

    The dense composition the reference runs for a batched decode step: batch_kv_tensors
    (src/decode_state.py:501-542) then the masked dense math (src/tp_runtime.py:2574-2605).
    Rows with length 0 give zeros (the reference's batched kernel, src/csrc/fp8_linear_cuda.cu:987-991).
    """
    batch = query.shape[0]
    out = np.zeros(query.shape, dtype=np.float32)
    live = [i for i in range(batch) if lens[i] > 0]
    if not live:
        return out
    keys, mask = batch_kv(pool_k, [tables[i] for i in live], [lens[i] for i in live])
    values, _ = batch_kv(pool_v, [tables[i] for i in live], [lens[i] for i in live])
    q = query[live][:, :, None, :]
    positions = np.asarray([[lens[i] - 1] for i in live], dtype=np.int64)
    res = dense_attention(q, to_f32(keys, dtype), to_f32(values, dtype), dtype=dtype, query_positions=positions,
                          valid_mask=mask, scale=scale, round_probs=round_probs)
    out[live] = res[:, :, 0, :]
    return out


def decode_rounding_bound(
    query: np.ndarray,
    pool_k: np.ndarray,
    pool_v: np.ndarray,
    tables: Sequence[Sequence[int]],
    lens: Sequence[int],
    *,
    dtype: str,
    scale: float | None = None,
) -> np.ndarray:
    """prob_rounding_bound for the batched decode composition of decode_attention."""
    out = np.zeros(query.shape, dtype=np.float32)
    live = [i for i in range(query.shape[0]) if lens[i] > 0]
    if not live:
        return out
    keys, mask = batch_kv(pool_k, [tables[i] for i in live], [lens[i] for i in live])
    values, _ = batch_kv(pool_v, [tables[i] for i in live], [lens[i] for i in live])
    positions = np.asarray([[lens[i] - 1] for i in live], dtype=np.int64)
    res = prob_rounding_bound(query[live][:, :, None, :], to_f32(keys, dtype), to_f32(values, dtype), dtype=dtype,
                              query_positions=positions, valid_mask=mask, scale=scale)
    out[live] = res[:, :, 0, :]
    return out


def prefill_attention(
    query: np.ndarray,
    pool_k: np.ndarray,
    pool_v: np.ndarray,
    table: Sequence[int],
    total_len: int,
    *,
    dtype: str,
    scale: float | None = None,
    round_probs: bool = True,
) -> np.ndarray:
    """Causal attention of a chunk of Tq query tokens at positions [total_len - Tq, total_len).

    Restates the prefill path: cache.as_tensors() (src/decode_state.py:295-303) then the dense causal
    math with position_offset = prefix length (src/tp_runtime.py:698-726). query (Hq, Tq, D) float32.
    """
    tq = query.shape[1]
    keys = to_f32(gather_blocks(pool_k, table, total_len), dtype)[None]
    values = to_f32(gather_blocks(pool_v, table, total_len), dtype)[None]
    positions = np.arange(total_len - tq, total_len, dtype=np.int64)[None]
    return dense_attention(query[None], keys, values, dtype=dtype, query_positions=positions, scale=scale,
                           round_probs=round_probs)[0]


def prefill_rounding_bound(
    query: np.ndarray, pool_k: np.ndarray, pool_v: np.ndarray, table: Sequence[int], total_len: int, *, dtype: str,
    scale: float | None = None,
) -> np.ndarray:
    """prob_rounding_bound for the causal chunk composition of prefill_attention."""
    tq = query.shape[1]
    keys = to_f32(gather_blocks(pool_k, table, total_len), dtype)[None]
    values = to_f32(gather_blocks(pool_v, table, total_len), dtype)[None]
    positions = np.arange(total_len - tq, total_len, dtype=np.int64)[None]
    return prob_rounding_bound(query[None], keys, values, dtype=dtype, query_positions=positions, scale=scale)[0]


# ---- a6: split-KV merge -----------------------------------------------------------------------------------------


def lse_merge(partial_out: np.ndarray, partial_lse: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Log-sum-exp merge of S partial results (S, R, D) with natural-log LSEs (S, R).

    No reference counterpart (the reference has no split-KV); this is the published flash-decoding
    combine: M = max_s lse_s, w_s = exp(lse_s - M), out = sum_s w_s out_s / sum_s w_s.
    """
    m = partial_lse.max(axis=0)
    base = np.where(np.isneginf(m), 0.0, m)
    w = np.exp(partial_lse - base[None])
    tot = w.sum(axis=0)
    out = (w[:, :, None] * partial_out).sum(axis=0) / np.where(tot > 0, tot, 1.0)[:, None]
    lse = np.where(tot > 0, base + np.log(np.where(tot > 0, tot, 1.0)), -np.inf)
    return out.astype(np.float32), lse.astype(np.float32)


def split_decode_partials(
    query: np.ndarray, keys: np.ndarray, values: np.ndarray, bounds: Sequence[tuple[int, int]], scale: float
) -> tuple[np.ndarray, np.ndarray]:
    """Per-split normalised outputs and LSEs of one query row over token ranges of one request.

    query (D,), keys/values (L, D) float32. Used to check that a split-KV decode equals whole-context
    attention (the merge has no reference counterpart).
    """
    outs, lses = [], []
    for lo, hi in bounds:
        s = (keys[lo:hi] @ query) * scale
        m = s.max()
        e = np.exp(s - m)
        outs.append((e @ values[lo:hi]) / e.sum())
        lses.append(m + np.log(e.sum()))
    return np.asarray(outs, dtype=np.float32), np.asarray(lses, dtype=np.float32)


# ---- a10: page copy ---------------------------------------------------------------------------------------------


def copy_pages(pool: np.ndarray, src: Sequence[int], dst: Sequence[int]) -> None:
    """pool (..., P, ...) with pages on axis 0: pool[dst_i] = pool[src_i] for every pair, in order.

    The page-move semantics of the pool growth copy grown[:, :, :old] = old (src/decode_state.py:66-67)
    applied to an explicit (src, dst) list; with disjoint src/dst the order does not matter.
    """
    for s, d in zip(src, dst):
        pool[d] = pool[s]


# ---- allocator ------------------------------------------------------------------------------------------------


@dataclass
class FreeList:
    """Sorted free list: allocate() takes the lowest ids, release() returns ids and re-sorts.

    PagedKVBlockPool.allocate / release (src/decode_state.py:72-84) without the growth step.
    """

    free: list[int]

    def allocate(self, count: int) -> list[int]:
        if count > len(self.free):
            raise MemoryError(f"need {count} pages, {len(self.free)} free")
        out = self.free[:count]
        del self.free[:count]
        return out

    def release(self, pages: Sequence[int]) -> None:
        self.free.extend(pages)
        self.free.sort()


# ---- f1: q/k RMSNorm + partial rotary embedding (in front of the append) ----------------------------------------


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float, *, dtype: str) -> np.ndarray:
    """rms_norm (src/reference_ops.py:166-169) over the last axis: x * (1 / sqrt(mean(x^2) + eps)) *
    (1 + weight) in float32, rounded to dtype. x and weight are float32 arrays holding dtype values.
    numpy sums the squares in its own order, so a result can differ from torch's by one unit in the
    last place of dtype."""
    x = np.asarray(x, dtype=np.float32)
    mean = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(mean + np.float32(eps))
    return round_to((x * inv) * (np.float32(1.0) + np.asarray(weight, dtype=np.float32)), dtype)


def rope_cos_sin(positions: np.ndarray, head_dim: int, partial_rotary_factor: float, rope_theta: float, *,
                 dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """rotary_embeddings (src/reference_ops.py:203-212): rotary_dim = int(head_dim * factor), inverse
    frequencies 1 / theta^(2i / rotary_dim), angles position * inv_freq duplicated over both halves,
    cos/sin in float32 rounded to dtype. numpy's pow/cos differ from torch's in the last float32 bit, so
    this table matches the reference's only to a rounding (the kernels take the table as an input)."""
    rotary_dim = int(head_dim * partial_rotary_factor)
    inv_freq = np.float32(1.0) / (np.float32(rope_theta) ** (np.arange(0, rotary_dim, 2, dtype=np.float32)
                                                              / np.float32(rotary_dim)))
    freqs = np.asarray(positions, dtype=np.float32).reshape(-1, 1) * inv_freq.reshape(1, -1)
    emb = np.concatenate([freqs, freqs], axis=-1).astype(np.float32)
    return round_to(np.cos(emb), dtype), round_to(np.sin(emb), dtype)


def apply_rotary(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, *, dtype: str) -> np.ndarray:
    """apply_rotary_pos_emb for one tensor (src/reference_ops.py:215-224, _rotate_half :422-427) with the
    reference's dtype arithmetic: the first rotary_dim = cos.shape[-1] elements become
    rnd(rnd(x * cos) + rnd(rotate_half(x) * sin)), rnd rounding to dtype (torch evaluates each dtype
    op in float32 and rounds); the rest pass through. x (..., D); cos/sin broadcast against x[..., :rd]."""
    x = np.asarray(x, dtype=np.float32)
    rd = cos.shape[-1]
    half = rd // 2
    xr = x[..., :rd]
    rotated = np.concatenate([-xr[..., half:], xr[..., :half]], axis=-1)
    out = x.copy()
    out[..., :rd] = round_to(round_to(xr * cos, dtype) + round_to(rotated * sin, dtype), dtype)
    return out


def qk_norm_rope(query: np.ndarray, key: np.ndarray, q_weight: np.ndarray, k_weight: np.ndarray, eps: float,
                 cos: np.ndarray, sin: np.ndarray, *, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """The norm + rotary composition of tp_full_attention (src/tp_runtime.py:510-517): query (T, Hq, D),
    key (T, Hkv, D), cos/sin (T, rotary_dim) -> the rotated, normalised query and key (float32 arrays
    holding dtype values). The value is appended unchanged."""
    q = apply_rotary(rms_norm(query, q_weight, eps, dtype=dtype), cos[:, None, :], sin[:, None, :], dtype=dtype)
    k = apply_rotary(rms_norm(key, k_weight, eps, dtype=dtype), cos[:, None, :], sin[:, None, :], dtype=dtype)
    return q, k


# ---- f4: FP8 (e4m3) pages with per-(slot, KV head) scales ------------------------------------------------------


def e4m3_values() -> np.ndarray:
    """float32 value of every e4m3 ("fn": no infinities) code 0..255: sign, 4 exponent bits (bias 7),
    3 mantissa bits, subnormals at exponent 0, 0x7f / 0xff NaN. The same decoding as the reference's
    e4m3 table (src/csrc/fp8_linear_cuda.cu:64-97)."""
    codes = np.arange(256)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    mag = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1.0 + man / 8.0) * 2.0 ** (exp - 7.0))
    val = np.where(codes & 0x80, -mag, mag)
    val[(codes & 0x7F) == 0x7F] = np.nan
    return val.astype(np.float32)


def round_to_e4m3(x: np.ndarray) -> np.ndarray:
    """e4m3 codes of float32 values: round to nearest, ties to an even code, saturating at +-448; NaN
    gives 0x7f."""
    x = np.asarray(x, dtype=np.float32)
    mags = e4m3_values()[:127]  # codes 0x00 .. 0x7e, increasing
    ax = np.abs(x)
    hi = np.clip(np.searchsorted(mags, ax), 1, 126)
    lo = hi - 1
    d_lo, d_hi = ax - mags[lo], mags[hi] - ax
    code = np.where((d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0)), hi, lo)
    code = np.where(ax >= mags[126], 126, code)
    code = np.where(np.signbit(x), code | 0x80, code)
    return np.where(np.isnan(x), 0x7F, code).astype(np.uint8)


def quantize_fp8_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per row (last axis): amax = max |x|, scale = amax / 448, codes = e4m3(x * (448 / amax)), all in
    float32; rows of zeros get scale 0 and codes 0. Returns (codes uint8, scales float32)."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(x), axis=-1)
    with np.errstate(divide="ignore"):
        inv = np.where(amax > 0, np.float32(448.0) / amax, np.float32(0.0)).astype(np.float32)
    scale = (amax / np.float32(448.0)).astype(np.float32)
    return round_to_e4m3(x * inv[..., None]), scale


def dequantize_fp8(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Row values code_value * scale (float32); scales has one entry per row of codes."""
    return (e4m3_values()[codes] * np.asarray(scales, dtype=np.float32)[..., None]).astype(np.float32)


# ---- attention output stage: gate, FP8 block-scaled o_proj, all-reduce -----------------------------------


def promote(a: str, b: str) -> str:
    """torch's result dtype of a binary op on two floating tensors (float32 > float16/bfloat16; float16
    with bfloat16 gives float32)."""
    if a == b:
        return a
    return "float32"


def gate_heads(heads: np.ndarray, gate: np.ndarray, heads_dtype: str, gate_dtype: str) -> tuple[np.ndarray, str]:
    """``out = heads * torch.sigmoid(gate)`` (src/tp_runtime.py:690-691) with torch's rounding points:
    sigmoid is computed in float32 and rounded to the gate's dtype, the product is computed in float32
    and rounded to the promoted dtype. heads (M, K) and gate (M, K) are float32 arrays holding values
    of their dtypes; returns (float32 values, the product's dtype)."""
    sig = round_to((1.0 / (1.0 + np.exp(-gate.astype(np.float64)))).astype(np.float32), gate_dtype)
    dtype = promote(heads_dtype, gate_dtype)
    return round_to(heads.astype(np.float32) * sig, dtype), dtype


def dequantize_fp8_weight(codes: np.ndarray, scale_inv_bits: np.ndarray, block: int = 128) -> np.ndarray:
    """dequantize_fp8_weight (src/reference_ops.py:500-506): float(e4m3 code) times the bf16 scale of
    its 128 x 128 block, in float32 (every such product is exact in float32)."""
    values = e4m3_values()[codes.astype(np.int64)]
    scale = bf16_to_f32(scale_inv_bits)
    expanded = np.repeat(np.repeat(scale, block, axis=0), block, axis=1)[: codes.shape[0], : codes.shape[1]]
    return values * expanded


def o_proj_partial(x: np.ndarray, codes: np.ndarray, scale_inv_bits: np.ndarray, out_dtype: str) -> np.ndarray:
    """One rank's ``weights.linear(out, o_proj).to(hidden_states.dtype)`` (src/tp_runtime.py:693; the
    linear is reference_ops.linear's dequantise + float32 F.linear, src/reference_ops.py:496-497):
    x (M, K_local) float32, codes (N, K_local) e4m3, scales (N/128, K_local/128) bf16 bits. The float32
    product is accumulated in float64 and rounded once (the reference's float32 GEMM order is not
    pinned; the difference is far below the output rounding)."""
    w = dequantize_fp8_weight(codes, scale_inv_bits).astype(np.float64)
    return round_to((x.astype(np.float64) @ w.T).astype(np.float32), out_dtype)


def all_reduce_sum(partials: Sequence[np.ndarray], dtype: str) -> np.ndarray:
    """``runtime.all_reduce_sum`` (src/tp_runtime.py:288-298, NCCL SUM in the partials' dtype): the
    rank partials summed in rank order in float32 and rounded once to `dtype` -- for two ranks exactly
    what a SUM of two tensors of that dtype gives."""
    total = np.zeros_like(partials[0], dtype=np.float32)
    for p in partials:
        total = total + p.astype(np.float32)
    return round_to(total, dtype)
