"""Seeded synthetic inputs shared by the fixture generator and the tests.

Every case is built on the CPU from a torch.Generator with a fixed seed, so the GPU box regenerates
exactly the inputs the fixtures in this directory were computed from. Nothing here imports the
reference. Shapes follow the reference's tests and the benchmark configurations of this path:

  config1   4 requests, context {17, 64, 130, 255} + 1 appended token, block_size 16, 16 q / 2 kv
            heads, head_dim 256, fp32, seed 0; request b's block table is a seeded permutation of its
            own 64-page pool.
  decode_*  a ragged fp16 / bf16 batch (lengths 1..300, empty row included) over one shuffled pool.
  prefill   two requests appending a chunk on top of a prefix (one empty prefix), bf16.
  norm_rope q/k RMSNorm + partial rotary embedding + append in front of attention: a bf16 prefill
            chunk, an fp16 chunk as rank 1 of a TP=2 group, and a bf16 batched decode step; the
            Qwen3.6 values head_dim 256 (128 for the TP case), partial_rotary_factor 0.25,
            rope_theta 1e7, eps 1e-6.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

BLOCK_SIZE = 16


@dataclass
class DecodeCase:
    name: str
    dtype: torch.dtype
    block_size: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    prefix_lens: list[int]  # tokens already cached before this step
    pages_per_request: int  # reference-side per-request pool size
    query: torch.Tensor  # (B, Hq, D) the step's query token
    prefix_k: list[torch.Tensor]  # per request (L_b, Hkv, D)
    prefix_v: list[torch.Tensor]
    new_k: torch.Tensor  # (B, Hkv, D) the step's appended token
    new_v: torch.Tensor
    perms: list[list[int]]  # per request: permutation of its pool's pages
    append_new: bool = True

    @property
    def batch(self) -> int:
        return len(self.prefix_lens)

    @property
    def lens(self) -> list[int]:
        extra = 1 if self.append_new else 0
        return [length + extra for length in self.prefix_lens]

    def tables(self) -> list[list[int]]:
        """Per request, the pages its context uses (logical order), in its own pool's numbering."""
        return [perm[: (length + self.block_size - 1) // self.block_size] for perm, length in zip(self.perms, self.lens)]


def _randn(gen: torch.Generator, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
    return torch.randn(shape, generator=gen, dtype=torch.float32).to(dtype)


def make_decode_case(
    name: str,
    *,
    prefix_lens: list[int],
    dtype: torch.dtype,
    head_dim: int,
    seed: int,
    num_q_heads: int = 16,
    num_kv_heads: int = 2,
    block_size: int = BLOCK_SIZE,
    pages_per_request: int = 64,
    append_new: bool = True,
) -> DecodeCase:
    gen = torch.Generator().manual_seed(seed)
    batch = len(prefix_lens)
    perms = [torch.randperm(pages_per_request, generator=gen).tolist() for _ in range(batch)]
    query = _randn(gen, (batch, num_q_heads, head_dim), dtype)
    prefix_k = [_randn(gen, (length, num_kv_heads, head_dim), dtype) for length in prefix_lens]
    prefix_v = [_randn(gen, (length, num_kv_heads, head_dim), dtype) for length in prefix_lens]
    new_k = _randn(gen, (batch, num_kv_heads, head_dim), dtype)
    new_v = _randn(gen, (batch, num_kv_heads, head_dim), dtype)
    return DecodeCase(name, dtype, block_size, num_q_heads, num_kv_heads, head_dim, list(prefix_lens),
                      pages_per_request, query, prefix_k, prefix_v, new_k, new_v, perms, append_new)


def config1() -> DecodeCase:
    return make_decode_case("config1", prefix_lens=[17, 64, 130, 255], dtype=torch.float32, head_dim=256, seed=0)


def decode_fp16() -> DecodeCase:
    return make_decode_case("decode_fp16", prefix_lens=[0, 14, 15, 16, 47, 300], dtype=torch.float16, head_dim=128,
                            seed=11)


def decode_bf16() -> DecodeCase:
    return make_decode_case("decode_bf16", prefix_lens=[5, 31, 33, 128, 260], dtype=torch.bfloat16, head_dim=256,
                            seed=12)


def decode_empty_row() -> DecodeCase:
    """A batch whose middle request holds no tokens at all (no append): the output row must be zero."""
    return make_decode_case("decode_empty_row", prefix_lens=[9, 0, 40], dtype=torch.float16, head_dim=64, seed=13,
                            append_new=False)


@dataclass
class PrefillCase:
    name: str
    dtype: torch.dtype
    block_size: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    prefix_lens: list[int]
    chunk_lens: list[int]
    pages_per_request: int
    query: list[torch.Tensor]  # per request (T_b, Hq, D)
    prefix_k: list[torch.Tensor]
    prefix_v: list[torch.Tensor]
    chunk_k: list[torch.Tensor]  # per request (T_b, Hkv, D)
    chunk_v: list[torch.Tensor]
    perms: list[list[int]] = field(default_factory=list)

    @property
    def batch(self) -> int:
        return len(self.prefix_lens)

    @property
    def lens(self) -> list[int]:
        return [p + c for p, c in zip(self.prefix_lens, self.chunk_lens)]

    def tables(self) -> list[list[int]]:
        return [perm[: (length + self.block_size - 1) // self.block_size] for perm, length in zip(self.perms, self.lens)]


def make_prefill_case(
    name: str,
    *,
    prefix_lens: list[int],
    chunk_lens: list[int],
    dtype: torch.dtype,
    head_dim: int,
    seed: int,
    num_q_heads: int = 16,
    num_kv_heads: int = 2,
    block_size: int = BLOCK_SIZE,
    pages_per_request: int = 16,
) -> PrefillCase:
    gen = torch.Generator().manual_seed(seed)
    batch = len(prefix_lens)
    perms = [torch.randperm(pages_per_request, generator=gen).tolist() for _ in range(batch)]
    query = [_randn(gen, (t, num_q_heads, head_dim), dtype) for t in chunk_lens]
    prefix_k = [_randn(gen, (p, num_kv_heads, head_dim), dtype) for p in prefix_lens]
    prefix_v = [_randn(gen, (p, num_kv_heads, head_dim), dtype) for p in prefix_lens]
    chunk_k = [_randn(gen, (t, num_kv_heads, head_dim), dtype) for t in chunk_lens]
    chunk_v = [_randn(gen, (t, num_kv_heads, head_dim), dtype) for t in chunk_lens]
    return PrefillCase(name, dtype, block_size, num_q_heads, num_kv_heads, head_dim, list(prefix_lens),
                       list(chunk_lens), pages_per_request, query, prefix_k, prefix_v, chunk_k, chunk_v, perms)


def prefill_bf16() -> PrefillCase:
    return make_prefill_case("prefill_bf16", prefix_lens=[0, 37], chunk_lens=[40, 33], dtype=torch.bfloat16,
                             head_dim=64, seed=21)


def prefill_fp16() -> PrefillCase:
    return make_prefill_case("prefill_fp16", prefix_lens=[70, 5], chunk_lens=[19, 64], dtype=torch.float16,
                             head_dim=128, seed=22)


@dataclass
class NormRopeCase:
    """Projected q/k/v of one full-attention layer call, before norm and rotary embedding.

    q_proj holds this rank's heads, each as [query (head_dim) | gate (head_dim)] like the reference's
    q_proj output; the gate half is +100 so sigmoid(gate) == 1 and the layer output is the attention
    itself. key/value hold all num_kv_heads heads (k_proj/v_proj are not sharded in the reference).
    """

    name: str
    dtype: torch.dtype
    block_size: int
    num_q_heads: int  # whole layer
    num_kv_heads: int
    head_dim: int
    world_size: int
    rank: int
    eps: float
    partial_rotary_factor: float
    rope_theta: float
    prefix_lens: list[int]  # cached tokens before the call (= position of the first new token)
    new_lens: list[int]  # tokens of the call (1 for decode)
    pages_per_request: int
    q_proj: list[torch.Tensor]  # per request (T_b, Hq_local, 2 * D)
    key: list[torch.Tensor]  # per request (T_b, Hkv, D)
    value: list[torch.Tensor]
    prefix_k: list[torch.Tensor]  # per request (L_b, Hkv, D), cache contents before the call
    prefix_v: list[torch.Tensor]
    q_norm: torch.Tensor  # (D,)
    k_norm: torch.Tensor
    perms: list[list[int]]
    batched_decode: bool

    @property
    def batch(self) -> int:
        return len(self.prefix_lens)

    @property
    def local_q_heads(self) -> int:
        return self.num_q_heads // self.world_size

    @property
    def local_kv_heads(self) -> int:
        return self.num_kv_heads // self.world_size

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def lens(self) -> list[int]:
        return [p + t for p, t in zip(self.prefix_lens, self.new_lens)]

    def tables(self) -> list[list[int]]:
        return [perm[: (length + self.block_size - 1) // self.block_size] for perm, length in zip(self.perms, self.lens)]


def make_norm_rope_case(name: str, *, prefix_lens: list[int], new_lens: list[int], dtype: torch.dtype, head_dim: int,
                        seed: int, world_size: int = 1, rank: int = 0, batched_decode: bool = False,
                        num_q_heads: int = 16, num_kv_heads: int = 2, pages_per_request: int = 80) -> NormRopeCase:
    gen = torch.Generator().manual_seed(seed)
    batch = len(prefix_lens)
    hq_local = num_q_heads // world_size
    perms = [torch.randperm(pages_per_request, generator=gen).tolist() for _ in range(batch)]
    q_proj = []
    for t in new_lens:
        q = _randn(gen, (t, hq_local, 2 * head_dim), dtype)
        q[:, :, head_dim:] = 100.0
        q_proj.append(q)
    key = [_randn(gen, (t, num_kv_heads, head_dim), dtype) for t in new_lens]
    value = [_randn(gen, (t, num_kv_heads, head_dim), dtype) for t in new_lens]
    prefix_k = [_randn(gen, (length, num_kv_heads, head_dim), dtype) for length in prefix_lens]
    prefix_v = [_randn(gen, (length, num_kv_heads, head_dim), dtype) for length in prefix_lens]
    q_norm = (0.1 * torch.randn((head_dim,), generator=gen)).to(dtype)
    k_norm = (0.1 * torch.randn((head_dim,), generator=gen)).to(dtype)
    return NormRopeCase(name, dtype, BLOCK_SIZE, num_q_heads, num_kv_heads, head_dim, world_size, rank, 1e-6, 0.25,
                        1e7, list(prefix_lens), list(new_lens), pages_per_request, q_proj, key, value, prefix_k,
                        prefix_v, q_norm, k_norm, perms, batched_decode)


def norm_rope_prefill_bf16() -> NormRopeCase:
    return make_norm_rope_case("norm_rope_prefill_bf16", prefix_lens=[45], new_lens=[37], dtype=torch.bfloat16,
                               head_dim=256, seed=31)


def norm_rope_prefill_tp2_fp16() -> NormRopeCase:
    return make_norm_rope_case("norm_rope_prefill_tp2_fp16", prefix_lens=[20], new_lens=[19], dtype=torch.float16,
                               head_dim=128, seed=32, world_size=2, rank=1)


def norm_rope_decode_bf16() -> NormRopeCase:
    return make_norm_rope_case("norm_rope_decode_bf16", prefix_lens=[0, 17, 300, 1000], new_lens=[1, 1, 1, 1],
                               dtype=torch.bfloat16, head_dim=256, seed=33, batched_decode=True)


NORM_ROPE_CASES = (norm_rope_prefill_bf16, norm_rope_prefill_tp2_fp16, norm_rope_decode_bf16)


@dataclass
class OProjCase:
    """Inputs of the attention layer's output stage (the reference's _tp_full_attention_finish_from_heads):
    head outputs (batch, num_heads, seq_len, head_dim), the output gate (batch, seq_len, num_heads *
    head_dim), an e4m3 o_proj weight (hidden, num_heads * head_dim) with bf16 128 x 128 block scales
    (scale_inv), split row-parallel over world_size ranks (rank r owns input columns
    [r K / world, (r + 1) K / world) and their scale columns)."""

    name: str
    heads: torch.Tensor
    gate: torch.Tensor
    weight: torch.Tensor  # float8_e4m3fn (hidden, K)
    scale_inv: torch.Tensor  # bfloat16 (hidden / 128, K / 128)
    hidden_dtype: torch.dtype
    world_size: int

    @property
    def num_heads(self) -> int:
        return self.heads.shape[1]

    @property
    def head_dim(self) -> int:
        return self.heads.shape[3]

    @property
    def hidden(self) -> int:
        return self.weight.shape[0]

    def rank_inputs(self, rank: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        """(heads, gate, weight, scale_inv) of one rank."""
        hl = self.num_heads // self.world_size
        kl = hl * self.head_dim
        return (self.heads[:, rank * hl : (rank + 1) * hl], self.gate[..., rank * kl : (rank + 1) * kl],
                self.weight[:, rank * kl : (rank + 1) * kl], self.scale_inv[:, rank * kl // 128 : (rank + 1) * kl // 128])


def make_oproj_case(name: str, *, batch: int, seq_len: int, num_heads: int, head_dim: int, hidden: int,
                    heads_dtype: torch.dtype, gate_dtype: torch.dtype, hidden_dtype: torch.dtype, world_size: int,
                    seed: int) -> OProjCase:
    gen = torch.Generator().manual_seed(seed)
    k = num_heads * head_dim
    heads = _randn(gen, (batch, num_heads, seq_len, head_dim), heads_dtype)
    gate = (2.0 * torch.randn((batch, seq_len, k), generator=gen)).to(gate_dtype)
    weight = (0.05 * torch.randn((hidden, k), generator=gen)).to(torch.float8_e4m3fn)
    scale_inv = (0.5 + torch.rand((hidden // 128, k // 128), generator=gen)).to(torch.bfloat16)
    return OProjCase(name, heads, gate, weight, scale_inv, hidden_dtype, world_size)


def oproj_decode_fp32_tp1() -> OProjCase:
    """The reference pipeline's own dtypes: fp32 heads and gate (its projections return fp32)."""
    return make_oproj_case("oproj_decode_fp32_tp1", batch=5, seq_len=1, num_heads=8, head_dim=64, hidden=384,
                           heads_dtype=torch.float32, gate_dtype=torch.float32, hidden_dtype=torch.bfloat16,
                           world_size=1, seed=41)


def oproj_prefill_bf16_tp2() -> OProjCase:
    return make_oproj_case("oproj_prefill_bf16_tp2", batch=1, seq_len=37, num_heads=8, head_dim=64, hidden=256,
                           heads_dtype=torch.bfloat16, gate_dtype=torch.bfloat16, hidden_dtype=torch.bfloat16,
                           world_size=2, seed=42)


def oproj_decode_fp16_tp2() -> OProjCase:
    """fp16 heads with an fp32 gate: torch promotes the gated product to fp32."""
    return make_oproj_case("oproj_decode_fp16_tp2", batch=6, seq_len=1, num_heads=4, head_dim=128, hidden=256,
                           heads_dtype=torch.float16, gate_dtype=torch.float32, hidden_dtype=torch.float16,
                           world_size=2, seed=43)


OPROJ_CASES = (oproj_decode_fp32_tp1, oproj_prefill_bf16_tp2, oproj_decode_fp16_tp2)

DECODE_CASES = (config1, decode_fp16, decode_bf16, decode_empty_row)
PREFILL_CASES = (prefill_bf16, prefill_fp16)


def allocator_script() -> list[tuple[str, int | list[int]]]:
    """A fixed allocate/release sequence for the free-list check (ids are released out of order)."""
    return [
        ("init", 12),
        ("allocate", 3),
        ("allocate", 4),
        ("release", [4, 2, 6]),
        ("allocate", 2),
        ("allocate", 3),
        ("release", [0, 1, 3]),
        ("allocate", 5),
    ]


def to_bits(t: torch.Tensor):
    """numpy view of a tensor: float32/float16 as such, bfloat16 as uint16 bit patterns."""
    import numpy as np

    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def dtype_name(dtype: torch.dtype) -> str:
    return {torch.float32: "float32", torch.float16: "float16", torch.bfloat16: "bfloat16"}[dtype]
