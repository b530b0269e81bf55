"""Seeded synthetic inputs shared by the fixture generator and the tests.

Every case is built on the CPU from a torch.Generator with a fixed seed, so the GPU box regenerates
exactly the inputs the fixtures in this directory were computed from. Nothing here imports the
reference. Shapes follow the reference's tests and the benchmark configurations of this path:

  config1   4 requests, context {17, 64, 130, 255} + 1 appended token, block_size 16, 16 q / 2 kv
            heads, head_dim 256, fp32, seed 0; request b's block table is a seeded permutation of its
            own 64-page pool.
  decode_*  a ragged fp16 / bf16 batch (lengths 1..300, empty row included) over one shuffled pool.
  prefill   two requests appending a chunk on top of a prefix (one empty prefix), bf16.
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
