"""Reference module name for the paged attention entry points (src/fp8_cuda.py:217-250).

Callers that import ``from fp8_cuda import paged_attention_decode`` keep working unchanged; the
functions now run the sm_100a kernels of libqwen36_paged_kv.so through paged_kv_ops. The reference's
FP8 linear / MoE entry points are not part of the paged KV hot path and are not provided here.
"""

from __future__ import annotations

from paged_kv_ops import (  # noqa: F401  (re-exported API)
    kv_append,
    kv_copy_pages,
    kv_gather,
    lse_merge,
    native_stats as paged_kv_native_stats,
    paged_attention_decode,
    paged_attention_decode_batched,
    paged_decode,
    paged_prefill,
    reset_native_stats as reset_paged_kv_native_stats,
)
