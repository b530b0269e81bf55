"""Loads the paged KV-cache C-ABI library (libqwen36_paged_kv.so) through ctypes.

Mirrors the reference's extension loader (src/cuda_loader.py:41-54): the library is looked up in
this package's ``lib/`` directory, and a missing build raises ``RuntimeError`` with the command that
builds it. The library is plain CUDA runtime code with no torch symbols, so unlike the reference no
torch libraries are preloaded. Every symbol declared in include/qwen36_paged_kv.h gets its argtypes
and restype set here, so a mismatch between header and binding fails at load time.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Any

PACKAGE_DIR = Path(__file__).resolve().parent
LIB_PATH = PACKAGE_DIR / "lib" / "libqwen36_paged_kv.so"
HEADER_PATH = PACKAGE_DIR.parent / "include" / "qwen36_paged_kv.h"

_LIB: ctypes.CDLL | None = None

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_int = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes); order follows include/qwen36_paged_kv.h
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "pkv_last_error": (ctypes.c_char_p, []),
    "pkv_abi_version": (_int, []),
    "pkv_stats": (_int, [ctypes.POINTER(_i64), _int]),
    "pkv_reset_stats": (None, []),
    "pkv_kv_append": (
        _int,
        [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p, _p],
    ),
    "pkv_kv_append_positions": (
        _int,
        [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
         _int, _p, _p],
    ),
    "pkv_decode_slot_mapping": (_int, [_p, _i64, _i64, _p, _int, _i64, _i64, _i64, _p, _int, _p, _p]),
    "pkv_gather_kv": (
        _int,
        [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _int, _i64, _i64, _p, _p,
         _i64, _i64, _i64, _int, _p, _p],
    ),
    "pkv_copy_pages": (_int, [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _i64, _p, _p]),
    "pkv_paged_decode_workspace_size": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "pkv_paged_decode": (
        _int,
        [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _int, _i64, _i64,
         _f32, _i64, _p, _i64, _p, _i64, _i64, _int, _p, _p],
    ),
    "pkv_paged_decode_ex": (
        _int,
        [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _int, _i64, _i64,
         _f32, _i64, _p, _i64, _p, _i64, _i64, _int, _int, _p, _p],
    ),
    "pkv_paged_decode_static_scratch": (
        _int,
        [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p, _int, _i64, _i64,
         _f32, _i64, _p, _i64, _i64, _int, _p, _p],
    ),
    "pkv_lse_merge": (_int, [_p, _p, _i64, _i64, _i64, _p, _i64, _p, _int, _p]),
    "pkv_paged_attention_decode": (
        _int,
        [_p, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _int, _p, _p],
    ),
    "pkv_paged_attention_decode_batched": (
        _int,
        [_p, _p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _int, _p, _p],
    ),
    "pkv_paged_decode_request_pools": (
        _int,
        [_p, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _i64, _i64, _f32, _p, _i64, _i64, _int, _p, _p],
    ),
    "pkv_paged_prefill": (
        _int,
        [_p, _i64, _i64, _p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p,
         _int, _i64, _i64, _f32, _p, _i64, _i64, _int, _p, _p],
    ),
    "pkv_qk_norm_rope_append": (
        _int,
        [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _f32, _p, _i64, _i64, _p, _i64, _int, _p, _p, _p,
         _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _int, _p, _p],
    ),
    "pkv_kv_append_fp8": (
        _int,
        [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
         _i64, _int, _p, _p],
    ),
    "pkv_paged_decode_fp8": (
        _int,
        [_p, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p,
         _int, _i64, _i64, _f32, _i64, _p, _i64, _p, _i64, _i64, _int, _p, _p],
    ),
    "pkv_paged_decode_fp8_ex": (
        _int,
        [_p, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p,
         _int, _i64, _i64, _f32, _i64, _p, _i64, _p, _i64, _i64, _int, _int, _p, _p],
    ),
    "pkv_decode_slot_mapping_layers": (_int, [_p, _i64, _i64, _p, _int, _i64, _i64, _i64, _i64, _p, _int, _p, _p]),
    "pkv_o_proj_workspace_size": (_i64, [_i64, _i64, _i64]),
    "pkv_o_proj_comm_bytes": (_i64, [_int, _i64, _i64, _int]),
    "pkv_gated_o_proj": (
        _int,
        [_p, _i64, _i64, _i64, _int, _p, _i64, _i64, _int, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64,
         _p, _i64, _int, _p, _i64, _int, _int, _p, _i64, _int, _p, _p],
    ),
    "pkv_ipc_handle_bytes": (_i64, []),
    "pkv_ipc_alloc": (_int, [_i64, _p, _p]),
    "pkv_ipc_open": (_int, [_p, _p]),
    "pkv_ipc_close": (_int, [_p]),
    "pkv_ipc_free": (_int, [_p]),
    "pkv_paged_prefill_ex": (
        _int,
        [_p, _i64, _i64, _p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p,
         _int, _i64, _i64, _f32, _p, _i64, _i64, _int, _int, _p, _p],
    ),
}


def library_path() -> Path:
    override = os.environ.get("QWEN36_PAGED_KV_LIB")
    return Path(override) if override else LIB_PATH


def load_paged_kv_library() -> ctypes.CDLL:
    """Returns the loaded library, raising RuntimeError when it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not path.exists():
        raise RuntimeError(
            f"qwen36 paged KV library is not built ({path}); run `python qwen3.6-2080ti_b200/build_native.py`"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def last_error() -> str:
    msg = load_paged_kv_library().pkv_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    """Maps a nonzero C-ABI status to RuntimeError carrying the library's message."""
    if status != 0:
        raise RuntimeError(f"{what}: {last_error() or f'status {status}'}")
