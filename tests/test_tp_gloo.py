"""Multi-rank host paths on CPU with gloo, world size 2 (mirrors the reference's spawn-based TP tests,
tests/unit/test_tp_runtime.py:591-620 in the reference project).

* TP=2 head split: rank r keeps KV head r and computes query heads 8r..8r+7; one all-gather of the head
  outputs rebuilds the full attention output.
* request sharding: ranks take balanced request shards and exchange nothing on the data path.
* failure: a rank that dies before the collective makes the other rank's collective fail within the
  process-group timeout instead of hanging.
"""

from __future__ import annotations

import os
import sys
import tempfile
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _setup_paths() -> None:
    for p in (ROOT / "qwen3.6-2080ti_b200", ROOT, ROOT / "tests", ROOT / "tests" / "golden"):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))


def _init(rank: int, world: int, init_file: str, timeout_s: float = 30.0) -> None:
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _tp_worker(rank: int, world: int, init_file: str, out_dir: str) -> None:
    _setup_paths()
    import cases
    import pkv_testlib as lib
    from oracle import paged_kv_oracle as oracle
    from tp_runtime import all_gather_heads, tp_head_range

    _init(rank, world, init_file)
    case = cases.decode_fp16()
    pk, pv, tables = lib.native_pools(case)
    kv0, kv_count = tp_head_range(case.num_kv_heads, world, rank)
    q0, q_count = tp_head_range(case.num_q_heads, world, rank)
    q = lib.as_f32(lib.np_bits(case.query), "float16")
    local = oracle.decode_attention(q[:, q0 : q0 + q_count], pk[:, kv0 : kv0 + kv_count],
                                    pv[:, kv0 : kv0 + kv_count], tables, case.lens, dtype="float16")
    full = all_gather_heads(torch.from_numpy(local))
    if rank == 0:
        expected = oracle.decode_attention(q, pk, pv, tables, case.lens, dtype="float16")
        np.save(os.path.join(out_dir, "tp.npy"), np.stack([full.numpy(), expected]))
    dist.barrier()
    dist.destroy_process_group()


def _shard_worker(rank: int, world: int, init_file: str, out_dir: str) -> None:
    _setup_paths()
    import cases
    import pkv_testlib as lib
    from oracle import paged_kv_oracle as oracle
    from scheduler import shard_requests

    _init(rank, world, init_file)
    case = cases.decode_bf16()
    pk, pv, tables = lib.native_pools(case)
    mine = shard_requests(case.lens, world)[rank]
    q = lib.as_f32(lib.np_bits(case.query), "bfloat16")
    rows = oracle.decode_attention(q[mine], pk, pv, [tables[i] for i in mine], [case.lens[i] for i in mine],
                                   dtype="bfloat16")
    gathered: list = [None] * world
    dist.all_gather_object(gathered, (mine, rows))  # result collection only, not part of the data path
    if rank == 0:
        full = np.zeros((case.batch, case.num_q_heads, case.head_dim), dtype=np.float32)
        for idx, part in gathered:
            full[idx] = part
        expected = oracle.decode_attention(q, pk, pv, tables, case.lens, dtype="bfloat16")
        np.save(os.path.join(out_dir, "shard.npy"), np.stack([full, expected]))
    dist.destroy_process_group()


def _failing_worker(rank: int, world: int, init_file: str, out_dir: str) -> None:
    _setup_paths()
    _init(rank, world, init_file, timeout_s=4.0)
    if rank == 1:
        raise RuntimeError("injected failure before the collective")
    try:
        from tp_runtime import all_gather_heads

        all_gather_heads(torch.zeros((2, 4, 8)))
        Path(out_dir, "no_error").write_text("collective returned")
    except Exception as exc:  # noqa: BLE001 - the point is that it surfaces
        Path(out_dir, "error").write_text(type(exc).__name__)


def _spawn(fn, tmp: str) -> None:
    init_file = os.path.join(tmp, "init")
    mp.spawn(fn, args=(2, init_file, tmp), nprocs=2, join=True)


def test_tp2_head_split_with_head_output_all_gather_equals_full_decode() -> None:
    with tempfile.TemporaryDirectory() as tmp:
        _spawn(_tp_worker, tmp)
        got, expected = np.load(os.path.join(tmp, "tp.npy"))
    np.testing.assert_array_equal(got, expected)


def test_request_sharding_over_two_ranks_covers_the_batch() -> None:
    with tempfile.TemporaryDirectory() as tmp:
        _spawn(_shard_worker, tmp)
        got, expected = np.load(os.path.join(tmp, "shard.npy"))
    np.testing.assert_array_equal(got, expected)


def test_a_rank_failing_before_the_collective_surfaces_as_an_error() -> None:
    with tempfile.TemporaryDirectory() as tmp:
        ctx = mp.spawn(_failing_worker, args=(2, os.path.join(tmp, "init"), tmp), nprocs=2, join=False)
        survivor, failing = ctx.processes
        survivor.join(timeout=60)  # waited for on its own, so it is never terminated early
        failing.join(timeout=60)
        assert survivor.exitcode is not None, "the surviving rank hung"
        assert failing.exitcode != 0
        assert Path(tmp, "error").exists(), "the surviving rank's collective did not fail"
        assert not Path(tmp, "no_error").exists()


def _gather_worker(rank: int, world: int, init_file: str, out_dir: str) -> None:
    _setup_paths()
    from tp_runtime import HeadGather

    _init(rank, world, init_file)
    layers, batch, local_heads, dim = 3, 5, 4, 8
    gather = HeadGather(layers, batch, local_heads, dim, torch.float32, "cpu")
    # what rank r's decode would write: a value naming (layer, request, global head, column)
    for layer in range(layers):
        for h in range(local_heads):
            head = rank * local_heads + h
            gather.local_out[layer, :, h] = (1000 * layer + 100 * torch.arange(batch)[:, None] + 10 * head
                                             + torch.arange(dim)[None, :] / 10).float()
        gather.launch(layer)
    gather.join()
    if rank == 0:
        np.save(os.path.join(out_dir, "gather.npy"), gather.full().numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_head_gather_rebuilds_the_reference_head_order() -> None:
    """HeadGather's in-place per-layer gather and full() give (layers, batch, heads, dim) with rank r's
    heads at [r*H_local, (r+1)*H_local), the order the reference's TP head split uses."""
    world = 2
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_gather_worker, args=(world, os.path.join(tmp, "init"), tmp), nprocs=world, join=True)
        full = np.load(os.path.join(tmp, "gather.npy"))
    layers, batch, heads, dim = full.shape
    assert (layers, batch, heads, dim) == (3, 5, 8, 8)
    want = (1000 * np.arange(layers)[:, None, None, None] + 100 * np.arange(batch)[None, :, None, None]
            + 10 * np.arange(heads)[None, None, :, None] + np.arange(dim)[None, None, None, :] / 10)
    np.testing.assert_array_equal(full, want.astype(np.float32))
