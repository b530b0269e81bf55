"""The attention output stage across real ranks: one process per GPU (torchrun, gloo for the IPC-handle
exchange), exchange buffers mapped from the peers, partials pushed over NVLink. Every rank checks its
output against the oracle's sum and the ranks' outputs against each other: twelve decode-sized calls (at
most 64 tokens, one wave of CTAs; both exchange-buffer parities six times over, new values every call, so
a stale or half-visible partial would show) and one of 1300 tokens (more tiles than SMs, several waves).
Skipped with fewer than two GPUs.

Also runnable directly as the worker: ``torchrun --nproc-per-node N tests/test_oproj_multigpu.py``.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_output_stage_across_gpus(world) -> None:
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(29600 + world), str(Path(__file__).resolve())]
    res = subprocess.run(cmd, env=env, cwd=str(ROOT), capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]


def _worker() -> int:
    from datetime import timedelta

    import numpy as np
    import torch
    import torch.distributed as dist

    sys.path[:0] = [str(HERE), str(HERE / "golden"), str(ROOT), str(ROOT / "qwen3.6-2080ti_b200")]
    import cases
    import paged_kv_ops as ops
    import pkv_testlib as lib
    from oracle import paged_kv_oracle as oracle

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    device = f"cuda:{rank}"
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    hidden, capacity = 2048, 1300
    exchange = ops.OutputExchange(rank, world, capacity, hidden, torch.bfloat16, device)
    handles = [None] * world
    dist.all_gather_object(handles, exchange.allocate())
    exchange.attach(handles)
    dist.barrier()
    flag = ops.new_error_flag(device)
    bad = 0
    calls = 13
    for call in range(calls):
        gen = torch.Generator().manual_seed(500 + call)
        tokens = 64 - 3 * call if call < calls - 1 else capacity
        heads = torch.randn((tokens, 16, 1, 256), generator=gen).to(torch.bfloat16)
        gate = (2 * torch.randn((tokens, 1, 16 * 256), generator=gen)).to(torch.bfloat16)
        weight = (0.05 * torch.randn((hidden, 16 * 256), generator=gen)).to(torch.float8_e4m3fn)
        scale = (0.5 + torch.rand((hidden // 128, 16 * 256 // 128), generator=gen)).to(torch.bfloat16)
        case = cases.OProjCase("mgpu", heads, gate, weight, scale, torch.bfloat16, world)
        h, g, w, s = (t.contiguous().to(device) for t in case.rank_inputs(rank))
        out = ops.gated_o_proj(h, g, w, s, out_dtype=torch.bfloat16, exchange=exchange, error_flag=flag)
        torch.cuda.synchronize()
        parts = []
        for r in range(world):
            hr, hd, gr, gd, codes, sc = lib.oproj_rank_arrays(case, r)
            x, _ = oracle.gate_heads(hr, gr, hd, gd)
            parts.append(oracle.o_proj_partial(x, codes, sc, "bfloat16"))
        exp = oracle.all_reduce_sum(parts, "bfloat16")
        got = lib.as_f32(lib.np_bits(out.reshape(tokens, hidden)), "bfloat16")
        try:
            lib.assert_close(got, exp, "bfloat16", f"rank {rank} call {call}",
                             extra=lib.partial_rounding_bound(parts, "bfloat16"))
        except AssertionError as e:
            print(e, flush=True)
            bad += 1
        digests = [None] * world
        dist.all_gather_object(digests, lib.sha(lib.np_bits(out)))
        if len(set(digests)) != 1:
            print(f"rank {rank} call {call}: ranks disagree", flush=True)
            bad += 1
    if int(flag.item()) != 0:
        print(f"rank {rank}: device error bits {int(flag.item())}", flush=True)
        bad += 1
    torch.cuda.synchronize()
    dist.barrier()  # no peer still writes into this rank's buffer
    exchange.close()
    dist.destroy_process_group()
    print(f"rank {rank}: {'ok' if bad == 0 else 'FAILED'}", flush=True)
    return 0 if bad == 0 else 1


if __name__ == "__main__":
    sys.exit(_worker())
