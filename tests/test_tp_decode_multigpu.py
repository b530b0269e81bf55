"""The TP=2 KV-head split of the decode step on two real GPUs, at the benchmark's decode shape.

Both ranks hold the same 64 requests (contexts U[1024, 8192], seed 0, fp16, pages shuffled in a pool of
1.2x the tokens, 2 of the 12 layers); rank r stores only KV head r and serves query heads 8r..8r+7
(the reference's head split, src/tp_runtime.py:504-522 and src/tensor_parallel.py:20-25, without the
repeated heads). Every step appends through the device slot mapping, decodes every layer and
all-gathers each layer's head outputs in place (tp_runtime.HeadGather, NCCL) -- eagerly once, then as
replays of one CUDA graph that holds the decode launches and the gathers. On every rank the gathered
(batch, 16, 256) output of every layer must match the oracle's dense attention over BOTH KV heads
(computed on the host from the full-head pools), and the two ranks' gathered buffers must be
identical. Skipped with fewer than two GPUs.

Also runnable directly as the worker: ``torchrun --nproc-per-node 2 tests/test_tp_decode_multigpu.py``.
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
def test_tp2_decode_step_with_gathers_matches_oracle_on_two_gpus() -> None:
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29651", str(Path(__file__).resolve())]
    res = subprocess.run(cmd, env=env, cwd=str(ROOT), capture_output=True, text=True, timeout=700)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count(": ok") == 2, res.stdout[-3000:]


def _worker() -> int:
    from datetime import timedelta

    import numpy as np
    import torch
    import torch.distributed as dist

    sys.path[:0] = [str(HERE), str(HERE / "golden"), str(ROOT), str(ROOT / "qwen3.6-2080ti_b200")]
    import bench
    import pkv_testlib as lib
    from oracle import paged_kv_oracle as oracle
    from tp_runtime import DecodeStepRunner, HeadGather, tp_head_range

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    assert world == 2
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=device)
    bs, hq, hkv, d, layers = bench.BLOCK, bench.HQ, bench.HKV, bench.HEAD_DIM, 2
    q0, hq_local = tp_head_range(hq, world, rank)
    k0, hkv_local = tp_head_range(hkv, world, rank)
    lens0 = bench.make_lengths(0, 0)
    batch = len(lens0)
    steps = 3
    # the full-head state, generated identically on both ranks (host)
    gen = torch.Generator().manual_seed(2024)
    need = [(n + steps + bs - 1) // bs for n in lens0]
    num_pages = max(int(bench.POOL_FACTOR * sum(lens0) / bs) + 1, sum(need) + 1)
    perm = torch.randperm(num_pages, generator=gen)
    tables = torch.full((batch, max(need)), -1, dtype=torch.int32)
    used = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[used:used + n].to(torch.int32)
        used += n
    host_tables = [row[:n].tolist() for row, n in zip(tables, need)]
    full_k = np.stack([torch.randn((num_pages, hkv, bs, d), generator=gen).to(torch.float16).numpy()
                       for _ in range(layers)])
    full_v = np.stack([torch.randn((num_pages, hkv, bs, d), generator=gen).to(torch.float16).numpy()
                       for _ in range(layers)])
    kp = torch.from_numpy(np.ascontiguousarray(full_k[:, :, k0:k0 + hkv_local])).to(device)
    vp = torch.from_numpy(np.ascontiguousarray(full_v[:, :, k0:k0 + hkv_local])).to(device)
    runner = DecodeStepRunner(kp, vp, tables.to(device), torch.tensor(lens0, dtype=torch.int32, device=device),
                              num_q_heads=hq_local)
    gather = HeadGather(layers, batch, hq_local, d, torch.float16, device)
    q = torch.empty((layers, batch, hq_local, d), dtype=torch.float16, device=device)
    k = torch.empty((layers, batch, hkv_local, d), dtype=torch.float16, device=device)
    v = torch.empty_like(k)
    lens = list(lens0)
    bad = 0
    stream = torch.cuda.Stream(device)
    graph = None
    group = hq // hkv
    for step in range(steps):
        step_gen = torch.Generator().manual_seed(77 + step)
        fq = torch.randn((layers, batch, hq, d), generator=step_gen).to(torch.float16)
        fk = torch.randn((layers, batch, hkv, d), generator=step_gen).to(torch.float16)
        fv = torch.randn((layers, batch, hkv, d), generator=step_gen).to(torch.float16)
        q.copy_(fq[:, :, q0:q0 + hq_local])
        k.copy_(fk[:, :, k0:k0 + hkv_local])
        v.copy_(fv[:, :, k0:k0 + hkv_local])
        torch.cuda.synchronize(device)
        if step == 0:  # eager (initialises the communicator and the library outside capture)
            with torch.cuda.stream(stream):
                runner.step(q, k, v, gather.local_out, gather=gather)
            torch.cuda.synchronize(device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(graph, stream=stream):
                    runner.step(q, k, v, gather.local_out, gather=gather)
        else:
            with torch.cuda.stream(stream):
                graph.replay()
        torch.cuda.synchronize(device)
        # the host copy of the full-head pools gets this step's token at the oracle's slots
        for layer in range(layers):
            for b in range(batch):
                slots = oracle.slot_mapping(host_tables[b], lens[b], 1, bs)
                oracle.append_slots(full_k[layer], slots, fk[layer, b][None].numpy())
                oracle.append_slots(full_v[layer], slots, fv[layer, b][None].numpy())
        lens = [n + 1 for n in lens]
        if runner.seq_lens.cpu().tolist() != lens:
            print(f"rank {rank} step {step}: seq_lens did not advance", flush=True)
            bad += 1
        got_all = gather.full()  # (layers, batch, 16, d)
        for layer in range(layers):
            expected = np.zeros((batch, hq, d), dtype=np.float32)
            qf = fq[layer].float().numpy()
            for b in range(batch):
                pages = host_tables[b][:(lens[b] + bs - 1) // bs]
                for h in range(hkv):
                    expected[b, h * group:(h + 1) * group] = oracle.decode_attention(
                        qf[b:b + 1, h * group:(h + 1) * group], full_k[layer][pages][:, h:h + 1],
                        full_v[layer][pages][:, h:h + 1], [list(range(len(pages)))], [lens[b]],
                        dtype="float16", round_probs=False)[0]
            got = lib.as_f32(lib.np_bits(got_all[layer]), "float16")
            try:
                assert np.isfinite(got).all(), "non-finite output"
                lib.assert_close(got, expected, "float16", f"rank {rank} step {step} layer {layer}")
            except AssertionError as e:
                print(e, flush=True)
                bad += 1
        digests = [None] * world
        dist.all_gather_object(digests, lib.sha(lib.np_bits(gather.buffer)))
        if len(set(digests)) != 1:
            print(f"rank {rank} step {step}: the ranks' gathered buffers differ", flush=True)
            bad += 1
    errors = runner.check_errors()
    if errors:
        print(f"rank {rank}: device error bits {errors}", flush=True)
        bad += 1
    del graph  # a graph holding NCCL calls goes before the process group
    torch.cuda.synchronize(device)
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: {'ok' if bad == 0 else 'FAILED'}", flush=True)
    return 0 if bad == 0 else 1


if __name__ == "__main__":
    sys.exit(_worker())
