#!/usr/bin/env python3
"""Paged-decode benchmark: KV HBM GB/s and decode tok/s over the 12 full-attention layers.

Workload (the path's headline decode configuration, per GPU): one decode step of batch 64, contexts uniform in
[1024, 8192] (seeded per rank), block_size 16, 16 query / 2 KV heads, head_dim 256, fp16, pages
shuffled in a pool of 1.2x the tokens, 12 full-attention layers (the 36 linear-attention layers hold
no pages and are not part of this path). A step appends one token per request to every layer through
a device slot mapping and runs paged GQA decode attention in every layer; contexts grow by one token
per step. Data are synthetic N(0, 1).

  value  algorithmic bytes of the timed steps / device time, summed over ranks (weak scaling: every
         rank runs the full batch on its own GPU); the step is captured once in a CUDA graph and
         replayed; pools (8.7 GB) exceed L2 (126 MB), so no flush is needed between steps.
  e2e    the same bytes over the device time of steps that go through the public API
         (tp_runtime.DecodePipeline.submit) with the step's query and new K/V copied from pinned host
         memory and the attention output copied back every step; transfers run on a copy stream and
         overlap the neighbouring steps' kernels.
  roofline  paged decode (attention + split merge) per launch: algorithmic bytes / CUDA-event
         duration on the launching stream, against MEASURED_PEAKS.json's HBM copy bandwidth.

Algorithmic bytes per layer and step (unique K+V read once, int32 table, Q and O, and the append's
read + write of the new K/V): sum_b 2*Hkv*D*s*L_b + 4*ceil(L_b/16) + 2*B*Hq*D*s + 4*B*Hkv*D*s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen3.6-2080ti_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "paged-decode KV HBM GB/s (% of peak) and decode tok/s, batch 64, 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
NUM_LAYERS, BATCH, HQ, HKV, HEAD_DIM, BLOCK = 12, 64, 16, 2, 256, 16
RL_STEPS = 5  # spare token capacity reserved for the per-launch measurements
RL_REPLAYS = 20  # replays of the graph of the step's decode launches (per-launch roofline)
MIN_LEN, MAX_LEN, POOL_FACTOR = 1024, 8192, 1.2
DTYPE_BYTES = 2


def parse_args(argv: list[str] | None = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="decode workload on one GPU: skip the brief secondary measurements of the other workloads")
    p.add_argument("--workload", choices=("decode", "long", "prefill", "churn", "churn_tp", "normrope", "decode_fp8",
                                          "oproj", "decode_tp", "attn_layer"),
                   default="decode",
                   help="decode: the headline configuration (default); long: batch 8 x 131072-token contexts "
                        "(bf16, split-KV); prefill: 8 x 2048-token chunks on U[0,4096] prefixes (bf16, causal); "
                        "churn: 256 lognormal contexts, 10%% replaced per step, page compaction (churn_tp: the same "
                        "on N GPUs as N/2 TP=2 pairs x request shards); normrope: fused "
                        "q/k RMSNorm + rotary + K/V append of 8 x 2048 chunk tokens (bf16); decode_fp8: the "
                        "decode configuration over e4m3 pages with per-slot scales; oproj: the attention output "
                        "stage (gate, FP8 o_proj, tensor-parallel all-reduce over the N GPUs) of 12 layers at "
                        "batch 64; decode_tp: the decode configuration on N GPUs composed as N/2 TP=2 pairs "
                        "(KV head split + head-output all-gather) x request shards; attn_layer: the decode "
                        "configuration with each layer's output stage (gate + FP8 o_proj) chained behind its decode")
    p.add_argument("--tokens", type=int, default=None,
                   help="oproj only: tokens per layer call (default 64, the decode batch; e.g. 8192 for a "
                        "prefill-sized call, whose roofline is then the bf16 tensor peak)")
    p.add_argument("--decode-kernel", choices=("tensor", "cuda"), default="tensor",
                   help="decode workload: 'cuda' runs the CUDA-core formulation of paged decode "
                        "(PKV_DECODE_CUDA_CORES) instead of the mma.sync one, for comparing the two")
    p.add_argument("--pages-per-split", type=int, default=0,
                   help="decode / decode_tp: about this many pages per warp of the decode (fewer warps, fewer "
                        "pieces to merge); 0 = every resident warp shares the work (default)")
    p.add_argument("--layers", type=int, default=NUM_LAYERS,
                   help="full-attention layers per step (12 for the benchmark; 1 gives the same per-layer "
                        "launches on a 0.7 GB pool for profiling)")
    return p.parse_args(argv)


# ---- output ----------------------------------------------------------------------------------------------
_COLLECT: list | None = None  # set while the headline run measures the other workloads as secondary figures


def emit(line: dict) -> None:
    """Prints a workload's JSON line (or hands it to the collecting headline run)."""
    if _COLLECT is not None:
        _COLLECT.append(line)
        return
    print(json.dumps(line), flush=True)


# ---- workload --------------------------------------------------------------------------------------------
def make_lengths(seed: int, rank: int) -> list[int]:
    import torch

    gen = torch.Generator().manual_seed(1000 * seed + rank)
    return torch.randint(MIN_LEN, MAX_LEN + 1, (BATCH,), generator=gen).tolist()


def layer_bytes(lens: list[int], hq: int = HQ, hkv: int = HKV) -> int:
    """Decode + append bytes of one layer and step (one new token per request)."""
    return decode_bytes(lens, hq, hkv) + 4 * len(lens) * hkv * HEAD_DIM * DTYPE_BYTES


def decode_bytes(lens: list[int], hq: int = HQ, hkv: int = HKV) -> int:
    """Bytes of one paged-decode launch (attention only, no append)."""
    kv = sum(2 * hkv * HEAD_DIM * DTYPE_BYTES * n for n in lens)
    table = sum(4 * ((n + BLOCK - 1) // BLOCK) for n in lens)
    return kv + table + 2 * len(lens) * hq * HEAD_DIM * DTYPE_BYTES


def build_state(lens: list[int], extra_tokens: int, seed: int, rank: int, device, layers: int, dtype=None,
                hq: int = HQ, hkv: int = HKV):
    """Pools, shuffled block tables with room for `extra_tokens` more tokens per request, and
    per-layer step inputs, all resident on `device` (hq/hkv: this rank's query / KV heads)."""
    import torch

    dtype = dtype or torch.float16
    batch = len(lens)
    gen = torch.Generator().manual_seed(1000 * seed + rank + 7)
    need = [(n + extra_tokens + BLOCK - 1) // BLOCK for n in lens]
    num_pages = max(int(POOL_FACTOR * sum(lens) / BLOCK) + 1, sum(need) + 1)
    perm = torch.randperm(num_pages, generator=gen)
    max_blocks = max(need)
    tables = torch.full((batch, max_blocks), -1, dtype=torch.int32)
    used = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[used : used + n].to(torch.int32)
        used += n
    shape = (layers, num_pages, hkv, BLOCK, HEAD_DIM)
    torch.manual_seed(1000 * seed + rank + 11)
    key_pools = torch.randn(shape, dtype=dtype, device=device)
    value_pools = torch.randn(shape, dtype=dtype, device=device)
    query = torch.randn((layers, batch, hq, HEAD_DIM), dtype=dtype, device=device)
    key = torch.randn((layers, batch, hkv, HEAD_DIM), dtype=dtype, device=device)
    value = torch.randn((layers, batch, hkv, HEAD_DIM), dtype=dtype, device=device)
    out = torch.empty_like(query)
    return {
        "key_pools": key_pools,
        "value_pools": value_pools,
        "tables": tables.to(device),
        "lens0": torch.tensor(lens, dtype=torch.int32),
        "num_pages": num_pages,
        "query": query,
        "key": key,
        "value": value,
        "out": out,
    }


# ---- clocks ----------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons (every 20 ms) while the measured work runs.

    `mark(name)` opens a named window at the current host time and closes the previous one; summary()
    reports the samples that fall inside the windows (the GPU is under load there), per window and
    together, so the record describes the timed replays rather than the idle time around them."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.proc = None
        self.out = ""
        self.windows: list[list] = []

    def __enter__(self) -> ClockSampler:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.3)
        return self

    def mark(self, name: str | None) -> None:
        """Ends the open window (if any) now and, with a name, opens the next one."""
        now = time.time()
        if self.windows and self.windows[-1][2] is None:
            self.windows[-1][2] = now
        if name is not None:
            self.windows.append([name, now, None])

    def __exit__(self, *exc) -> None:
        self.mark(None)
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""

    def _samples(self) -> list[tuple[float, float, float, set]]:
        from datetime import datetime

        rows = []
        for line in (self.out or "").splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                sm, smax = float(parts[2]), float(parts[3])
            except ValueError:
                continue
            reasons = {name for name, flag in zip(self.NAMES, parts[6:10]) if flag.lower() == "active"}
            rows.append((ts, sm, smax, reasons))
        return rows

    def summary(self) -> dict:
        rows = self._samples()
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        inside, per_window = [], {}
        for name, t0, t1 in self.windows:
            sel = [r for r in rows if t0 <= r[0] <= (t1 or float("inf"))]
            inside += sel
            per_window[name] = {"samples": len(sel), "seconds": round((t1 or t0) - t0, 3),
                                "sm_mhz": statistics.median(r[1] for r in sel) if sel else None}
        use = inside or rows
        reasons = sorted(set().union(*(r[3] for r in use)))
        return {"sm_mhz": statistics.median(r[1] for r in use), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": reasons, "samples": len(use), "samples_total": len(rows), "windows": per_window,
                "basis": "samples inside the named windows of measured replays" if inside else "all samples"}


# ---- CPU baseline (the reference's composition, restated in torch) ------------------------------------------
def host_threads() -> int:
    """Host cores this process may use (its affinity mask), the thread count of the CPU baseline."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class ReferenceSample:
    """A sub-batch of the workload's requests in the reference's own CPU layout (oracle/reference_torch.py:
    per-request pools of 16 repeated heads, shuffled tables), ready for decode steps of one layer."""

    def __init__(self, lens: list[int], seed: int, extra_tokens: int) -> None:
        import torch

        from oracle import reference_torch as ref

        gen = torch.Generator().manual_seed(seed + 99)
        tile = torch.randn(1 << 20, generator=gen).to(torch.float16)
        self.caches = []
        for n in lens:
            pages = (n + extra_tokens + BLOCK - 1) // BLOCK
            cache = ref.RequestCache(HQ, HEAD_DIM, pages, BLOCK, torch.float16,
                                     torch.randperm(pages, generator=gen).tolist())
            for blocks in (cache.key_blocks, cache.value_blocks):  # context values (timing only)
                flat = blocks.view(-1)
                for i in range(0, flat.numel(), tile.numel()):
                    flat[i:i + tile.numel()] = tile[:flat.numel() - i]
            cache.valid = n
            self.caches.append(cache)
        self.query = torch.randn((len(lens), HQ, 1, HEAD_DIM), generator=gen).to(torch.float16)
        self.key = torch.randn((len(lens), HKV, 1, HEAD_DIM), generator=gen).to(torch.float16)
        self.value = torch.randn((len(lens), HKV, 1, HEAD_DIM), generator=gen).to(torch.float16)

    def step(self) -> tuple[float, int]:
        """One decode step of the layer (append + gather + dense attention); returns (seconds, bytes)."""
        from oracle import reference_torch as ref

        t0 = time.perf_counter()
        ref.decode_step_layer(self.query, self.key, self.value, self.caches, HKV)
        seconds = time.perf_counter() - t0
        return seconds, decode_bytes([c.valid for c in self.caches]) + 4 * len(self.caches) * HKV * HEAD_DIM * 2


def rank0_cpu_baseline(args: argparse.Namespace, world: int, rank: int, lens: list[int]) -> dict | None:
    """cpu_baseline on rank 0 while the other ranks wait in a gloo barrier (a blocking socket read, so no
    rank spins a CPU core in a CUDA or NCCL wait while the baseline runs: a spinning thread per rank next to
    the baseline's thread pool slowed it down ~100x in multi-GPU runs)."""
    import torch

    if args.no_cpu_baseline:
        return None
    if world == 1:
        return cpu_baseline(lens, args.seed, args.cpu_seconds)
    import torch.distributed as dist

    from datetime import timedelta

    torch.cuda.synchronize()
    dist.barrier()
    host_group = dist.new_group(backend="gloo", timeout=timedelta(seconds=600))  # every rank creates it
    result = None
    try:
        if rank == 0:
            result = cpu_baseline(lens, args.seed, args.cpu_seconds, reserve=world - 1)
    finally:
        dist.barrier(group=host_group)  # a gloo barrier blocks in a socket read: no spinning core
        dist.destroy_process_group(host_group)
    return result


def cpu_baseline(lens: list[int], seed: int, budget_s: float, group: int = 8, reserve: int = 0) -> dict:
    """Times the reference's CPU composition of one decode step (per-row append of repeated heads,
    batch_kv_tensors, masked dense attention; oracle/reference_torch.py) on sub-batches of `group`
    requests of one layer of the workload, with every host core this process may use, until `budget_s`
    of timed work is done. GB/s counts the path's algorithmic bytes (unique K/V once), as on the GPU."""
    import torch

    threads = max(1, host_threads() - reserve)  # leave a core to each waiting rank's process
    before = torch.get_num_threads()
    torch.set_num_threads(threads)  # torchrun sets OMP_NUM_THREADS=1; the baseline gets every core
    try:
        done, bytes_done, elapsed = 0, 0, 0.0
        for start in range(0, len(lens), group):
            sample = ReferenceSample(lens[start:start + group], seed + start, 1)
            seconds, nbytes = sample.step()
            elapsed += seconds
            bytes_done += nbytes
            done += len(sample.caches)
            if elapsed >= budget_s:
                break
    finally:
        torch.set_num_threads(before)
    return {"value": bytes_done / elapsed / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "torch_threads": threads, "os_cpu_count": os.cpu_count(),
            "sample": f"{done} of {len(lens)} requests (sub-batches of {group}) x 1 of {NUM_LAYERS} layers of the "
                      f"workload, {elapsed:.1f} s: the reference's CPU decode composition restated in torch "
                      f"(per-row append of repeated heads, batch_kv_tensors, masked dense attention), "
                      f"bit-identical to the reference on its fixtures",
            "seconds": round(elapsed, 2)}


# ---- helpers -----------------------------------------------------------------------------------------------
def measured_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(summary: str = "paged_decode_config2.md") -> float | None:
    """dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel from the
    committed ncu summary of this workload (profiles/), or None."""
    path = ROOT / "profiles" / summary
    try:
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


# ---- our arm ---------------------------------------------------------------------------------------------
def run_ours(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    from tp_runtime import DecodeStepRunner

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    long_ctx = args.workload == "long"
    lens = [131072] * 8 if long_ctx else make_lengths(args.seed, rank)
    dtype = torch.bfloat16 if long_ctx else torch.float16
    layers = args.layers
    # every phase appends one token per step: first call, value (W + K), roofline, e2e (W + K)
    total_steps = 1 + 2 * (args.warmup + args.steps) + RL_STEPS + 8
    st = build_state(lens, total_steps, args.seed, rank, device, layers, dtype)
    cuda_cores = args.decode_kernel == "cuda"
    runner = DecodeStepRunner(st["key_pools"], st["value_pools"], st["tables"], st["lens0"].to(device),
                              num_q_heads=HQ, cuda_cores=cuda_cores, pages_per_split=args.pages_per_split)
    stream = torch.cuda.Stream(device)

    def barrier() -> None:
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()

    # ---- value: graph-captured step, device time
    with torch.cuda.stream(stream):
        runner.step(st["query"], st["key"], st["value"], st["out"])  # warm the library (attributes, maps)
    torch.cuda.synchronize(device)
    runner.seq_lens.copy_(st["lens0"].to(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            runner.step(st["query"], st["key"], st["value"], st["out"])
    torch.cuda.synchronize(device)
    runner.seq_lens.copy_(st["lens0"].to(device))
    cur = list(lens)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    cur = [n + args.warmup for n in cur]
    timed_lens = [[n + i + 1 for n in cur] for i in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    import paged_kv_ops as ops

    with ClockSampler(local) as clocks:
        clocks.mark("timed steps")
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            end.record(stream)
        barrier()
        clocks.mark(None)
        ms = start.elapsed_time(end)
        errors = runner.check_errors()
        ms_max = ms
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_max = float(t.item())
        step_bytes = sum(layers * layer_bytes(l) for l in timed_lens)
        value = world * step_bytes / (ms_max / 1e3) / 1e9  # every rank moves the same byte count
        batch = len(lens)
        tok_s = world * batch * args.steps / (ms_max / 1e3)
        del graph

        # ---- roofline: the step's paged-decode launches (attention + split merge of every layer, chained
        # as inside the step) captured alone in a CUDA graph and replayed; per launch = time / launches
        cur = [n + args.steps for n in cur]
        runner.seq_lens.copy_(torch.tensor(cur, dtype=torch.int32, device=device))
        torch.cuda.synchronize(device)
        rl_graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(rl_graph, stream=stream):
                for layer in range(layers):
                    ops.paged_decode(st["query"][layer], runner.key_pools[layer], runner.value_pools[layer],
                                     runner.block_tables, runner.seq_lens, workspace=runner.workspace,
                                     pages_per_split=runner.pages_per_split,
                                     out=st["out"][layer], error_flag=runner.error_flag, chained=True,
                                     cuda_cores=cuda_cores, prefetch=layer > 0)
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            rl_graph.replay()
            r0.record(stream)
            for _ in range(RL_REPLAYS):
                rl_graph.replay()
            r1.record(stream)
        torch.cuda.synchronize(device)
        dur_ms = r0.elapsed_time(r1) / (RL_REPLAYS * layers)
        rl_bytes = decode_bytes(cur)  # no append in this graph: the contexts stay at `cur`
        achieved = rl_bytes / (dur_ms / 1e3) / 1e9
        peak, peak_kind = measured_peak()
        # a sustained window of the same replays (about 1.5 s), so the clock record has samples under load
        window_replays = max(RL_REPLAYS, int(1500.0 / max(dur_ms * layers, 1e-3)))
        clocks.mark("decode-graph window")
        w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            w0.record(stream)
            for _ in range(window_replays):
                rl_graph.replay()
            w1.record(stream)
        torch.cuda.synchronize(device)
        clocks.mark(None)
        window_ms = w0.elapsed_time(w1) / (window_replays * layers)
        errors |= runner.check_errors()
        del rl_graph

    # ---- e2e: public API with host buffers (DecodePipeline: transfers overlap the previous step)
    from tp_runtime import DecodePipeline

    host_q = torch.empty(st["query"].shape, dtype=dtype, pin_memory=True).copy_(st["query"].cpu())
    host_k = torch.empty(st["key"].shape, dtype=dtype, pin_memory=True).copy_(st["key"].cpu())
    host_v = torch.empty(st["value"].shape, dtype=dtype, pin_memory=True).copy_(st["value"].cpu())
    host_out = [torch.empty(st["out"].shape, dtype=dtype, pin_memory=True) for _ in range(2)]
    runner.seq_lens.copy_(torch.tensor(cur, dtype=torch.int32, device=device))
    pipe = DecodePipeline(runner, dtype)
    for i in range(args.warmup):
        pipe.submit(host_q, host_k, host_v, host_out[i % 2])
    pipe.finish()
    cur = [n + args.warmup for n in cur]
    e2e_lens = [[n + i + 1 for n in cur] for i in range(args.steps)]
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(pipe.copy)
    pipe.compute.wait_stream(pipe.copy)
    last = None
    for i in range(args.steps):
        last = pipe.submit(host_q, host_k, host_v, host_out[i % 2])
    pipe.download.wait_event(last)
    e2.record(pipe.download)
    pipe.finish()
    barrier()
    e2e_ms = s2.elapsed_time(e2)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_bytes = sum(layers * layer_bytes(l) for l in e2e_lens)
    e2e_value = world * e2e_bytes / (e2e_ms / 1e3) / 1e9
    h2d = pipe.h2d_bytes
    d2h = pipe.d2h_bytes
    errors |= runner.check_errors()

    tp2 = None
    if world > 1 and world % 2 == 0 and not long_ctx:
        # the same GPUs composed as TP=2 pairs x request shards: the layout with a data-path exchange
        del pipe
        tp2 = tp_pairs_run(args, world, rank, local, layers, full=False)
    extras = None
    if not long_ctx and not args.no_extras:
        if world == 1:
            del pipe
        extras = secondary_workloads(args, world)
    cpu = None if long_ctx else rank0_cpu_baseline(args, world, rank, lens)
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16" if long_ctx else "f16",
            "data": "synthetic N(0,1) K/V/Q, seeded; " + ("contexts 131072" if long_ctx else "contexts U[1024,8192]"),
            "config": {"workload": (f"long-context split-KV decode step, batch 8 x 131072, {layers} layers"
                                    if long_ctx else
                                    f"decode step, batch 64, contexts U[1024,8192], {layers} full-attention layers"),
                       "batch": batch,
                       "contexts": "131072 each" if long_ctx else "uniform [1024, 8192] per rank",
                       "block_size": BLOCK,
                       "heads": f"{HQ}q/{HKV}kv", "head_dim": HEAD_DIM, "pool": f"{POOL_FACTOR}x tokens, shuffled",
                       "parallelism": f"request-sharded x{world} (weak)",
                       "l2": "inputs larger than L2 (pools 8.7 GB per GPU); no flush",
                       "timing": "CUDA graph of the step, replayed; CUDA events; max over ranks",
                       "decode_kernel": ("CUDA cores (PKV_DECODE_CUDA_CORES)" if cuda_cores
                                         else "mma.sync tensor cores, TMA page tiles")},
            "decode_tok_s": round(tok_s, 1),
            "pct_of_peak": round(100.0 * value / (world * peak), 1),
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "tok_s": round(world * batch * args.steps / (e2e_ms / 1e3), 1)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 3),
                         "traffic": (None if cuda_cores else
                                     profiled_traffic("paged_decode_long.md" if long_ctx else "paged_decode_config2.md")),
                         "kernel": ("paged_decode (decode_plan_kernel + decode_generic_kernel, CUDA cores)"
                                    if cuda_cores else "paged_decode (decode_tc_kernel + decode_tc_merge_kernel)"),
                         "algorithmic_bytes_per_launch": int(rl_bytes), "ms_per_launch": round(dur_ms, 4),
                         "launches_timed": RL_REPLAYS * layers,
                         "timing": "CUDA graph of the step's chained decode launches (no append), replayed; "
                                   "per launch = graph time / launches",
                         "ms_per_launch_sustained": round(window_ms, 4),
                         "frac_per_step": round(value / world / peak, 3),
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"},
            "gpu_launches": runner.launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "device_errors": errors,
        }
        if tp2 is not None:
            line["tp2_pairs"] = tp2
        if extras is not None:
            line["secondary_workloads"] = extras
        if cpu is not None:
            line["cpu_baseline"] = cpu
        emit(line)
    if world > 1 and _COLLECT is None:
        dist.destroy_process_group()


def secondary_workloads(args: argparse.Namespace, world: int) -> dict:
    """The other rows of the path measured in the same run, briefly (10 timed steps after 3 warm-up, no CPU
    baselines). One GPU: chunked prefill, decode over FP8 pages, the fused q/k norm + RoPE + append, the
    output stage alone and chained behind each layer's decode, the long-context split-KV decode (config 4)
    and continuous-batching churn (config 5). Several GPUs: configs 4 and 5 request-sharded over the ranks,
    config 5 also as TP=2 pairs x request shards (even N), the output stage with its tensor-parallel sum
    over all of them (NVLink exchange) and, on 2 GPUs, the chunked prefill with the KV heads split TP-style
    (config 3). Each entry keeps
    the figures of that workload's own line (bench.py --workload NAME prints it in full). Collective on
    every rank at N > 1."""
    global _COLLECT
    keep = ("metric", "value", "unit", "n_gpus", "ms_per_step", "decode_tok_s", "pct_of_peak", "roofline",
            "exact_probabilities", "ms_per_step_decode_only", "output_stage_us_per_layer_in_step",
            "output_stage_us_per_layer_unchained", "hbm_gbs", "tflops", "nccl_baseline", "device_errors")
    out = {}
    if world == 1:
        plan = (("prefill", run_prefill), ("decode_fp8", run_decode_fp8), ("normrope", run_normrope),
                ("oproj", run_oproj), ("attn_layer", run_attn_layer), ("long", run_ours), ("churn", run_churn))
    else:
        plan = (("long", run_ours), ("churn", run_churn), ("oproj", run_oproj))
        if world % 2 == 0:  # config 5 as TP=2 pairs x request shards
            plan += (("churn_tp", lambda sub: run_churn(sub, tp=2)),)
        if world == HKV:  # chunked prefill with the KV heads split over the ranks (config 3 at 2 GPUs)
            plan += (("prefill", run_prefill),)
    for name, fn in plan:
        sub = argparse.Namespace(**vars(args))
        sub.workload, sub.steps, sub.warmup, sub.no_cpu_baseline = name, min(args.steps, 10), 3, True
        sub.tokens, sub.layers = None, NUM_LAYERS
        _COLLECT = []
        import torch

        try:
            fn(sub)
            if _COLLECT:  # ranks other than 0 emit nothing
                line = _COLLECT[-1]
                entry = {k: line[k] for k in keep if k in line}
                clocks = line.get("clocks") or {}
                entry["clocks"] = {"sm_mhz": clocks.get("sm_mhz"), "reasons": clocks.get("reasons")}
                if name == "long":
                    entry["config"] = line.get("config", {}).get("workload")
                out[name] = entry
        except Exception as exc:  # noqa: BLE001 - a secondary figure must not cost the headline line
            out[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        finally:
            _COLLECT = None
            torch.cuda.empty_cache()
    return out


# ---- chunked-prefill workload -------------------------------------------------------------------------------
PREFILL_BATCH, PREFILL_CHUNK, PREFILL_MAX_PREFIX = 8, 2048, 4096


def measured_tensor_peak() -> tuple[float, str]:
    try:
        data = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(data["bf16_tflops"]), "measured burst"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def run_prefill(args: argparse.Namespace) -> None:
    """8 requests append a 2048-token bf16 chunk onto prefixes U[0, 4096] and attend causally over their
    pages. A step = kv_append of all chunks + paged_prefill. With N >= 2 ranks the KV heads are split
    TP-style (rank r: KV heads r*Hkv/N.., query heads r*Hq/N..) and head outputs are all-gathered."""
    import torch
    import torch.distributed as dist

    import paged_kv_ops as ops
    from tp_runtime import all_gather_heads, tp_head_range

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > HKV:
        raise SystemExit("prefill splits KV heads across ranks: use --gpus 1 or 2")
    kv0, hkv = tp_head_range(HKV, world, rank)
    q0, hq = tp_head_range(HQ, world, rank)
    gen = torch.Generator().manual_seed(1000 * args.seed + 3)
    prefixes = torch.randint(0, PREFILL_MAX_PREFIX + 1, (PREFILL_BATCH,), generator=gen).tolist()
    lens = [p + PREFILL_CHUNK for p in prefixes]
    need = [(n + BLOCK - 1) // BLOCK for n in lens]
    num_pages = sum(need) + 8
    perm = torch.randperm(num_pages, generator=gen)
    tables = torch.full((PREFILL_BATCH, max(need)), -1, dtype=torch.int32)
    used = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[used : used + n].to(torch.int32)
        used += n
    torch.manual_seed(1000 * args.seed + 5)
    dt = torch.bfloat16
    key_pool = torch.randn((num_pages, hkv, BLOCK, HEAD_DIM), dtype=dt, device=device)
    value_pool = torch.randn_like(key_pool)
    total_q = PREFILL_BATCH * PREFILL_CHUNK
    query = torch.randn((total_q, hq, HEAD_DIM), dtype=dt, device=device)
    chunk_k = torch.randn((total_q, hkv, HEAD_DIM), dtype=dt, device=device)
    chunk_v = torch.randn_like(chunk_k)
    slots = []
    for b in range(PREFILL_BATCH):
        row = tables[b].tolist()
        slots += [row[p // BLOCK] * BLOCK + p % BLOCK for p in range(prefixes[b], lens[b])]
    slots = torch.tensor(slots, dtype=torch.int64, device=device)
    cu = torch.arange(0, total_q + 1, PREFILL_CHUNK, dtype=torch.int32, device=device)
    bt, sl = tables.to(device), torch.tensor(lens, dtype=torch.int32, device=device)
    out = torch.empty_like(query)
    stream = torch.cuda.Stream(device)
    flag = ops.new_error_flag(device)

    def step(round_probs: bool, pre: list | None = None, post: list | None = None) -> None:
        ops.kv_append(chunk_k, chunk_v, slots, key_pool, value_pool, error_flag=flag)
        if pre is not None:
            pre.append(torch.cuda.Event(enable_timing=True))
            pre[-1].record(stream)
        ops.paged_prefill(query, cu, key_pool, value_pool, bt, sl, max_q_len=PREFILL_CHUNK, out=out,
                          error_flag=flag, round_probs=round_probs)
        if post is not None:
            post.append(torch.cuda.Event(enable_timing=True))
            post[-1].record(stream)
        if world > 1:
            all_gather_heads(out.view(PREFILL_BATCH * PREFILL_CHUNK, hq, HEAD_DIM))

    def timed(round_probs: bool) -> tuple[float, float, dict]:
        """(ms per step, ms per prefill launch, clocks) over args.steps steps after args.warmup."""
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step(round_probs)
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        pre, post = [], []
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            with torch.cuda.stream(stream):
                s0.record(stream)
                for _ in range(args.steps):
                    step(round_probs, pre, post)
                s1.record(stream)
            torch.cuda.synchronize(device)
        ms = s0.elapsed_time(s1) / args.steps
        kern_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(pre, post))
        if world > 1:
            t = torch.tensor([ms, kern_ms], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, kern_ms = float(t[0]), float(t[1])
        return ms, kern_ms, clocks.summary()

    # headline: probabilities rounded once to bf16 before P.V, as the reference does (probs.to(dtype),
    # src/tp_runtime.py:723); second line item: fp32-accurate probabilities (hi + lo bf16 parts)
    ms, kern_ms, clocks = timed(True)
    ms_exact, kern_exact, _ = timed(False)
    flops_total = sum(4 * HEAD_DIM * HQ * (PREFILL_CHUNK * p + PREFILL_CHUNK * (PREFILL_CHUNK + 1) // 2)
                      for p in prefixes)
    rank_flops = flops_total * hq / HQ
    peak, peak_kind = measured_tensor_peak()
    errors = int(flag.item())
    if rank == 0:
        emit({
            "metric": "chunked-prefill paged causal attention TFLOP/s (algorithmic), 8 x 2048-token chunks",
            "value": round(flops_total / (ms / 1e3) / 1e12, 1), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0,1), seeded; prefixes U[0,4096]",
            "config": {"workload": "chunked prefill: append 8 x 2048 tokens + causal paged attention",
                       "prefixes": prefixes, "heads": f"{HQ}q/{HKV}kv", "head_dim": HEAD_DIM,
                       "parallelism": f"TP={world} KV-head split" if world > 1 else "1 GPU"},
            "probabilities": "rounded once to bf16 before P.V, as the reference's probs.to(dtype)",
            "roofline": {"bound": "tensor", "achieved": round(rank_flops / (kern_ms / 1e3) / 1e12, 1),
                         "peak": peak, "unit": "TFLOP/s",
                         "frac": round(rank_flops / (kern_ms / 1e3) / 1e12 / peak, 3), "traffic": None,
                         "kernel": "prefill_tc_kernel", "ms_per_launch": round(kern_ms, 4),
                         "peak_source": f"MEASURED_PEAKS.json bf16_tflops ({peak_kind})"},
            "exact_probabilities": {
                "value": round(flops_total / (ms_exact / 1e3) / 1e12, 1), "unit": "TFLOP/s",
                "ms_per_step": round(ms_exact, 4), "ms_per_launch": round(kern_exact, 4),
                "frac": round(rank_flops / (kern_exact / 1e3) / 1e12 / peak, 3),
                "note": "P kept fp32-accurate as hi + lo bf16 parts: 1.5x the algorithmic tensor work"},
            "gpu_launches": 2 * args.steps, "clocks": clocks, "device_errors": errors,
        })
    if world > 1 and _COLLECT is None:
        dist.destroy_process_group()


# ---- continuous-batching churn workload -------------------------------------------------------------------
CHURN_REQUESTS, CHURN_FINISH, CHURN_MAX_COPIES = 256, 0.10, 20000


def churn_length(gen) -> int:
    import math

    import torch

    x = math.exp(7.5 + 1.0 * float(torch.randn((), generator=gen)))
    return int(min(max(x, 16), 32768))


def run_churn(args: argparse.Namespace, tp: int = 1) -> None:
    """256 concurrent requests (lognormal(7.5, 1) contexts clipped to [16, 32768]) decode over the 12
    layers; each step 10% finish and are replaced. Arrivals write their context into staging pages at
    the top of the pool (kv_append), the host compacts the pool into the lowest ids (kv_copy_pages over
    all layers, at most 20k pages), uploads the changed tables and decodes every request.

    tp = 1: every rank runs its own request set (request shards). tp = 2 (`--workload churn_tp`, an even
    number of GPUs): the ranks form TP=2 pairs that share one request set (the same plan on both ranks);
    rank r of a pair holds KV head r's pages only, serves query heads 8r..8r+7, and after each layer's
    decode the pair all-gathers the layer's head outputs (tp_runtime.HeadGather, on a side stream that
    overlaps the next layer's decode).

    The host scheduling (KVBlockManager) of all steps is planned before the timed region and its
    per-step results (copy lists, arrival slots, tables, lengths) are resident on the device, so the
    timed region is the device work of the steps back to back; the planning time is reported beside.
    value = bytes of the copy + append + decode kernels / device time, summed over the ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import paged_kv_ops as ops
    from scheduler import KVBlockManager
    from tp_runtime import DecodeStepRunner, HeadGather, tp_head_range

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    layers = args.layers
    if world % tp:
        raise SystemExit("TP=2 pairs need an even number of GPUs")
    shard, tp_rank = rank // tp, rank % tp
    group = None
    if tp > 1:
        groups = [dist.new_group([tp * p + r for r in range(tp)]) for p in range(world // tp)]
        group = groups[shard]
    _, hkv = tp_head_range(HKV, tp, tp_rank)
    _, hq = tp_head_range(HQ, tp, tp_rank)
    gen = torch.Generator().manual_seed(1000 * args.seed + 77 + shard)
    lengths0 = [churn_length(gen) for _ in range(CHURN_REQUESTS)]
    num_pages = int(1.6 * sum(lengths0) / BLOCK) + CHURN_REQUESTS * 8
    max_blocks = 32768 // BLOCK + 8
    mgr = KVBlockManager(num_pages, BLOCK, max_blocks)
    ids = [f"r{i}" for i in range(CHURN_REQUESTS)]
    for rid, n in zip(ids, lengths0):
        mgr.add_request(rid, n)
    page_bytes = hkv * BLOCK * HEAD_DIM * 2

    # ---- plan every step on the host
    t_plan = time.perf_counter()
    plans = []
    counter = CHURN_REQUESTS
    n_steps = args.warmup + args.steps
    for _ in range(n_steps):
        arrive = []
        for i in range(CHURN_REQUESTS):
            if float(torch.rand((), generator=gen)) < CHURN_FINISH:
                mgr.free_request(ids[i])
                ids[i] = f"r{counter}"
                counter += 1
                n = churn_length(gen)
                mgr.add_request(ids[i], n, staging=True)
                arrive += mgr.slots(ids[i], 0, n)
        src, dst = mgr.compact(max_moves=CHURN_MAX_COPIES)
        remap = {s_: d_ for s_, d_ in zip(src, dst)}
        arrive = [remap.get(x // BLOCK, x // BLOCK) * BLOCK + x % BLOCK for x in arrive]  # slots after the move
        for rid in ids:  # a page for this step's decode token where a request fills its last one
            entry = mgr.requests[rid]
            if len(entry.pages) * BLOCK <= entry.length:
                entry.pages.extend(mgr.allocator.allocate(1))
        lens_now = mgr.lengths(ids)
        plans.append({
            "src": np.asarray(src, dtype=np.int32), "dst": np.asarray(dst, dtype=np.int32),
            "arrive": np.asarray(arrive, dtype=np.int64),
            "tables": np.asarray(mgr.block_table_rows(ids), dtype=np.int32),
            "lens": np.asarray(lens_now, dtype=np.int32),
            "bytes": layers * layer_bytes([n + 1 for n in lens_now], hq, hkv) + 4 * layers * len(src) * page_bytes
                     + 4 * layers * len(arrive) * hkv * HEAD_DIM * 2,
        })
        for rid in ids:
            mgr.requests[rid].length += 1
    plan_ms = 1e3 * (time.perf_counter() - t_plan) / n_steps
    dev = []
    for pl in plans:
        dev.append({k: torch.from_numpy(v).to(device) for k, v in pl.items() if k != "bytes"})

    # ---- device state: pools hold lengths0 worth of tokens (random), tables of step 0
    shape = (layers, num_pages, hkv, BLOCK, HEAD_DIM)
    torch.manual_seed(1000 * args.seed + 79 + rank)
    key_pools = torch.randn(shape, dtype=torch.float16, device=device)
    value_pools = torch.randn_like(key_pools)
    longest = max((int(d["arrive"].numel()) for d in dev), default=1)
    src_kv = torch.randn((max(longest, 1), hkv, HEAD_DIM), dtype=torch.float16, device=device)
    runner = DecodeStepRunner(key_pools, value_pools, dev[0]["tables"].clone(), dev[0]["lens"].clone(),
                              num_q_heads=hq)
    q = torch.randn((layers, CHURN_REQUESTS, hq, HEAD_DIM), dtype=torch.float16, device=device)
    k = torch.randn((layers, CHURN_REQUESTS, hkv, HEAD_DIM), dtype=torch.float16, device=device)
    v = torch.randn_like(k)
    gather = HeadGather(layers, CHURN_REQUESTS, hq, HEAD_DIM, torch.float16, device, group) if tp > 1 else None
    out = gather.local_out if gather is not None else torch.empty_like(q)
    stream = torch.cuda.Stream(device)

    def device_step(d) -> None:
        if d["src"].numel():
            ops.kv_copy_pages(key_pools, value_pools, d["src"], d["dst"], error_flag=runner.error_flag)
        n = int(d["arrive"].numel())
        if n:
            for layer in range(layers):
                ops.kv_append(src_kv[:n], src_kv[:n], d["arrive"], key_pools[layer], value_pools[layer],
                              error_flag=runner.error_flag)
        runner.block_tables.copy_(d["tables"])
        runner.seq_lens.copy_(d["lens"])
        runner.step(q, k, v, out, gather=gather)

    with torch.cuda.stream(stream):
        for d in dev[: args.warmup]:
            device_step(d)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            s0.record(stream)
            for d in dev[args.warmup :]:
                device_step(d)
            s1.record(stream)
        torch.cuda.synchronize(device)
    ms = s0.elapsed_time(s1)
    errors = runner.check_errors()
    total_bytes = sum(pl["bytes"] for pl in plans[args.warmup :])
    copies = sum(len(pl["src"]) for pl in plans[args.warmup :]) / args.steps
    arrived = sum(len(pl["arrive"]) for pl in plans[args.warmup :]) / args.steps
    job_bytes = float(total_bytes)
    if world > 1:
        t = torch.tensor([ms, float(total_bytes)], dtype=torch.float64, device=device)
        dist.all_reduce(t[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[1:])  # every rank's copy + append + decode bytes
        ms, job_bytes = float(t[0].item()), float(t[1].item())
    del gather
    peak, _ = measured_peak()
    if rank == 0:
        parallelism = (f"request-sharded x{world} (weak)" if tp == 1 else
                       f"{world // tp} TP=2 pairs x request shards (rank: {hq}q/{hkv}kv heads; per-layer head-output "
                       "all-gather on a side stream)")
        emit({
            "metric": METRIC, "value": round(job_bytes / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic N(0,1), seeded; lognormal(7.5, 1) contexts clipped to [16, 32768]",
            "config": {"workload": f"continuous-batching churn, 256 requests, {layers} layers, 10% replaced per step",
                       "page_copies_per_step": round(copies, 1), "arrived_tokens_per_step": round(arrived, 1),
                       "host_planning_ms_per_step": round(plan_ms, 2), "parallelism": parallelism},
            "decode_tok_s": round((world // tp) * CHURN_REQUESTS * args.steps / (ms / 1e3), 1),
            "pct_of_peak": round(100.0 * job_bytes / world / (ms / 1e3) / 1e9 / peak, 1),
            "gpu_launches": None, "clocks": clocks.summary(), "device_errors": errors,
        })
    if world > 1 and _COLLECT is None:
        dist.destroy_process_group()


# ---- reference arm -----------------------------------------------------------------------------------------
def run_reference(args: argparse.Namespace) -> None:
    """The reference's own CPU composition for this path on the host cores (the reference package is
    Python and does not travel to the GPU box; oracle/reference_torch.py restates it op for op and is
    bit-identical to it on its fixtures): per step, one decode step of one layer over a bounded
    sub-batch of the workload's requests, with every host core. Under torchrun only rank 0 runs."""
    import torch

    if int(os.environ.get("RANK", "0")) != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    lens = make_lengths(args.seed, 0)
    per_step_requests = 8
    threads = host_threads()
    torch.set_num_threads(threads)
    sample = ReferenceSample(lens[:per_step_requests], args.seed, args.warmup + args.steps + 1)
    for _ in range(args.warmup):
        sample.step()
    results = [sample.step() for _ in range(args.steps)]
    seconds = sum(r[0] for r in results)
    value = sum(r[1] for r in results) / seconds / 1e9
    ms_per_step = 1e3 * seconds / args.steps
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic N(0,1), seeded; contexts U[1024,8192]",
        "config": {"workload": "decode step, batch 64, contexts U[1024,8192], 12 full-attention layers (sampled)",
                   "batch": BATCH, "block_size": BLOCK, "heads": f"{HQ}q/{HKV}kv", "head_dim": HEAD_DIM,
                   "parallelism": "host CPU, rank 0 only"},
        "impl": "reference",
        "decode_tok_s": round(per_step_requests / (NUM_LAYERS * seconds / args.steps), 3),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "torch_threads": threads, "os_cpu_count": os.cpu_count(),
                         "sample": f"{per_step_requests} requests x 1 layer per step: the reference's CPU decode "
                                   "composition (per-row append of repeated heads, batch_kv_tensors, masked dense "
                                   "attention) restated in torch, bit-identical to the reference on its fixtures"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- fused norm + rotary + append workload ---------------------------------------------------------------
def run_normrope(args: argparse.Namespace) -> None:
    """pkv_qk_norm_rope_append over the prefill chunk of config 3 (8 x 2048 tokens, 16q/2kv heads, head_dim
    256, partial rotary 0.25, bf16) into a shuffled pool. A step = one fused launch. HBM-bound: the
    algorithmic bytes are the pre-norm q/k/v read, the rotated query written, K and V written into their
    slots (the 64-row cos/sin table and the norm weights stay in L2)."""
    import torch

    import paged_kv_ops as ops

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    tokens = PREFILL_BATCH * PREFILL_CHUNK
    dt = torch.bfloat16
    gen = torch.Generator().manual_seed(1000 * args.seed + 11)
    num_pages = (tokens + BLOCK - 1) // BLOCK + 64
    slots = torch.randperm(num_pages * BLOCK, generator=gen)[:tokens].to(device)
    positions = torch.randint(0, 8192, (tokens,), generator=gen, dtype=torch.int32).to(device)
    torch.manual_seed(1000 * args.seed + 12)
    q_proj = torch.randn((tokens, HQ, 2 * HEAD_DIM), dtype=dt, device=device)  # query | gate per head
    key = torch.randn((tokens, HKV, HEAD_DIM), dtype=dt, device=device)
    value = torch.randn_like(key)
    q_norm = (0.1 * torch.randn((HEAD_DIM,), device=device)).to(dt)
    k_norm = (0.1 * torch.randn((HEAD_DIM,), device=device)).to(dt)
    table = ops.rope_cos_sin_table(8192, HEAD_DIM, 0.25, 1e7, dt, device)
    key_pool = torch.zeros((num_pages, HKV, BLOCK, HEAD_DIM), dtype=dt, device=device)
    value_pool = torch.zeros_like(key_pool)
    q_out = torch.empty((tokens, HQ, HEAD_DIM), dtype=dt, device=device)
    flag = ops.new_error_flag(device)
    stream = torch.cuda.Stream(device)

    def step() -> None:
        ops.qk_norm_rope_append(q_proj[:, :, :HEAD_DIM], key, value, q_norm, k_norm, table, positions, slots, key_pool,
                                value_pool, eps=1e-6, q_out=q_out, error_flag=flag)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize(device)
    # one launch per step (~0.07 ms) is shorter than the host's call: replay a CUDA graph of it so the
    # events time the kernel, not the Python call between kernels
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        clocks.mark("timed launches")
        with torch.cuda.stream(stream):
            graph.replay()
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / args.steps
    del graph
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    el = 2
    bytes_step = tokens * el * (HQ * HEAD_DIM * 2 + HKV * HEAD_DIM * 4)  # q read+write, k/v read + pool write
    peak, peak_kind = measured_peak()
    gbs = bytes_step / (ms / 1e3) / 1e9
    if rank == 0:
        emit({
            "metric": "fused q/k RMSNorm + rotary + K/V append GB/s (algorithmic), 16384 chunk tokens",
            "value": round(gbs * world, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seeded; random positions and slots",
            "config": {"workload": "pkv_qk_norm_rope_append, 8 x 2048 tokens, 16q/2kv, head_dim 256, rotary 64",
                       "bytes_per_step": bytes_step, "l2": "inputs 335 MB (> L2); no flush"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 3), "traffic": profiled_traffic("norm_rope_append_16k_tokens.md"),
                         "kernel": "norm_rope_append_kernel",
                         "ms_per_launch": round(ms, 4), "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"},
            "gpu_launches": args.steps, "clocks": clocks.summary(), "device_errors": int(flag.item()),
        })
    if world > 1 and _COLLECT is None:
        import torch.distributed as dist

        dist.destroy_process_group()


# ---- FP8 decode workload ----------------------------------------------------------------------------------
def run_decode_fp8(args: argparse.Namespace) -> None:
    """The decode configuration (batch 64, contexts U[1024, 8192], 12 layers, 16q/2kv, head_dim 256) over
    e4m3 K/V pages with one fp32 scale per (slot, KV head); query/output fp16. A step = slot mapping +
    per layer a quantising append and paged decode, replayed as a CUDA graph. The algorithmic bytes count
    the fp8 K/V (1 byte per element), their scales (4 bytes per row), tables, Q and O."""
    import torch
    import torch.distributed as dist

    import paged_kv_ops as ops
    from tp_runtime import DecodeStepRunner

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    lens = make_lengths(args.seed, rank)
    layers = args.layers
    total_steps = 1 + args.warmup + args.steps + RL_STEPS + 4
    gen = torch.Generator().manual_seed(1000 * args.seed + rank + 7)
    need = [(n + total_steps + BLOCK - 1) // BLOCK for n in lens]
    num_pages = max(int(POOL_FACTOR * sum(lens) / BLOCK) + 1, sum(need) + 1)
    perm = torch.randperm(num_pages, generator=gen)
    tables = torch.full((len(lens), max(need)), -1, dtype=torch.int32)
    used = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[used : used + n].to(torch.int32)
        used += n
    shape = (layers, num_pages, HKV, BLOCK, HEAD_DIM)
    torch.manual_seed(1000 * args.seed + rank + 11)
    # random finite e4m3 codes (0x7f / 0xff are NaN) and positive scales
    key_pools = (torch.randint(0, 0x7F, shape, dtype=torch.uint8, device=device)
                 | (torch.randint(0, 2, shape, dtype=torch.uint8, device=device) << 7))
    value_pools = (torch.randint(0, 0x7F, shape, dtype=torch.uint8, device=device)
                   | (torch.randint(0, 2, shape, dtype=torch.uint8, device=device) << 7))
    key_scales = torch.rand(shape[:4], device=device) / 448.0 + 1e-4
    value_scales = torch.rand(shape[:4], device=device) / 448.0 + 1e-4
    dt = torch.float16
    query = torch.randn((layers, len(lens), HQ, HEAD_DIM), dtype=dt, device=device)
    key = torch.randn((layers, len(lens), HKV, HEAD_DIM), dtype=dt, device=device)
    value = torch.randn_like(key)
    out = torch.empty_like(query)
    lens0 = torch.tensor(lens, dtype=torch.int32, device=device)
    runner = DecodeStepRunner(key_pools, value_pools, tables.to(device), lens0.clone(), num_q_heads=HQ,
                              key_scales=key_scales, value_scales=value_scales)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        runner.step(query, key, value, out)  # library set-up outside capture
    torch.cuda.synchronize(device)
    runner.seq_lens.copy_(lens0)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            runner.step(query, key, value, out)
    torch.cuda.synchronize(device)
    runner.seq_lens.copy_(lens0)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    cur = [n + args.warmup for n in lens]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize(device)
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del graph

    def fp8_decode_bytes(ls: list[int]) -> int:
        kv = sum(2 * HKV * (HEAD_DIM + 4) * n for n in ls)
        return kv + sum(4 * ((n + BLOCK - 1) // BLOCK) for n in ls) + 2 * len(ls) * HQ * HEAD_DIM * 2

    step_bytes = sum(layers * (fp8_decode_bytes([n + i + 1 for n in cur]) + len(lens) * HKV * 2 * (HEAD_DIM * 3 + 4))
                     for i in range(args.steps))
    value_gbs = world * step_bytes / (ms / 1e3) / 1e9
    tok_s = world * len(lens) * args.steps / (ms / 1e3)
    # roofline: the step's chained fp8 decode launches alone in a CUDA graph, replayed; per launch
    cur = [n + args.steps for n in cur]
    runner.seq_lens.copy_(torch.tensor(cur, dtype=torch.int32, device=device))
    torch.cuda.synchronize(device)
    rl_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(rl_graph, stream=stream):
            for layer in range(layers):
                ops.paged_decode_fp8(query[layer], key_pools[layer], value_pools[layer], key_scales[layer],
                                     value_scales[layer], runner.block_tables, runner.seq_lens,
                                     workspace=runner.workspace, out=out[layer], error_flag=runner.error_flag,
                                     chained=True, prefetch=layer > 0)
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        rl_graph.replay()
        r0.record(stream)
        for _ in range(RL_REPLAYS):
            rl_graph.replay()
        r1.record(stream)
    torch.cuda.synchronize(device)
    dur_ms = r0.elapsed_time(r1) / (RL_REPLAYS * layers)
    del rl_graph
    rl_bytes = fp8_decode_bytes(cur)
    achieved = rl_bytes / (dur_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    errors = runner.check_errors()
    if rank == 0:
        emit({
            "metric": "paged-decode KV HBM GB/s and decode tok/s over e4m3 KV pages, batch 64",
            "value": round(value_gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp8 e4m3 KV, f16 query",
            "data": "synthetic random e4m3 pages and scales, N(0,1) query; contexts U[1024,8192]",
            "config": {"workload": f"decode step over fp8 pages, batch 64, contexts U[1024,8192], {layers} layers",
                       "block_size": BLOCK, "heads": f"{HQ}q/{HKV}kv", "head_dim": HEAD_DIM,
                       "scales": "fp32 per (slot, KV head)", "timing": "CUDA graph of the step, replayed"},
            "decode_tok_s": round(tok_s, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 3),
                         "traffic": profiled_traffic("paged_decode_fp8_config2.md"),
                         "kernel": "paged_decode_fp8 (decode_tc_kernel<fp8> + merge)",
                         "ms_per_launch": round(dur_ms, 4), "algorithmic_bytes_per_launch": int(rl_bytes),
                         "timing": "CUDA graph of the step's chained decode launches (no append), replayed",
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"},
            "gpu_launches": runner.launches_per_step * args.steps, "clocks": clocks.summary(),
            "device_errors": errors,
        })
    if world > 1 and _COLLECT is None:
        dist.destroy_process_group()


# ---- TP pairs x request shards ------------------------------------------------------------------------
def tp_pairs_run(args: argparse.Namespace, world: int, rank: int, local: int, layers: int, *,
                 full: bool) -> dict:
    """The decode configuration on `world` GPUs composed as world/2 tensor-parallel pairs x request shards.

    The two ranks of a pair share one batch-64 request set (contexts U[1024, 8192], seeded by pair);
    rank r of a pair holds KV head r (its pages only) and serves query heads 8r..8r+7. A step is the
    12-layer paged step (slot mapping, append, chained decode per layer) with every layer's head outputs
    all-gathered inside the pair right after that layer's decode (tp_runtime.HeadGather: preallocated,
    in place, on a side stream that overlaps the next layer's decode), all in one CUDA graph.
    Collective: every rank calls it. Returns the figures of the whole job (max time over ranks)."""
    import torch
    import torch.distributed as dist

    import paged_kv_ops as ops
    from tp_runtime import DecodePipeline, DecodeStepRunner, HeadGather, tp_head_range

    device = torch.device("cuda", local)
    tp = 2
    if world % tp:
        raise SystemExit("TP=2 pairs need an even number of GPUs")
    pair, tp_rank = rank // tp, rank % tp
    groups = [dist.new_group([tp * p + r for r in range(tp)]) for p in range(world // tp)]
    group = groups[pair]
    _, hkv = tp_head_range(HKV, tp, tp_rank)
    _, hq = tp_head_range(HQ, tp, tp_rank)
    lens = make_lengths(args.seed, pair)  # the pair's requests
    batch = len(lens)
    total_steps = 1 + 3 * (args.warmup + args.steps) + 8
    st = build_state(lens, total_steps, args.seed, rank, device, layers, torch.float16, hq=hq, hkv=hkv)
    runner = DecodeStepRunner(st["key_pools"], st["value_pools"], st["tables"], st["lens0"].to(device),
                              num_q_heads=hq, pages_per_split=args.pages_per_split)
    gather = HeadGather(layers, batch, hq, HEAD_DIM, torch.float16, device, group)
    stream = torch.cuda.Stream(device)

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(graph, steps: int) -> float:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        dist.barrier()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize(device)
        dist.barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    # eager step first: initialises the pair's communicator and the library outside any capture
    with torch.cuda.stream(stream):
        runner.step(st["query"], st["key"], st["value"], gather.local_out, gather=gather)
    torch.cuda.synchronize(device)
    runner.seq_lens.copy_(st["lens0"].to(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            runner.step(st["query"], st["key"], st["value"], gather.local_out, gather=gather)
    paged = torch.cuda.CUDAGraph()  # the same step without the exchange: the gather's share of the step
    with torch.cuda.stream(stream):
        with torch.cuda.graph(paged, stream=stream):
            runner.step(st["query"], st["key"], st["value"], gather.local_out)
    torch.cuda.synchronize(device)
    cur = list(lens)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    cur = [n + args.warmup for n in cur]
    ms = timed(graph, args.steps)
    rank_bytes = sum(layers * layer_bytes([n + i + 1 for n in cur], hq, hkv) for i in range(args.steps))
    cur = [n + args.steps for n in cur]
    ms_paged = timed(paged, args.steps)
    cur = [n + args.steps for n in cur]
    b = torch.tensor([float(rank_bytes)], dtype=torch.float64, device=device)
    dist.all_reduce(b)  # every rank moves its KV head's pages and its query heads' Q/O
    job_bytes = float(b.item())
    value = job_bytes / (ms / 1e3) / 1e9
    out = {
        "value": round(value, 1), "unit": "GB/s", "ms_per_step": round(ms / args.steps, 4),
        "decode_tok_s": round((world // tp) * batch * args.steps / (ms / 1e3), 1),
        "ms_per_step_without_exchange": round(ms_paged / args.steps, 4),
        "exchange_share_of_step": round(max(0.0, 1.0 - ms_paged / ms), 3),
        "layout": f"{world // tp} TP=2 pairs x batch 64; rank: {hq}q/{hkv}kv heads",
        "exchange": "per layer, in-place NCCL all_gather_into_tensor of 64 x 8 x 256 fp16 head outputs on a "
                    "side stream overlapping the next layer's decode; captured with the step in one CUDA graph",
    }
    del graph, paged
    if full:
        # roofline: the step's chained decode launches alone, in a graph, per launch
        runner.seq_lens.copy_(torch.tensor(cur, dtype=torch.int32, device=device))
        torch.cuda.synchronize(device)
        rl = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(rl, stream=stream):
                for layer in range(layers):
                    ops.paged_decode(st["query"][layer], runner.key_pools[layer], runner.value_pools[layer],
                                     runner.block_tables, runner.seq_lens, workspace=runner.workspace,
                                     pages_per_split=runner.pages_per_split,
                                     out=gather.local_out[layer], error_flag=runner.error_flag, chained=True,
                                     prefetch=layer > 0)
        with torch.cuda.stream(stream):
            rl.replay()
        rl_ms = timed(rl, RL_REPLAYS) / (RL_REPLAYS * layers)
        rl_bytes = decode_bytes(cur, hq, hkv)
        del rl
        peak, peak_kind = measured_peak()
        out["roofline"] = {"bound": "hbm", "achieved": round(rl_bytes / (rl_ms / 1e3) / 1e9, 1), "peak": peak,
                           "unit": "GB/s", "frac": round(rl_bytes / (rl_ms / 1e3) / 1e9 / peak, 3),
                           "traffic": None, "kernel": "paged_decode (decode_tc_kernel + decode_tc_merge_kernel), "
                                                       "one KV head per rank",
                           "algorithmic_bytes_per_launch": int(rl_bytes), "ms_per_launch": round(rl_ms, 4),
                           "timing": "CUDA graph of the step's chained decode launches, max over ranks",
                           "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"}
        # e2e through the public pipeline: pinned host q/k/v in, the gathered heads back, every step
        gathers = (HeadGather(layers, batch, hq, HEAD_DIM, torch.float16, device, group), gather)
        host_q = torch.empty(st["query"].shape, dtype=torch.float16, pin_memory=True).copy_(st["query"].cpu())
        host_k = torch.empty(st["key"].shape, dtype=torch.float16, pin_memory=True).copy_(st["key"].cpu())
        host_v = torch.empty(st["value"].shape, dtype=torch.float16, pin_memory=True).copy_(st["value"].cpu())
        host_out = [torch.empty(gather.buffer.shape, dtype=torch.float16, pin_memory=True) for _ in range(2)]
        runner.seq_lens.copy_(torch.tensor(cur, dtype=torch.int32, device=device))
        with torch.cuda.stream(stream):  # the second buffer set's communicator use, outside capture
            runner.step(st["query"], st["key"], st["value"], gathers[0].local_out, gather=gathers[0])
        torch.cuda.synchronize(device)
        cur = [n + 1 for n in cur]
        pipe = DecodePipeline(runner, torch.float16, gathers=gathers)
        for i in range(args.warmup):
            pipe.submit(host_q, host_k, host_v, host_out[i % 2])
        pipe.finish()
        cur = [n + args.warmup for n in cur]
        dist.barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(pipe.copy)
        pipe.compute.wait_stream(pipe.copy)
        last = None
        for i in range(args.steps):
            last = pipe.submit(host_q, host_k, host_v, host_out[i % 2])
        pipe.download.wait_event(last)
        e2.record(pipe.download)
        pipe.finish()
        dist.barrier()
        e2e_ms = max_over_ranks(s2.elapsed_time(e2))
        e2e_bytes = sum(layers * layer_bytes([n + i + 1 for n in cur], hq, hkv) for i in range(args.steps))
        b = torch.tensor([float(e2e_bytes)], dtype=torch.float64, device=device)
        dist.all_reduce(b)
        out["e2e"] = {"value": round(float(b.item()) / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
                      "h2d_bytes_per_step": pipe.h2d_bytes, "d2h_bytes_per_step": pipe.d2h_bytes,
                      "tok_s": round((world // tp) * batch * args.steps / (e2e_ms / 1e3), 1),
                      "path": "tp_runtime.DecodePipeline with HeadGather per buffer set"}
        pipe.release()
        del pipe
    out["device_errors"] = runner.check_errors()
    out["gpu_launches"] = runner.launches_per_step * args.steps
    out["nccl_calls_per_step"] = layers
    torch.cuda.synchronize(device)
    dist.barrier()
    return out


def run_decode_tp(args: argparse.Namespace) -> None:
    """bench.py --workload decode_tp --gpus N: the TP=2 pairs x request shards composition (tp_pairs_run)
    as a full benchmark line."""
    world, rank, local = dist_setup()
    if world < 2:
        raise SystemExit("decode_tp needs at least 2 GPUs (torchrun --nproc-per-node N, N even)")
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    layers = args.layers
    with ClockSampler(local) as clocks:
        clocks.mark("tp pairs")
        res = tp_pairs_run(args, world, rank, local, layers, full=True)
    cpu = rank0_cpu_baseline(args, world, rank, make_lengths(args.seed, 0))
    dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": res.pop("value"), "unit": res.pop("unit"), "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": res.pop("ms_per_step"),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic N(0,1) K/V/Q, contexts U[1024,8192], shuffled pages",
            "config": {"workload": f"decode step, {layers} layers, {world // 2} TP=2 pairs x batch 64",
                       "parallelism": f"tp2 x dp{world // 2}", "layout": res.pop("layout"),
                       "exchange": res.pop("exchange"), "l2": "KV pools far larger than L2",
                       "timing": "CUDA graph of the step with its per-layer gathers; CUDA events; max over ranks"},
            "clocks": clocks.summary(),
        }
        line.update(res)
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


# ---- attention output stage workload ------------------------------------------------------------------------
OPROJ_HIDDEN = 2048  # hidden size of the Qwen3-Next-style configuration (16 q heads x 256 -> 2048)


def run_oproj(args: argparse.Namespace) -> None:
    """The output stage of the decode step's 12 full-attention layers at batch 64 (src/tp_runtime.py:672-695):
    bf16 heads and gate (64 tokens, 16/N heads x 256), this rank's e4m3 o_proj shard (2048, 4096/N) with bf16
    block scales, the rank partials summed over the N GPUs (N = the tensor-parallel size; N = 1 is the whole
    projection on one GPU). A step = 12 layers through pkv_gated_o_proj, replayed as a CUDA graph; L2 is
    flushed (256 MB write) before every timed step, outside its events. At N > 1 the same step is also timed
    with the reference's composition (each rank's partial, then NCCL all_reduce), both eager."""
    import torch
    import torch.distributed as dist

    import paged_kv_ops as ops

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    tokens, hidden, layers = args.tokens or BATCH, OPROJ_HIDDEN, args.layers
    if HQ % world:
        raise SystemExit("the tensor-parallel size must divide the 16 query heads")
    hl = HQ // world
    k = hl * HEAD_DIM
    dt = torch.bfloat16
    torch.manual_seed(1000 * args.seed + 41 + rank)
    heads = [torch.randn((tokens, hl, 1, HEAD_DIM), device=device).to(dt) for _ in range(layers)]
    gates = [(2 * torch.randn((tokens, 1, k), device=device)).to(dt) for _ in range(layers)]
    weights = [(0.05 * torch.randn((hidden, k), device=device)).to(torch.float8_e4m3fn) for _ in range(layers)]
    scales = [(0.5 + torch.rand((hidden // 128, k // 128), device=device)).to(torch.bfloat16) for _ in range(layers)]
    outs = [torch.empty((tokens, 1, hidden), dtype=dt, device=device) for _ in range(layers)]
    work = torch.empty(ops.o_proj_workspace_size(tokens, k, hidden), dtype=torch.uint8, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    flag = ops.new_error_flag(device)
    exchange = None
    if world > 1:
        exchange = ops.OutputExchange(rank, world, tokens, hidden, dt, device)
        handles = [None] * world
        dist.all_gather_object(handles, exchange.allocate())
        exchange.attach(handles)
        dist.barrier()
    stream = torch.cuda.Stream(device)

    def step_fused() -> None:
        for i in range(layers):
            ops.gated_o_proj(heads[i], gates[i], weights[i], scales[i], out_dtype=dt, exchange=exchange, out=outs[i],
                             workspace=work, error_flag=flag)

    def step_nccl() -> None:
        for i in range(layers):
            ops.gated_o_proj(heads[i], gates[i], weights[i], scales[i], out_dtype=dt, out=outs[i], workspace=work,
                             error_flag=flag)
            dist.all_reduce(outs[i])

    def timed(run, steps: int) -> float:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        with torch.cuda.stream(stream):
            for a, b in evs:
                flush.zero_()
                a.record(stream)
                run()
                b.record(stream)
        torch.cuda.synchronize(device)
        ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t[0])
        return ms

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step_fused()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_fused()
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clocks:
        ms = timed(graph.replay, args.steps)
    ms_eager = timed(step_fused, max(args.steps // 4, 3))
    nccl_ms = None
    if world > 1:
        with torch.cuda.stream(stream):
            for _ in range(3):
                step_nccl()
        torch.cuda.synchronize(device)
        nccl_ms = timed(step_nccl, max(args.steps // 4, 3))
    errors = int(flag.item())
    per_layer = hidden * k + (hidden // 128) * (k // 128) * 2 + 2 * tokens * k * 2 + tokens * hidden * 2
    bytes_step = layers * per_layer
    flops_step = layers * 2.0 * tokens * hidden * k
    peak, peak_kind = measured_peak()
    gbs = bytes_step / (ms / 1e3) / 1e9
    tflops = flops_step / (ms / 1e3) / 1e12
    tpeak, tpeak_kind = measured_tensor_peak()
    # the roofline that bounds this call: HBM below the ridge point (flops per byte of the two peaks), tensor above
    tensor_bound = flops_step / bytes_step > tpeak * 1e12 / (peak * 1e9)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import numpy as np

        from oracle import paged_kv_oracle as oracle

        h = heads[0].float().reshape(tokens, k).cpu().numpy()
        g = gates[0].float().reshape(tokens, k).cpu().numpy()
        codes = weights[0].view(torch.uint8).cpu().numpy()
        sb = scales[0].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 10.0) or reps == 0:
            x, _ = oracle.gate_heads(h, g, "bfloat16", "bfloat16")
            oracle.o_proj_partial(x, codes, sb, "bfloat16")
            reps += 1
        layer_s = (time.perf_counter() - t0) / reps
        cpu = {"value": round(tokens / (layer_s * layers), 1), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{reps} x one layer (gate + dequantise + fp64 GEMM, numpy/BLAS), reported x{layers} layers"}
    if world > 1:
        del graph
        torch.cuda.synchronize(device)
        dist.barrier()
        exchange.close()
    if rank == 0:
        line = {
            "metric": f"attention output stage (gate, FP8 o_proj, TP all-reduce) tok/s, "
                      f"{'decode batch' if tokens == BATCH else 'tokens per call'} {tokens}, {layers} layers",
            "value": round(tokens / (ms / 1e3), 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 activations, e4m3 weight, fp32 accumulation",
            "data": "synthetic N(0,1) heads, 2 N(0,1) gate, 0.05 N(0,1) e4m3 weights, U[0.5,1.5] scales",
            "config": {"workload": f"pkv_gated_o_proj x {layers} layers, {tokens} tokens, hidden {hidden}, TP={world} "
                                   f"(K per rank {k})", "l2": "256 MB flush before each timed step",
                       "timing": "CUDA graph of the step, replayed", "ms_per_step_eager": round(ms_eager, 4)},
            "hbm_gbs": round(gbs, 1), "tflops": round(tflops, 1),
            "roofline": ({"bound": "tensor", "achieved": round(tflops, 1), "peak": tpeak, "unit": "TFLOP/s",
                          "frac": round(tflops / tpeak, 3),
                          "traffic": profiled_traffic("oproj_prefill_8192_tokens.md") if tokens == 8192 else None,
                          "peak_source": f"MEASURED_PEAKS.json bf16_tflops ({tpeak_kind})"} if tensor_bound else
                         {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                          "frac": round(gbs / peak, 3),
                          "traffic": profiled_traffic("oproj_decode_tp1.md") if world == 1 and tokens == BATCH else None,
                          "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"})
            | {"kernel": "gated_o_proj (gate + oproj_kernel" + (" + finish)" if world > 1 else ")"),
               "ms_per_launch": round(ms / layers, 5), "algorithmic_bytes_per_launch": per_layer,
               "algorithmic_flops_per_launch": 2.0 * tokens * hidden * k},
            "gpu_launches": layers * (3 if world > 1 else 2) * args.steps, "clocks": clocks.summary(),
            "device_errors": errors,
        }
        if nccl_ms is not None:
            line["nccl_baseline"] = {"ms_per_step": round(nccl_ms, 4), "what": "same partials + NCCL all_reduce, eager",
                                     "fused_eager_ms_per_step": round(ms_eager, 4)}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        emit(line)
    if world > 1 and _COLLECT is None:
        dist.destroy_process_group()


# ---- decode step with each layer's output stage --------------------------------------------------------------
def run_attn_layer(args: argparse.Namespace) -> None:
    """The decode configuration with every full-attention layer's output stage behind its decode: per layer
    the paged decode (attention + split merge) and then gate * sigmoid, the FP8 block-scaled o_proj
    (2048 x 4096 e4m3 with bf16 128 x 128 scales) and, on one GPU, no all-reduce -- what
    _tp_full_attention_batch does after its projections (src/tp_runtime.py:2498-2555, :672-695). The
    output stage is launched chained (PKV_OPROJ_CHAINED): it is resident while the layer's decode drains
    and streams its weights at once. The same step is also timed without the output stage and with it
    launched unchained, so the stage's cost inside the step is measured directly. All CUDA graphs."""
    import torch

    import paged_kv_ops as ops
    from tp_runtime import DecodeStepRunner, finish_from_heads

    world, rank, local = dist_setup()
    if world > 1:
        raise SystemExit("attn_layer runs on one GPU (the multi-GPU output stage is --workload oproj)")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    layers = args.layers
    lens = make_lengths(args.seed, rank)
    total_steps = 3 * (1 + args.warmup + args.steps) + 8
    st = build_state(lens, total_steps, args.seed, rank, device, layers, torch.float16)
    runner = DecodeStepRunner(st["key_pools"], st["value_pools"], st["tables"], st["lens0"].to(device), num_q_heads=HQ)
    k, hidden, batch = HQ * HEAD_DIM, OPROJ_HIDDEN, len(lens)
    torch.manual_seed(1000 * args.seed + 43)
    gate = (2 * torch.randn((layers, batch, k), device=device)).to(torch.float16)
    weight = (0.05 * torch.randn((layers, hidden, k), device=device)).to(torch.float8_e4m3fn)
    scale = (0.5 + torch.rand((layers, hidden // 128, k // 128), device=device)).to(torch.bfloat16)
    hid = torch.empty((layers, batch, hidden), dtype=torch.float16, device=device)
    work = torch.empty(ops.o_proj_workspace_size(batch, k, hidden), dtype=torch.uint8, device=device)
    stream = torch.cuda.Stream(device)

    def output_stage(chained: bool):
        def run(layer: int) -> None:
            finish_from_heads(st["out"][layer], gate[layer], weight[layer], scale[layer], torch.float16,
                              out=hid[layer], workspace=work, error_flag=runner.error_flag, chained=chained)
        return run

    variants = {"layer": output_stage(True), "layer_unchained": output_stage(False), "decode_only": None}
    with torch.cuda.stream(stream):  # the library's one-time set-up, outside any capture
        runner.step(st["query"], st["key"], st["value"], st["out"], after_layer=variants["layer"])
    torch.cuda.synchronize(device)
    graphs = {}
    for name, hook in variants.items():
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                runner.step(st["query"], st["key"], st["value"], st["out"], after_layer=hook)
        graphs[name] = g
    torch.cuda.synchronize(device)
    cur = [n + 1 for n in lens]
    times, step_lens = {}, {}
    with ClockSampler(local) as clocks:
        for name in ("layer", "decode_only", "layer_unchained"):
            runner.seq_lens.copy_(torch.tensor(cur, dtype=torch.int32, device=device))
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    graphs[name].replay()
            torch.cuda.synchronize(device)
            cur = [n + args.warmup for n in cur]
            step_lens[name] = [[n + i + 1 for n in cur] for i in range(args.steps)]
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            clocks.mark(name)
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(args.steps):
                    graphs[name].replay()
                e1.record(stream)
            torch.cuda.synchronize(device)
            clocks.mark(None)
            times[name] = e0.elapsed_time(e1) / args.steps
            cur = [n + args.steps for n in cur]
    errors = runner.check_errors()
    del graphs
    oproj_bytes = hidden * k + (hidden // 128) * (k // 128) * 2 + 2 * batch * k * 2 + batch * hidden * 2
    step_bytes = statistics.mean(layers * (layer_bytes(l) + oproj_bytes) for l in step_lens["layer"])
    ms = times["layer"]
    peak, peak_kind = measured_peak()
    value = step_bytes / (ms / 1e3) / 1e9
    emit({
        "metric": "decode step with each layer's output stage, KV + o_proj weight HBM GB/s and tok/s, batch 64",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 (e4m3 o_proj weights, fp32 accumulation)",
        "data": "synthetic N(0,1) K/V/Q, 2 N(0,1) gate, 0.05 N(0,1) e4m3 weights; contexts U[1024,8192]",
        "config": {"workload": f"decode step, batch 64, contexts U[1024,8192], {layers} layers, each followed by "
                               "gate + FP8 o_proj (hidden 2048), TP=1",
                   "timing": "CUDA graphs of each variant, replayed; CUDA events",
                   "l2": "KV pools far larger than L2; weights read once per step"},
        "decode_tok_s": round(batch / (ms / 1e3), 1), "pct_of_peak": round(100 * value / peak, 1),
        "ms_per_step_decode_only": round(times["decode_only"], 4),
        "ms_per_step_output_stage_unchained": round(times["layer_unchained"], 4),
        "output_stage_us_per_layer_in_step": round(1e3 * (ms - times["decode_only"]) / layers, 2),
        "output_stage_us_per_layer_unchained": round(1e3 * (times["layer_unchained"] - times["decode_only"]) / layers, 2),
        "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
        "gpu_launches": (runner.launches_per_step + 2 * layers) * args.steps, "clocks": clocks.summary(),
        "device_errors": errors,
    })


def main(argv: list[str] | None = None) -> int:
    args = parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "churn":
        run_churn(args)
    elif args.workload == "churn_tp":
        run_churn(args, tp=2)
    elif args.workload == "normrope":
        run_normrope(args)
    elif args.workload == "decode_fp8":
        run_decode_fp8(args)
    elif args.workload == "oproj":
        run_oproj(args)
    elif args.workload == "decode_tp":
        run_decode_tp(args)
    elif args.workload == "attn_layer":
        run_attn_layer(args)
    else:
        run_ours(args)
    return 0


if __name__ == "__main__":
    sys.exit(main())
