"""Parity at the benchmark's own shapes, through the objects the benchmark times.

config 2 (the headline): batch 64, contexts U[1024, 8192] (seed 0, rank 0), fp16, 16q/2kv heads,
head_dim 256, pages shuffled in a pool of 1.2x the tokens, 12 stacked layers -- built by
bench.build_state itself. Steps run (a) eagerly, (b) as replays of one CUDA graph of
DecodeStepRunner.step (what `value` times) and (c) through DecodePipeline.submit from pinned host
buffers (what `e2e` times). After every step the appended K/V rows of all 12 layers are bit-exact at
the oracle's slots and every request of one layer matches the oracle's dense decode attention.

config 4: batch 8 x 131072 tokens, bf16; every request matches the oracle with automatic splits and
with 64 partitions of 2048 tokens.

config 5: 256 concurrent requests, lognormal(7.5, 1) contexts clipped to [16, 32768], 10 % replaced
per step, arrivals staged at the top of the pool and compacted by kv_copy_pages with the scheduler's
real copy lists (capped at 20k pages as the benchmark does), one decode token per request per step
through DecodeStepRunner, 5 steps over 2 layers (two layers keep the host-side expected copy of every
token at 1.5 GB; the kernels are the same for 12): every request's pages hold exactly its tokens
after every step, and every request of layer 0 matches the oracle.

Tolerance of the attention outputs (fp16/bf16): |got - oracle| <= 2e-3 + 1e-2 * |oracle|, against the
oracle's fp32-probability mode (the kernels keep P in fp32).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
import pkv_testlib as lib
from oracle import paged_kv_oracle as oracle

pytestmark = pytest.mark.gpu
DEVICE = torch.device("cuda", 0)
BS, HQ, HKV, D = bench.BLOCK, bench.HQ, bench.HKV, bench.HEAD_DIM


def _host_tables(tables: torch.Tensor) -> list[list[int]]:
    rows = tables.cpu().tolist()
    return [[p for p in row if p >= 0] for row in rows]


def _check_appended(key_pools, value_pools, key, value, tables, lens_before, what: str) -> None:
    """The step's new K/V of every layer sit bit for bit at the oracle's slot of each request."""
    slots = [int(oracle.slot_mapping(t, n, 1, BS)[0]) for t, n in zip(tables, lens_before)]
    page = torch.tensor([s // BS for s in slots], device=DEVICE)
    off = torch.tensor([s % BS for s in slots], device=DEVICE)
    for layer in range(key_pools.shape[0]):
        got_k = key_pools[layer][page, :, off, :]  # (batch, hkv, d)
        got_v = value_pools[layer][page, :, off, :]
        assert torch.equal(got_k.view(torch.int16), key[layer].view(torch.int16)), (what, layer)
        assert torch.equal(got_v.view(torch.int16), value[layer].view(torch.int16)), (what, layer)


def _oracle_layer(query_layer, key_pool, value_pool, tables, lens, dtype_name: str) -> np.ndarray:
    """Dense decode attention of every request over its first lens[b] tokens, one request (and KV
    head) at a time: the oracle's composition on that request's pages gathered from the device."""
    q = lib.as_f32(lib.np_bits(query_layer), dtype_name)  # (batch, hq, d)
    out = np.zeros(q.shape, dtype=np.float32)
    group = HQ // HKV
    for b, (table, n) in enumerate(zip(tables, lens)):
        pages = (n + BS - 1) // BS
        idx = torch.tensor(table[:pages], device=DEVICE)
        pk = lib.np_bits(key_pool[idx])
        pv = lib.np_bits(value_pool[idx])
        local = [list(range(pages))]
        for h in range(HKV):
            out[b, h * group:(h + 1) * group] = oracle.decode_attention(
                q[b:b + 1, h * group:(h + 1) * group], pk[:, h:h + 1], pv[:, h:h + 1], local, [n],
                dtype=dtype_name, round_probs=False)[0]
    return out


def test_config2_full_shape_eager_graph_and_pipeline_match_oracle() -> None:
    from tp_runtime import DecodePipeline, DecodeStepRunner

    lens0 = bench.make_lengths(0, 0)
    assert len(lens0) == 64 and min(lens0) >= 1024 and max(lens0) <= 8192
    steps_total = 1 + 3 + 3
    st = bench.build_state(lens0, steps_total + 1, 0, 0, DEVICE, bench.NUM_LAYERS, torch.float16)
    assert st["key_pools"].shape == (12, st["num_pages"], HKV, BS, D)
    assert st["num_pages"] >= int(bench.POOL_FACTOR * sum(lens0) / BS)
    tables = _host_tables(st["tables"])
    runner = DecodeStepRunner(st["key_pools"], st["value_pools"], st["tables"], st["lens0"].to(DEVICE),
                              num_q_heads=HQ)
    gen = torch.Generator(device=DEVICE).manual_seed(123)
    lens = list(lens0)
    checked_layers = iter([0, 5, 11, 3, 7, 9, 1])

    def fresh_inputs(q, k, v) -> None:
        for t in (q, k, v):
            t.copy_(torch.randn(t.shape, generator=gen, device=DEVICE, dtype=torch.float32).to(t.dtype))

    def check(query, key, value, out_layers, what: str) -> None:
        nonlocal lens
        _check_appended(runner.key_pools, runner.value_pools, key, value, tables, lens, what)
        lens = [n + 1 for n in lens]
        assert runner.seq_lens.cpu().tolist() == lens, what
        layer = next(checked_layers)
        expected = _oracle_layer(query[layer], runner.key_pools[layer], runner.value_pools[layer], tables, lens,
                                 "float16")
        got = lib.as_f32(lib.np_bits(out_layers[layer]), "float16")
        assert np.isfinite(got).all(), what
        lib.assert_close(got, expected, "float16", f"{what}, layer {layer}")
        assert runner.check_errors() == 0, what

    stream = torch.cuda.Stream(DEVICE)
    # (a) one eager step (also the library's one-time set-up before any capture)
    fresh_inputs(st["query"], st["key"], st["value"])
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        runner.step(st["query"], st["key"], st["value"], st["out"])
    torch.cuda.synchronize()
    check(st["query"], st["key"], st["value"], st["out"], "eager step")

    # (b) a CUDA graph of the step, replayed with new inputs each time
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            runner.step(st["query"], st["key"], st["value"], st["out"])
    torch.cuda.synchronize()
    assert runner.seq_lens.cpu().tolist() == lens  # capturing does not run the step
    for i in range(3):
        fresh_inputs(st["query"], st["key"], st["value"])
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize()
        check(st["query"], st["key"], st["value"], st["out"], f"graph replay {i}")
    del graph

    # (c) the public pipeline: pinned host inputs in, host outputs back, transfers overlapped
    pipe = DecodePipeline(runner, torch.float16)
    host_in, host_out = [], []
    for i in range(3):
        q = torch.empty(st["query"].shape, dtype=torch.float16, pin_memory=True)
        k = torch.empty(st["key"].shape, dtype=torch.float16, pin_memory=True)
        v = torch.empty(st["value"].shape, dtype=torch.float16, pin_memory=True)
        host_gen = torch.Generator().manual_seed(500 + i)
        for t in (q, k, v):
            t.copy_(torch.randn(t.shape, generator=host_gen).to(torch.float16))
        host_in.append((q, k, v))
        host_out.append(torch.full(st["out"].shape, float("nan"), dtype=torch.float16, pin_memory=True))
    for i in range(3):
        pipe.submit(*host_in[i], host_out[i])
    pipe.finish()
    # the three steps ran in order; check each one's appends and outputs from the host copies
    lens_at = [list(lens)]
    for _ in range(3):
        lens_at.append([n + 1 for n in lens_at[-1]])
    assert runner.seq_lens.cpu().tolist() == lens_at[3]
    for i in range(3):
        q, k, v = host_in[i]
        slots = [int(oracle.slot_mapping(t, n, 1, BS)[0]) for t, n in zip(tables, lens_at[i])]
        page = torch.tensor([s // BS for s in slots], device=DEVICE)
        off = torch.tensor([s % BS for s in slots], device=DEVICE)
        for layer in range(bench.NUM_LAYERS):
            assert torch.equal(runner.key_pools[layer][page, :, off, :].cpu().view(torch.int16),
                               k[layer].view(torch.int16)), ("pipeline", i, layer)
            assert torch.equal(runner.value_pools[layer][page, :, off, :].cpu().view(torch.int16),
                               v[layer].view(torch.int16)), ("pipeline", i, layer)
        layer = next(checked_layers)
        # step i read the pool as it was after its own append; later steps only add later slots
        expected = _oracle_layer(q[layer].to(DEVICE), runner.key_pools[layer], runner.value_pools[layer], tables,
                                 lens_at[i + 1], "float16")
        got = lib.as_f32(lib.np_bits(host_out[i][layer]), "float16")
        assert np.isfinite(got).all(), ("pipeline", i)
        lib.assert_close(got, expected, "float16", f"pipeline step {i}, layer {layer}")
    assert runner.check_errors() == 0


def test_config4_full_shape_every_request_matches_oracle() -> None:
    import paged_kv_ops as ops

    batch, length = 8, 131072
    pages = batch * length // BS
    gen = torch.Generator(device=DEVICE).manual_seed(41)
    key_pool = torch.randn((pages + 5, HKV, BS, D), generator=gen, device=DEVICE).bfloat16()
    value_pool = torch.randn((pages + 5, HKV, BS, D), generator=gen, device=DEVICE).bfloat16()
    perm = torch.randperm(pages + 5, generator=torch.Generator().manual_seed(41))[:pages]
    tables_dev = perm.view(batch, length // BS).to(torch.int32).to(DEVICE)
    query = torch.randn((batch, HQ, D), generator=gen, device=DEVICE).bfloat16()
    lens = torch.full((batch,), length, dtype=torch.int32, device=DEVICE)
    flag = ops.new_error_flag(DEVICE)
    auto = ops.paged_decode(query, key_pool, value_pool, tables_dev, lens, error_flag=flag)
    parts = ops.paged_decode(query, key_pool, value_pool, tables_dev, lens, pages_per_split=128, error_flag=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    expected = _oracle_layer(query, key_pool, value_pool, _host_tables(tables_dev), [length] * batch, "bfloat16")
    for name, out in (("automatic splits", auto), ("64 partitions", parts)):
        got = lib.as_f32(lib.np_bits(out), "bfloat16")
        assert np.isfinite(got).all(), name
        lib.assert_close(got, expected, "bfloat16", name)


def test_config5_full_shape_churn_keeps_pages_exact_and_decode_matches_oracle() -> None:
    import paged_kv_ops as ops
    from scheduler import KVBlockManager
    from tp_runtime import DecodeStepRunner

    layers, steps = 2, 5
    gen = torch.Generator().manual_seed(1077)
    rng = np.random.default_rng(1077)
    lengths0 = [bench.churn_length(gen) for _ in range(bench.CHURN_REQUESTS)]
    num_pages = int(1.6 * sum(lengths0) / BS) + bench.CHURN_REQUESTS * 8
    max_blocks = 32768 // BS + 8
    mgr = KVBlockManager(num_pages, BS, max_blocks)
    ids = [f"r{i}" for i in range(bench.CHURN_REQUESTS)]
    # host copy of every live request's tokens (layer 0; layer 1 stores the negation, exact in fp16)
    tokens_k: dict[str, np.ndarray] = {}
    tokens_v: dict[str, np.ndarray] = {}
    shape = (layers, num_pages, HKV, BS, D)
    key_pools = torch.zeros(shape, dtype=torch.float16, device=DEVICE)
    value_pools = torch.zeros_like(key_pools)

    def write_context(rid: str, n: int) -> None:
        k = rng.standard_normal((n, HKV, D), dtype=np.float32).astype(np.float16)
        v = rng.standard_normal((n, HKV, D), dtype=np.float32).astype(np.float16)
        tokens_k[rid], tokens_v[rid] = k, v
        slots = torch.tensor(mgr.slots(rid, 0, n), dtype=torch.int64, device=DEVICE)
        kd, vd = torch.from_numpy(k).to(DEVICE), torch.from_numpy(v).to(DEVICE)
        for layer in range(layers):
            sign = 1 if layer == 0 else -1
            ops.kv_append(sign * kd, sign * vd, slots, key_pools[layer], value_pools[layer])

    for rid, n in zip(ids, lengths0):
        mgr.add_request(rid, n)
        write_context(rid, n)
    runner = DecodeStepRunner(key_pools, value_pools,
                              torch.full((bench.CHURN_REQUESTS, max_blocks), -1, dtype=torch.int32, device=DEVICE),
                              torch.zeros(bench.CHURN_REQUESTS, dtype=torch.int32, device=DEVICE), num_q_heads=HQ)
    q = torch.empty((layers, bench.CHURN_REQUESTS, HQ, D), dtype=torch.float16, device=DEVICE)
    k_new = torch.empty((layers, bench.CHURN_REQUESTS, HKV, D), dtype=torch.float16, device=DEVICE)
    v_new = torch.empty_like(k_new)
    out = torch.empty_like(q)
    counter = bench.CHURN_REQUESTS
    copies_seen = []
    for step in range(steps):
        for i in range(bench.CHURN_REQUESTS):
            if float(torch.rand((), generator=gen)) < bench.CHURN_FINISH:
                mgr.free_request(ids[i])
                del tokens_k[ids[i]], tokens_v[ids[i]]
                ids[i] = f"r{counter}"
                counter += 1
                n = bench.churn_length(gen)
                mgr.add_request(ids[i], n, staging=True)
                write_context(ids[i], n)
        src, dst = mgr.compact(max_moves=bench.CHURN_MAX_COPIES)
        copies_seen.append(len(src))
        if src:
            ops.kv_copy_pages(key_pools, value_pools, torch.tensor(src, dtype=torch.int32, device=DEVICE),
                              torch.tensor(dst, dtype=torch.int32, device=DEVICE), error_flag=runner.error_flag)
        for rid in ids:  # a page for this step's decode token where a request fills its last one
            entry = mgr.requests[rid]
            if len(entry.pages) * BS <= entry.length:
                entry.pages.extend(mgr.allocator.allocate(1))
        tables = mgr.block_table_rows(ids)
        lens_before = mgr.lengths(ids)
        bt = torch.full((bench.CHURN_REQUESTS, max_blocks), -1, dtype=torch.int32)
        for b, row in enumerate(tables):
            bt[b, :len(row)] = torch.tensor(row, dtype=torch.int32)
        runner.block_tables.copy_(bt.to(DEVICE))
        runner.seq_lens.copy_(torch.tensor(lens_before, dtype=torch.int32, device=DEVICE))
        qh = rng.standard_normal((bench.CHURN_REQUESTS, HQ, D), dtype=np.float32).astype(np.float16)
        kh = rng.standard_normal((bench.CHURN_REQUESTS, HKV, D), dtype=np.float32).astype(np.float16)
        vh = rng.standard_normal((bench.CHURN_REQUESTS, HKV, D), dtype=np.float32).astype(np.float16)
        for layer in range(layers):
            sign = 1 if layer == 0 else -1
            q[layer].copy_(torch.from_numpy(qh))
            k_new[layer].copy_(sign * torch.from_numpy(kh))
            v_new[layer].copy_(sign * torch.from_numpy(vh))
        runner.step(q, k_new, v_new, out)
        torch.cuda.synchronize()
        for b, rid in enumerate(ids):
            tokens_k[rid] = np.concatenate([tokens_k[rid], kh[b:b + 1]])
            tokens_v[rid] = np.concatenate([tokens_v[rid], vh[b:b + 1]])
            mgr.requests[rid].length += 1
        lens = mgr.lengths(ids)
        assert lens == [n + 1 for n in lens_before]
        assert runner.seq_lens.cpu().tolist() == lens
        assert runner.check_errors() == 0, step
        # every request's pages hold exactly its tokens, in both layers
        for b, rid in enumerate(ids):
            n = lens[b]
            pages = (n + BS - 1) // BS
            idx = torch.tensor(tables[b][:pages], device=DEVICE)
            want_k = torch.from_numpy(tokens_k[rid]).to(DEVICE).transpose(0, 1)  # (hkv, n, d)
            want_v = torch.from_numpy(tokens_v[rid]).to(DEVICE).transpose(0, 1)
            for layer in range(layers):
                sign = 1 if layer == 0 else -1
                got_k = key_pools[layer][idx].transpose(0, 1).reshape(HKV, pages * BS, D)[:, :n]
                got_v = value_pools[layer][idx].transpose(0, 1).reshape(HKV, pages * BS, D)[:, :n]
                assert torch.equal(got_k.view(torch.int16), (sign * want_k).view(torch.int16)), (step, rid, layer)
                assert torch.equal(got_v.view(torch.int16), (sign * want_v).view(torch.int16)), (step, rid, layer)
        # every request of layer 0 against the oracle on the expected tokens (not the pools)
        qf = qh.astype(np.float32)
        group = HQ // HKV
        expected = np.zeros(qf.shape, dtype=np.float32)
        for b, rid in enumerate(ids):
            n = lens[b]
            pages = (n + BS - 1) // BS
            pk = np.zeros((pages * BS, HKV, D), dtype=np.float16)
            pv = np.zeros((pages * BS, HKV, D), dtype=np.float16)
            pk[:n], pv[:n] = tokens_k[rid], tokens_v[rid]
            pk = pk.reshape(pages, BS, HKV, D).transpose(0, 2, 1, 3)
            pv = pv.reshape(pages, BS, HKV, D).transpose(0, 2, 1, 3)
            for h in range(HKV):
                expected[b, h * group:(h + 1) * group] = oracle.decode_attention(
                    qf[b:b + 1, h * group:(h + 1) * group], pk[:, h:h + 1], pv[:, h:h + 1], [list(range(pages))],
                    [n], dtype="float16", round_probs=False)[0]
        got = lib.as_f32(lib.np_bits(out[0]), "float16")
        assert np.isfinite(got).all(), step
        lib.assert_close(got, expected, "float16", f"churn step {step}")
    # the copy lists have the benchmark's sizes: thousands of pages per step
    assert max(copies_seen[1:]) >= 1000, copies_seen
