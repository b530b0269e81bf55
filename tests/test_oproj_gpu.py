"""GPU parity of the attention output stage (gate, FP8 block-scaled o_proj, tensor-parallel all-reduce)
against the reference's fixtures (tests/golden: src/tp_runtime.py:672-695 run per rank) and the oracle.

Tensor-parallel groups run here as ``OutputExchange.local_group``: every rank's buffers on one GPU
and the ranks' kernels one after another on one stream, phase 1 (gate, project, push) of every rank
before phase 2 (finish) of any, so no kernel ever waits for one that has not run. The real
multi-process, multi-GPU group is tests/test_oproj_multigpu.py.

The tensor cores take 16-bit activations as f16 (exact) and fp32 activations as two f16 parts
(within 2^-22): outputs are compared with the exact oracle at the path's tolerance, plus -- for
more than one rank -- one unit of each rank's rounded partial (partial_rounding_bound), and almost
all of them are bit-identical to the reference's fixtures."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
import pkv_testlib as lib
from oracle import paged_kv_oracle as oracle

pytestmark = pytest.mark.gpu
DEVICE = "cuda:0"


def _ops():
    import paged_kv_ops

    return paged_kv_ops


def _out_f32(t: torch.Tensor) -> np.ndarray:
    return lib.as_f32(lib.np_bits(t.reshape(-1, t.shape[-1])), cases.dtype_name(t.dtype))


def _run_group(ops, inputs, world, hidden, out_dtype, exchanges=None, error_flag=None):
    """inputs[r] = (heads, gate, weight, scale) on the device; returns every rank's output."""
    own = exchanges is None
    if own:
        heads = inputs[0][0]
        capacity = max(256, heads.shape[0] * heads.shape[2])  # tokens = batch x seq_len
        exchanges = ops.OutputExchange.local_group(world, capacity, hidden, out_dtype, DEVICE) if world > 1 else [None]
    outs = []
    for r in range(world):
        h, g, w, s = inputs[r]
        outs.append(ops.gated_o_proj(h, g, w, s, out_dtype=out_dtype, exchange=exchanges[r],
                                     phases=1 if world > 1 else 3, error_flag=error_flag))
    if world > 1:
        for r in range(world):
            h, g, w, s = inputs[r]
            ops.gated_o_proj(h, g, w, s, out_dtype=out_dtype, exchange=exchanges[r], out=outs[r], phases=2,
                             error_flag=error_flag)
    torch.cuda.synchronize()
    if own and world > 1:
        for e in exchanges:
            e.close()
    return outs


def _to_dev(case, rank):
    return tuple(t.contiguous().to(DEVICE) for t in case.rank_inputs(rank))


@pytest.mark.parametrize("make", cases.OPROJ_CASES, ids=lambda m: m.__name__)
def test_output_stage_matches_reference_fixtures(make) -> None:
    ops = _ops()
    case = make()
    name = case.name
    od = cases.dtype_name(case.hidden_dtype)
    g = lib.golden()
    inputs = [_to_dev(case, r) for r in range(case.world_size)]
    flag = ops.new_error_flag(DEVICE)
    # each rank alone (no exchange) gives the reference's all-reduce input
    for r in range(case.world_size):
        part = ops.gated_o_proj(*inputs[r], out_dtype=case.hidden_dtype, error_flag=flag)
        ref = oracle.to_f32(g[f"{name}/partial{r}"], od)
        got = _out_f32(part)
        lib.assert_close(got, ref, od, f"{name} partial {r}")
        assert float((got == ref).mean()) >= 0.97
    outs = _run_group(ops, inputs, case.world_size, case.hidden, case.hidden_dtype, error_flag=flag)
    assert int(flag.item()) == 0
    ref = oracle.to_f32(g[f"{name}/out"], od)
    bound = lib.partial_rounding_bound([oracle.to_f32(g[f"{name}/partial{r}"], od) for r in range(case.world_size)], od)
    for r, o in enumerate(outs):
        assert tuple(o.shape) == (case.heads.shape[0], case.heads.shape[2], case.hidden)
        got = _out_f32(o)
        lib.assert_close(got, ref, od, f"{name} rank {r}", extra=bound)
        assert float((got == ref).mean()) >= 0.97
        np.testing.assert_array_equal(lib.np_bits(o), lib.np_bits(outs[0]))  # every rank holds the same sum


def _random_inputs(gen, tokens, num_heads, head_dim, hidden, hd, gd, world, seq_len=1):
    batch = tokens // seq_len
    k = num_heads * head_dim
    heads = torch.randn((batch, num_heads, seq_len, head_dim), generator=gen).to(hd)
    gate = (2 * torch.randn((batch, seq_len, k), generator=gen)).to(gd)
    weight = (0.05 * torch.randn((hidden, k), generator=gen)).to(torch.float8_e4m3fn)
    scale = (0.5 + torch.rand((hidden // 128, k // 128), generator=gen)).to(torch.bfloat16)
    return cases.OProjCase("random", heads, gate, weight, scale, torch.bfloat16, world)


def test_output_stage_many_positions_per_request() -> None:
    """A prefill-sized call with several positions per request (heads (batch, H, seq_len, D)): the gating
    kernel splits each token index into (request, position)."""
    ops = _ops()
    gen = torch.Generator().manual_seed(77)
    case = _random_inputs(gen, 2 * 601, 4, 128, 256, torch.bfloat16, torch.bfloat16, 1, seq_len=601)
    (out,) = _run_group(ops, [_to_dev(case, 0)], 1, 256, torch.bfloat16)
    assert tuple(out.shape) == (2, 601, 256)
    exp, bound = _oracle_out(case, "bfloat16")
    lib.assert_close(_out_f32(out), exp, "bfloat16", "many positions", extra=bound)


def _oracle_out(case, out_dtype: str) -> tuple[np.ndarray, np.ndarray | float]:
    """The oracle's all-reduced output and the partial-rounding bound of its ranks."""
    parts = []
    for r in range(case.world_size):
        h, hd, gt, gd, codes, scale = lib.oproj_rank_arrays(case, r)
        x, _ = oracle.gate_heads(h, gt, hd, gd)
        parts.append(oracle.o_proj_partial(x, codes, scale, out_dtype))
    return oracle.all_reduce_sum(parts, out_dtype), lib.partial_rounding_bound(parts, out_dtype)


@pytest.mark.parametrize(
    "tokens,num_heads,head_dim,hidden,hd,gd,od,world",
    [
        (64, 16, 256, 2048, torch.bfloat16, torch.bfloat16, torch.bfloat16, 1),  # the decode step, one rank
        (64, 16, 256, 2048, torch.bfloat16, torch.bfloat16, torch.bfloat16, 2),  # ... TP=2
        (1, 2, 64, 128, torch.float32, torch.float32, torch.float32, 1),         # one block, split 1
        (100, 6, 64, 256, torch.float16, torch.float32, torch.float16, 1),       # 3 blocks -> split 3; two token chunks
        (200, 10, 64, 384, torch.float32, torch.bfloat16, torch.bfloat16, 1),    # 5 blocks -> split 5; 4 token chunks
        (7, 32, 256, 256, torch.bfloat16, torch.bfloat16, torch.float32, 1),     # 64 blocks: 8 per CTA, stage refills
        (4803, 8, 128, 256, torch.bfloat16, torch.bfloat16, torch.bfloat16, 1),  # 76 tiles: split 1, no sums
        (33, 16, 128, 384, torch.float16, torch.float16, torch.float16, 4),      # TP=4
        (300, 16, 128, 256, torch.bfloat16, torch.bfloat16, torch.bfloat16, 2),  # TP=2, 128-token tiles, split 8
    ],
)
def test_output_stage_matches_oracle(tokens, num_heads, head_dim, hidden, hd, gd, od, world) -> None:
    ops = _ops()
    gen = torch.Generator().manual_seed(tokens * 7 + hidden + world)
    case = _random_inputs(gen, tokens, num_heads, head_dim, hidden, hd, gd, world)
    outs = _run_group(ops, [_to_dev(case, r) for r in range(world)], world, hidden, od)
    name = cases.dtype_name(od)
    exp, bound = _oracle_out(case, name)
    for o in outs:
        got = _out_f32(o)
        assert np.isfinite(got).all()
        lib.assert_close(got, exp, name, f"rank output ({name})", extra=bound)
        np.testing.assert_array_equal(lib.np_bits(o), lib.np_bits(outs[0]))


def test_prefill_chunk_with_strided_heads() -> None:
    """Heads as the attention kernels leave them ((B, H, S, D) views of a (B, S, H, D) buffer) and a
    gate slice of a wider projection output."""
    ops = _ops()
    gen = torch.Generator().manual_seed(5)
    b, s, h, d, hidden = 2, 45, 4, 128, 256
    base = torch.randn((b, s, h, d), generator=gen).to(torch.bfloat16).to(DEVICE)
    heads = base.permute(0, 2, 1, 3)  # strides (S*H*D, D, H*D, 1)
    wide = (2 * torch.randn((b, s, 2 * h * d), generator=gen)).to(torch.bfloat16).to(DEVICE)
    gate = wide[..., h * d :]
    weight = (0.05 * torch.randn((hidden, h * d), generator=gen)).to(torch.float8_e4m3fn).to(DEVICE)
    scale = (0.5 + torch.rand((hidden // 128, h * d // 128), generator=gen)).to(torch.bfloat16).to(DEVICE)
    out = ops.gated_o_proj(heads, gate, weight, scale, out_dtype=torch.bfloat16)
    case = cases.OProjCase("strided", heads.cpu(), gate.cpu(), weight.cpu(), scale.cpu(), torch.bfloat16, 1)
    lib.assert_close(_out_f32(out), _oracle_out(case, "bfloat16")[0], "bfloat16", "strided heads")


def test_repeated_calls_advance_the_exchange() -> None:
    """Five calls of a 4-rank group on the same buffers (epochs 1..5, both buffer parities), new
    inputs each time; every result is the oracle's sum and no wait ran out."""
    ops = _ops()
    world, hidden = 4, 256
    exchanges = ops.OutputExchange.local_group(world, 64, hidden, torch.bfloat16, DEVICE)
    flag = ops.new_error_flag(DEVICE)
    try:
        for call in range(5):
            gen = torch.Generator().manual_seed(100 + call)
            case = _random_inputs(gen, 16 + call, 8, 64, hidden, torch.bfloat16, torch.bfloat16, world)
            outs = _run_group(ops, [_to_dev(case, r) for r in range(world)], world, hidden, torch.bfloat16,
                              exchanges=exchanges, error_flag=flag)
            exp, bound = _oracle_out(case, "bfloat16")
            for o in outs:
                lib.assert_close(_out_f32(o), exp, "bfloat16", f"call {call}", extra=bound)
        assert int(flag.item()) == 0
    finally:
        for e in exchanges:
            e.close()


def test_group_step_replays_as_a_cuda_graph() -> None:
    """Both ranks' phases of a 2-rank group captured once and replayed with new inputs copied into the
    captured tensors: the exchange epoch lives on the device, so every replay is a new call."""
    ops = _ops()
    world, hidden, tokens = 2, 256, 24
    exchanges = ops.OutputExchange.local_group(world, tokens, hidden, torch.bfloat16, DEVICE)
    gen = torch.Generator().manual_seed(9)
    case = _random_inputs(gen, tokens, 8, 64, hidden, torch.bfloat16, torch.bfloat16, world)
    static = [_to_dev(case, r) for r in range(world)]
    outs = [torch.empty((tokens, 1, hidden), dtype=torch.bfloat16, device=DEVICE) for _ in range(world)]
    works = [torch.empty(ops.o_proj_workspace_size(tokens, 256, hidden), dtype=torch.uint8, device=DEVICE) for _ in range(world)]
    flag = ops.new_error_flag(DEVICE)

    def step():
        for phase in (1, 2):
            for r in range(world):
                ops.gated_o_proj(*static[r], out_dtype=torch.bfloat16, exchange=exchanges[r], out=outs[r],
                                 workspace=works[r], phases=phase, error_flag=flag)

    try:
        stream = torch.cuda.Stream(DEVICE)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            step()  # warm-up: one real call (epoch 1)
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for rep in range(3):
            gen = torch.Generator().manual_seed(20 + rep)
            new = _random_inputs(gen, tokens, 8, 64, hidden, torch.bfloat16, torch.bfloat16, world)
            for r in range(world):
                for dst, src in zip(static[r], new.rank_inputs(r)):
                    dst.copy_(src)
            graph.replay()
            torch.cuda.synchronize()
            exp, bound = _oracle_out(new, "bfloat16")
            for o in outs:
                lib.assert_close(_out_f32(o), exp, "bfloat16", f"replay {rep}", extra=bound)
        assert int(flag.item()) == 0
        del graph
    finally:
        for e in exchanges:
            e.close()


def test_output_stage_rejects_unsupported_shapes() -> None:
    ops = _ops()
    heads = torch.zeros((2, 3, 1, 32), dtype=torch.bfloat16, device=DEVICE)  # K = 96
    gate = torch.zeros((2, 1, 96), dtype=torch.bfloat16, device=DEVICE)
    weight = torch.zeros((128, 96), dtype=torch.uint8, device=DEVICE)
    scale = torch.ones((1, 1), dtype=torch.bfloat16, device=DEVICE)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        ops.gated_o_proj(heads, gate, weight, scale)
    heads = torch.zeros((2, 4, 1, 32), dtype=torch.bfloat16, device=DEVICE)
    gate = torch.zeros((2, 1, 128), dtype=torch.bfloat16, device=DEVICE)
    with pytest.raises(RuntimeError, match="scale_inv"):
        ops.gated_o_proj(heads, gate, torch.zeros((128, 128), dtype=torch.uint8, device=DEVICE),
                         torch.ones((2, 1), dtype=torch.bfloat16, device=DEVICE))
    with pytest.raises(RuntimeError, match="hidden must be a positive multiple of 128"):
        ops.gated_o_proj(heads, gate, torch.zeros((192, 128), dtype=torch.uint8, device=DEVICE),
                         torch.ones((2, 1), dtype=torch.bfloat16, device=DEVICE))


def test_missing_peer_ends_the_wait_with_an_error() -> None:
    """Rank 1 of a 2-rank group never runs: rank 0's finishing kernel waits for exchange words that nothing
    writes, gives up after its bounded wait (2 s), reports PKV_DEVERR_WAIT_TIMEOUT and writes its own partial;
    the context stays usable (the next call on fresh buffers is correct)."""
    ops = _ops()
    world, hidden, tokens = 2, 256, 8
    gen = torch.Generator().manual_seed(77)
    case = _random_inputs(gen, tokens, 4, 64, hidden, torch.bfloat16, torch.bfloat16, world)
    inputs = [_to_dev(case, r) for r in range(world)]
    exchanges = ops.OutputExchange.local_group(world, tokens, hidden, torch.bfloat16, DEVICE)
    flag = ops.new_error_flag(DEVICE)
    try:
        out = ops.gated_o_proj(*inputs[0], out_dtype=torch.bfloat16, exchange=exchanges[0], error_flag=flag)
        torch.cuda.synchronize()
        assert int(flag.item()) & ops.DEVERR_WAIT_TIMEOUT
        alone = ops.gated_o_proj(*inputs[0], out_dtype=torch.bfloat16)  # rank 0's partial
        np.testing.assert_array_equal(lib.np_bits(out), lib.np_bits(alone))
    finally:
        for e in exchanges:
            e.close()
    outs = _run_group(ops, inputs, world, hidden, torch.bfloat16)
    exp, bound = _oracle_out(case, "bfloat16")
    lib.assert_close(_out_f32(outs[0]), exp, "bfloat16", "after the timeout", extra=bound)


def test_output_stage_chained_behind_each_layers_decode_is_bit_identical() -> None:
    """The decode step with every layer's output stage launched chained behind that layer's decode
    (PKV_OPROJ_CHAINED, as bench.py's attn_layer workload runs it, in a CUDA graph) gives what the same
    stages give launched plainly after the whole step: the attention bit for bit, the projection up to the
    order in which the split-k partials' float additions land (at most one unit in the last place)."""
    ops = _ops()
    from tp_runtime import DecodeStepRunner, finish_from_heads

    gen = torch.Generator().manual_seed(808)
    layers, hq, hkv, d, bs, hidden = 3, 16, 2, 256, 16, 2048
    lens = [40, 700, 1, 2049, 333]
    need = [(n + 2 + bs - 1) // bs for n in lens]
    pages = sum(need) + 5
    perm = torch.randperm(pages, generator=gen).tolist()
    tables = torch.full((len(lens), max(need)), -1, dtype=torch.int32)
    used = 0
    for b, n in enumerate(need):
        tables[b, :n] = torch.tensor(perm[used:used + n], dtype=torch.int32)
        used += n
    pools = [torch.randn((layers, pages, hkv, bs, d), generator=gen).to(torch.float16).to(DEVICE) for _ in range(2)]
    q = torch.randn((layers, len(lens), hq, d), generator=gen).to(torch.float16).to(DEVICE)
    k = torch.randn((layers, len(lens), hkv, d), generator=gen).to(torch.float16).to(DEVICE)
    v = torch.randn((layers, len(lens), hkv, d), generator=gen).to(torch.float16).to(DEVICE)
    gate = (2 * torch.randn((layers, len(lens), hq * d), generator=gen)).to(torch.float16).to(DEVICE)
    weight = (0.05 * torch.randn((layers, hidden, hq * d), generator=gen)).to(torch.float8_e4m3fn).to(DEVICE)
    scale = (0.5 + torch.rand((layers, hidden // 128, hq * d // 128), generator=gen)).to(torch.bfloat16).to(DEVICE)
    results = []
    for chained in (True, False):
        kp, vp = pools[0].clone(), pools[1].clone()
        runner = DecodeStepRunner(kp, vp, tables.to(DEVICE), torch.tensor(lens, dtype=torch.int32, device=DEVICE),
                                  num_q_heads=hq)
        out = torch.empty_like(q)
        hid = torch.empty((layers, len(lens), hidden), dtype=torch.float16, device=DEVICE)
        work = torch.empty(ops.o_proj_workspace_size(len(lens), hq * d, hidden), dtype=torch.uint8, device=DEVICE)

        def stage(layer: int) -> None:
            finish_from_heads(out[layer], gate[layer], weight[layer], scale[layer], torch.float16, out=hid[layer],
                              workspace=work, error_flag=runner.error_flag, chained=True)

        stream = torch.cuda.Stream(DEVICE)
        if chained:
            with torch.cuda.stream(stream):  # one eager step for the one-time set-up, then a graph step
                runner.step(q, k, v, out, after_layer=stage)
            torch.cuda.synchronize()
            runner.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32, device=DEVICE))
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(graph, stream=stream):
                    runner.step(q, k, v, out, after_layer=stage)
            with torch.cuda.stream(stream):
                graph.replay()
        else:
            with torch.cuda.stream(stream):
                runner.step(q, k, v, out)
                for layer in range(layers):
                    finish_from_heads(out[layer], gate[layer], weight[layer], scale[layer], torch.float16,
                                      out=hid[layer], workspace=work, error_flag=runner.error_flag)
        torch.cuda.synchronize()
        assert runner.check_errors() == 0
        results.append((lib.np_bits(out), lib.np_bits(hid)))
    np.testing.assert_array_equal(results[0][0], results[1][0])
    lib.assert_ulp_close(lib.as_f32(results[0][1], "float16"), lib.as_f32(results[1][1], "float16"), "float16",
                         "chained vs plain output stage", max_ulp=1, min_exact=0.99)
