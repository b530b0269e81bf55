"""CPU checks of the benchmark's contract with its evidence: the arguments it documents, the ncu summaries
it reads its DRAM-traffic figures from, and the capture commands those summaries quote."""

from __future__ import annotations

import importlib.util
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_defaults_are_the_headline_run() -> None:
    args = _bench().parse_args([])
    assert (args.workload, args.gpus, args.impl, args.tokens) == ("decode", 1, "ours", None)
    assert args.warmup >= 3 and args.steps > 0
    wide = _bench().parse_args(["--workload", "oproj", "--tokens", "8192", "--layers", "1"])
    assert (wide.tokens, wide.layers) == (8192, 1)


def test_every_traffic_figure_comes_from_a_committed_summary() -> None:
    bench = _bench()
    names = set(re.findall(r'profiled_traffic\("([^"]+)"\)', (ROOT / "bench.py").read_text()))
    assert names, "the benchmark reads no traffic figures"
    for name in sorted(names):
        assert (ROOT / "profiles" / name).is_file(), name
        value = bench.profiled_traffic(name)
        assert value is not None and value > 0, name


def test_quoted_ncu_commands_leave_the_clocks_alone() -> None:
    for path in sorted((ROOT / "profiles").glob("*.md")):
        text = path.read_text()
        for command in re.findall(r"^\s*ncu .*(?:\\\n.*)*", text, flags=re.M):
            assert "--clock-control none" in command, (path.name, command)


def test_secondary_figures_collect_each_workloads_line_and_keep_failures_local(monkeypatch) -> None:
    """The headline line's secondary figures: each workload runs with brief settings, its line is collected
    instead of printed, and a workload that fails is recorded without costing the others (or the line)."""
    bench = _bench()
    seen = []

    def fake(name, fail=False):
        def run(args, **_layout):
            seen.append((name, args.workload, args.steps, args.warmup, args.no_cpu_baseline))
            if fail:
                raise RuntimeError("no device")
            bench.emit({"metric": name, "value": 1.0, "unit": "GB/s", "roofline": {"frac": 0.5}, "extra": 1,
                        "clocks": {"sm_mhz": 1965.0, "reasons": []}, "config": {"workload": name}})
        return run

    for attr in ("run_prefill", "run_decode_fp8", "run_normrope", "run_attn_layer", "run_ours", "run_churn"):
        monkeypatch.setattr(bench, attr, fake(attr))
    monkeypatch.setattr(bench, "run_oproj", fake("run_oproj", fail=True))
    import torch

    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)
    args = bench.parse_args(["--steps", "20", "--warmup", "5"])
    out = bench.secondary_workloads(args, 1)
    assert set(out) == {"prefill", "decode_fp8", "normrope", "oproj", "attn_layer", "long", "churn"}
    assert out["oproj"] == {"error": "RuntimeError: no device"}
    assert out["prefill"]["value"] == 1.0 and "extra" not in out["prefill"]
    assert all(s[2] == 10 and s[3] == 3 and s[4] for s in seen)
    assert bench._COLLECT is None  # printing is restored afterwards
    four = bench.secondary_workloads(args, 4)
    assert set(four) == {"long", "churn", "oproj", "churn_tp"} and four["churn_tp"]["value"] == 1.0
    assert set(bench.secondary_workloads(args, 2)) == {"long", "churn", "oproj", "churn_tp", "prefill"}
    assert set(bench.secondary_workloads(args, 3)) == {"long", "churn", "oproj"}


def test_reference_arm_prints_the_contract_line(capsys, monkeypatch) -> None:
    """`bench.py --impl reference` (the reference's CPU composition on the host cores): one JSON line on the
    headline's metric, unit and direction, marked impl=reference, with its cpu_baseline description and an
    e2e figure equal to the value with no host-device copies. One timed step keeps this at a few seconds."""
    import json

    bench = _bench()
    monkeypatch.delenv("RANK", raising=False)
    assert bench.main(["--impl", "reference", "--steps", "1", "--warmup", "3"]) == 0
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 3 and line["value"] > 0
    assert line["cpu_baseline"]["kind"] in ("port", "reference") and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["sample"] and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only(capsys, monkeypatch) -> None:
    """Under torchrun the reference arm is timed by rank 0 alone; the other ranks exit 0 without a line."""
    bench = _bench()
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    assert bench.main(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"]) == 0
    assert not [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
