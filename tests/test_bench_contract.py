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
