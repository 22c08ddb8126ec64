"""The JSON line of ``bench.py --impl reference`` (the CPU arm), on a shrunken workload.

The reference arm times the numpy restatement of the draft round on the host
cores.  Here the module's workload constants are replaced by a tiny geometry so
that the whole arm (set-up, warm-up rounds, timed rounds, JSON line) runs in
seconds without a GPU.
"""

from __future__ import annotations

import argparse
import json
import math
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

TINY = dict(hidden=64, intermediate=128, heads=4, kv_heads=2, head_dim=16, layers=2, slots=4, taps=2,
            window=64, epsilon=1e-6, theta=1e4)


@pytest.fixture
def bench(monkeypatch):
    import bench as module

    monkeypatch.setattr(module, "GEOMETRY", dict(TINY))
    monkeypatch.setattr(module, "VOCAB", 101)
    monkeypatch.setattr(module, "CONTEXT", 24)
    monkeypatch.setattr(module, "SLOTS", 4)
    monkeypatch.setattr(module, "INGEST", 4)
    return module


def _args(steps: int, warmup: int) -> argparse.Namespace:
    return argparse.Namespace(steps=steps, warmup=warmup, impl="reference", gpus=1, no_cpu=False)


def test_reference_arm_prints_one_contract_line(bench, capsys):
    bench.reference_arm(_args(steps=2, warmup=3), rank=0, world=1)
    lines = [line for line in capsys.readouterr().out.splitlines() if line.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["higher_is_better"] is True and line["scaling"] == "weak"
    assert line["n_gpus"] == 1 and 1 <= line["steps"] <= 2 and line["warmup"] >= 3
    assert math.isfinite(line["value"]) and line["value"] > 0
    # rate and per-round time describe the same measurement: (slots - 1) tokens per round
    assert line["value"] == pytest.approx((bench.SLOTS - 1) / (line["ms_per_step"] * 1e-3), rel=1e-9)
    assert line["config"]["workload"]
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["value"] == line["value"] and base["unit"] == line["unit"]
    assert base["cores"] >= 1 and "round" in base["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_runs_on_rank_zero_only(bench, capsys):
    bench.reference_arm(_args(steps=2, warmup=3), rank=1, world=2)
    assert capsys.readouterr().out == ""


def test_cpu_round_rate_stops_at_its_budget(bench):
    tensors, vocabulary, features, tokens = bench.make_tensors(seed=1)
    rate, per_round, rounds = bench.cpu_round_rate(tensors, vocabulary, features, tokens, steps=50, budget_s=0.0)
    assert rounds == 1 and per_round > 0 and rate == pytest.approx((bench.SLOTS - 1) / per_round)
