"""The reference arm of bench.py (`--impl reference`) on the CPU: the oracle's
restatement of the reference fp32 step, timed on the host cores, printed as
one JSON line with the same metric, unit and direction as the B200 arm plus
its `cpu_baseline` and a zero-copy `e2e`. Shrunk to d=64, F=512 here so that
it runs in seconds; the line's shape does not depend on the sizes."""
import argparse
import json

import pytest

import bench


def _shrink(monkeypatch):
    monkeypatch.setattr(bench, "D_IN", 64)
    monkeypatch.setattr(bench, "N_FEAT", 512)
    monkeypatch.setattr(bench, "TOKENS", 4096)
    monkeypatch.setattr(bench, "_CPU_DICT", {})


def test_reference_arm_prints_the_contract_line(monkeypatch, capsys):
    _shrink(monkeypatch)
    monkeypatch.delenv("RANK", raising=False)
    assert bench.run_reference(argparse.Namespace(gpus=1, steps=2, warmup=1)) == 0
    out = capsys.readouterr().out.strip().splitlines()
    assert len(out) == 1
    line = json.loads(out[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["steps"] == 2 and line["warmup"] == 1
    assert line["value"] > 0
    assert line["ms_per_step"] == pytest.approx(bench.TOKENS / line["value"] * 1e3, rel=1e-9)
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert "32 of the 512 features" in cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    _shrink(monkeypatch)
    monkeypatch.setenv("RANK", "1")
    assert bench.run_reference(argparse.Namespace(gpus=2, steps=2, warmup=1)) == 0
    assert capsys.readouterr().out == ""


def test_sliced_optimizer_timing_scales_to_the_whole_parameter_count(monkeypatch):
    """opt_features times the clip norm and Adam on a feature slice; the
    returned time is scaled by P / P_slice (P = 2 F d + 2 F + d)."""
    _shrink(monkeypatch)
    calls = []
    real = bench.time.perf_counter
    ticks = iter(range(1000))

    def fake_clock():
        calls.append(1)
        return float(next(ticks))

    monkeypatch.setattr(bench.time, "perf_counter", fake_clock)
    t_mb, t_opt, l0 = bench.cpu_reference_step_time(256, seed=0, opt_features=32)
    monkeypatch.setattr(bench.time, "perf_counter", real)
    F, d, fs = 512, 64, 32
    assert t_mb == 1.0
    assert t_opt == (2 * F * d + 2 * F + d) / (2 * fs * d + 2 * fs + d)
    assert l0 >= 0
