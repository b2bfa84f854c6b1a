"""The reference arm of bench.py (`--impl reference`) on the CPU: the torch
restatement of the reference's fp32 step (oracle/torch_step.py), timed on the
host cores on a bounded sample, printed as one JSON line with the same metric,
unit and direction as the B200 arm plus its `cpu_baseline`, a full unscaled
step of the CPU benchmark configuration, and a zero-copy `e2e`. Shrunk here so
that it runs in seconds; the line's shape does not depend on the sizes."""
import argparse
import json

import pytest

import bench


def _shrink(monkeypatch):
    monkeypatch.setattr(bench, "D_IN", 64)
    monkeypatch.setattr(bench, "N_FEAT", 512)
    monkeypatch.setattr(bench, "TOKENS", 4096)
    monkeypatch.setattr(bench, "CPU_SAMPLE_TOKENS", 256)
    monkeypatch.setattr(bench, "CFG1", dict(d=32, F=256, tokens=512))


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
    # the value is the sample's own tokens over its own measured time
    assert line["ms_per_step"] == pytest.approx(256 / line["value"] * 1e3, rel=1e-9)
    assert line["config"]["sample_fraction_of_step"] == pytest.approx(256 / 4096)
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] == bench.host_threads()
    assert cb["value"] == line["value"] and cb["extrapolated"] is False
    assert "over 32 features" in cb["sample"]
    c1 = line["cfg1_full_step"]
    assert c1["tokens_per_s"] > 0 and c1["ms_per_step"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    _shrink(monkeypatch)
    monkeypatch.setenv("RANK", "1")
    assert bench.run_reference(argparse.Namespace(gpus=2, steps=2, warmup=1)) == 0
    assert capsys.readouterr().out == ""


def test_sampler_uses_every_host_thread_and_calibrates_l0(monkeypatch):
    """torchrun sets OMP_NUM_THREADS=1; the sampler sets torch's thread count
    to the process's whole affinity set anyway, and its thresholds put the
    mean L0 near the target."""
    import torch
    _shrink(monkeypatch)
    monkeypatch.setattr(bench, "K_TARGET", 16)
    torch.set_num_threads(1)
    s = bench.CpuReferenceSampler(sample_tokens=256)
    assert s.threads == bench.host_threads() == torch.get_num_threads()
    t, l0 = s.sample(0)
    assert t > 0
    assert 4 <= l0 <= 64
