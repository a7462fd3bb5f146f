"""bench.py's JSON contract on CPU: the reference arm's line (host cores, no
GPU) carries the same metric, unit and config as the GPU arm plus `impl`,
`cpu_baseline` and a zero-copy `e2e`; only rank 0 prints; the roofline's
traffic figure is read from the committed ncu summary; the CPU sampler runs
the oracle's decode on a small config."""
from __future__ import annotations

import argparse
import json

import bench
from sparse_decode.synth import CONFIGS, algorithmic_bytes


def _args(steps=2, warmup=1):
    return argparse.Namespace(gpus=1, steps=steps, warmup=warmup, impl="reference", config="c1", layers=None,
                              cpu_seconds=10.0, no_cpu_baseline=False)


def test_reference_arm_line(monkeypatch, capsys):
    calls = []

    def fake_sample(w, seconds, threads):
        calls.append(seconds)
        return 1234.5, 7

    monkeypatch.setattr(bench, "cpu_sample", fake_sample)
    w = CONFIGS["c1"]
    bench.run_reference(_args(), w, 0, 1)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["impl"] == "reference" and line["higher_is_better"] is False
    assert line["value"] == 1234.5 and line["n_gpus"] == 1 and line["scaling"] == "weak"
    assert line["config"]["workload"] == w.name and line["config"]["context"] == w.T
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": 1234.5, "unit": bench.UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert len(calls) == 3  # one warm-up and two timed samples


def test_reference_arm_other_ranks_print_nothing(monkeypatch, capsys):
    monkeypatch.setattr(bench, "cpu_sample", lambda *a: (_ for _ in ()).throw(AssertionError("rank 1 ran")))
    bench.run_reference(_args(), CONFIGS["c1"], 1, 2)
    assert capsys.readouterr().out == ""


def test_traffic_comes_from_the_committed_summary():
    w = CONFIGS["c1"]
    t = bench._traffic("decode_kernel", w.name)
    assert t is not None
    # the measured DRAM bytes of a launch match the algorithmic bytes within a few percent
    assert 1.0 <= t / algorithmic_bytes(w) < 1.05
    assert bench._traffic("decode_kernel", "no_such_workload") is None


def test_cpu_sample_runs_the_oracle(oracle_lib):
    us, n = bench.cpu_sample(CONFIGS["c0"], 0.05, 2)
    assert n >= 1 and us > 0.0
