"""bench.py's JSON contract on CPU: the reference arm's line (host cores, no
GPU) carries the same metric, unit and config as the GPU arm plus `impl`,
`cpu_baseline` (with the threads that actually ran) and a zero-copy `e2e`;
only rank 0 prints; the default workload is config 4; the roofline's traffic
figure is read from the committed ncu summary; the CPU sampler runs the
timed CPU implementation on a small config and selects what the oracle does."""
from __future__ import annotations

import argparse
import json

import bench
from sparse_decode.synth import CONFIGS, algorithmic_bytes


def _args(steps=2, warmup=1):
    return argparse.Namespace(gpus=1, steps=steps, warmup=warmup, impl="reference", config="c4", layers=None,
                              cpu_seconds=10.0, no_cpu_baseline=False)


def test_reference_arm_line(monkeypatch, capsys):
    calls = []

    def fake_time(w, inp, seconds, threads):
        calls.append(seconds)
        return 1234.5, 7, 3, None, None

    monkeypatch.setattr(bench, "cpu_inputs_generated", lambda w, seed: {"dummy": True})
    monkeypatch.setattr(bench, "cpu_time", fake_time)
    w = CONFIGS["c4"]
    bench.run_reference(_args(), w, 0, 1)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["impl"] == "reference" and line["higher_is_better"] is False
    assert line["value"] == 1234.5 and line["n_gpus"] == 1 and line["scaling"] == "strong"
    assert line["config"]["workload"] == w.name and line["config"]["context"] == w.T
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["cores"] == 3  # the threads that ran tasks, not the machine's count
    assert line["e2e"] == {"value": 1234.5, "unit": bench.UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert len(calls) == 3  # one warm-up and two timed samples


def test_reference_arm_other_ranks_print_nothing(monkeypatch, capsys):
    monkeypatch.setattr(bench, "cpu_inputs_generated", lambda *a: (_ for _ in ()).throw(AssertionError("rank 1 ran")))
    bench.run_reference(_args(), CONFIGS["c4"], 1, 2)
    assert capsys.readouterr().out == ""


def test_default_workload_is_config_4():
    import inspect
    src = inspect.getsource(bench.main)
    assert 'ap.add_argument("--config", default="c4")' in src


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


def test_cpu_time_reports_threads_and_matches_the_oracle(oracle_lib):
    import numpy as np

    import oracle
    w = CONFIGS["c2q8"].with_(name="c2q8_reduced_B1_T4096", B=1, T=4096)
    inp = bench.cpu_inputs_generated(w, 5)
    us, n, used, out, sel = bench.cpu_time(w, inp, 0.05, 2)
    assert n >= 1 and us > 0.0 and 1 <= used <= 2
    sc = oracle.scores(inp["q"], inp["dt"], inp["summ"], inp["dt"], w.B, w.Hq, w.Hkv, w.D, w.NB, 1 / np.sqrt(w.D))
    assert np.array_equal(sel, oracle.select(sc, w.K))
