"""Telemetry recorder under a simulated clock (the reference's
``tests/test_metrics.py``): window summaries at the interval, TTFT/TBT
percentiles and SLO attainment, GPU time by step kind (mixed steps split by
tokens), decode-run folding in the live step feed, and the files written."""

import csv
import gzip
import json
import os
from types import SimpleNamespace

import pytest

from deltaserve_vllm_b200.engine.ft.estimator import StepFeatures
from deltaserve_vllm_b200.utils import metrics as metrics_mod
from deltaserve_vllm_b200.utils.metrics import MetricsRecorder


class FakeClock:
    def __init__(self, t=1000.0):
        self.t = t

    def time(self):
        return self.t


def _engine():
    return SimpleNamespace(ftcfg=SimpleNamespace(ttft_slo=0.5, avg_tbt_slo=0.06), step_listeners=[],
                           request_listeners=[], backward_listeners=[])


def _req(i, ttft, gaps, is_ft=False):
    return SimpleNamespace(is_ft=is_ft, request_id=f"r{i}", adapter=None, num_prompt=10,
                           output_ids=[0] * (len(gaps) + 1), arrival_time=0.0,
                           finish_time=ttft + sum(gaps), ttft=lambda: ttft, tbts=lambda: list(gaps))


def _step(eng, dur, **f):
    rec = SimpleNamespace(features=StepFeatures(**f), predicted=dur * 1.1)
    for cb in eng.step_listeners:
        cb(rec, dur)


def test_window_summary_and_files(tmp_path, monkeypatch):
    clock = FakeClock()
    monkeypatch.setattr(metrics_mod, "time", clock)
    eng = _engine()
    d = str(tmp_path / "m")
    rec = MetricsRecorder(eng, d, interval_s=10.0)
    # inference prefill, a mixed step (100 of 400 prefill tokens are FT), an FT-only step
    _step(eng, 0.020, t_in=300.0, p=2, prefill_lens=[150, 150])
    _step(eng, 0.040, t_in=400.0, p=3, t_ft=100.0, prefill_lens=[150, 150, 100])
    _step(eng, 0.030, t_in=256.0, p=1, t_ft=256.0, prefill_lens=[256])
    for _ in range(5):                      # a decode-only run folds into one feed entry
        _step(eng, 0.010, b_d=4, k=600.0)
    assert len(rec.steps) == 4 and rec.steps[-1]["n"] == 5
    assert rec.steps[-1]["gpu_ms"] == pytest.approx(50.0)
    # requests: 3 within SLO, 1 TTFT miss, 1 TBT miss; FT requests are not counted
    for i, (ttft, gaps) in enumerate([(0.1, [0.02, 0.03]), (0.2, [0.05]), (0.3, []),
                                      (0.9, [0.01]), (0.1, [0.08, 0.09])]):
        for cb in eng.request_listeners:
            cb("finish", _req(i, ttft, gaps))
    for cb in eng.request_listeners:
        cb("finish", _req(99, 0.01, [], is_ft=True))
    for cb in eng.backward_listeners:
        cb(SimpleNamespace(gpu_ms=12.5, n_tokens=512, loss=2.5, wall_ms=14.0))

    w = rec.window_summary()
    assert w["requests"] == 5 and w["slo_attainment"] == pytest.approx(3 / 5)
    assert w["fwd_gpu_s"]["inference"] == pytest.approx(0.020 + 0.050)
    assert w["fwd_gpu_s"]["mixed"] == pytest.approx(0.040)
    assert w["fwd_gpu_s"]["mixed_ft_share"] == pytest.approx(0.040 * 100 / 400)
    assert w["fwd_gpu_s"]["ft_only"] == pytest.approx(0.030)
    assert w["bwd_gpu_s"] == pytest.approx(0.0125)
    assert w["ttft_p50_s"] == pytest.approx(0.2)
    assert rec.totals["inf_tokens"] == 300 + 300 + 5 * 4 and rec.totals["ft_tokens"] == 356
    assert rec.last_summary is None

    clock.t += 10.5                         # the next step closes the window
    _step(eng, 0.010, b_d=2, k=100.0)
    s = rec.last_summary
    assert s is not None and s["window_s"] == pytest.approx(10.5)
    assert s["inf_tok_s"] == pytest.approx((620 + 2) / 10.5)
    assert s["ft_tok_s"] == pytest.approx(356 / 10.5)
    assert rec.window_summary()["requests"] == 0       # fresh window
    assert len(rec.series) == 1
    assert [x["seq"] for x in rec.data(steps_since=3)["steps"]] == [4, 9]

    rec.close()
    rows = list(csv.reader(open(os.path.join(d, "requests.csv"))))
    assert rows[0][0] == "finish_time" and len(rows) == 1 + 5
    bwd = list(csv.reader(open(os.path.join(d, "backward.csv"))))
    assert len(bwd) == 2 and float(bwd[1][4]) == 12.5
    lines = open(os.path.join(d, "summary.jsonl")).read().splitlines()
    assert len(lines) == 1 and json.loads(lines[0])["requests"] == 5
    seg = [f for f in os.listdir(d) if f.startswith("steps.")]
    assert seg
    with gzip.open(os.path.join(d, seg[0]), "rt") as f:
        logged = [json.loads(x) for x in f]
    assert len(logged) == 3 + 5 + 1 and logged[0]["kind"] == "inference"
    assert [x["kind"] for x in logged[:3]] == ["inference", "mixed", "ft_only"]


def test_recorder_without_directory_and_inactive(monkeypatch):
    monkeypatch.setattr(metrics_mod, "time", FakeClock())
    eng = _engine()
    rec = MetricsRecorder(eng, None)
    _step(eng, 0.01, b_d=1, k=10.0)
    assert rec.totals["inf_tokens"] == 1
    rec.close()
    _step(eng, 0.01, b_d=1, k=10.0)         # closed: hooks are no-ops
    assert rec.totals["inf_tokens"] == 1
