"""Step-time estimator, launch profiling shapes and the step trace on CPU.

Synthetic step durations are generated from known per-regime coefficients; a
fit must recover them, route each step to its regime (with the documented
fallbacks), refit only on the cadence, and apply each margin mode as stated
(the reference's checks: ``tests/test_merged_estimator.py``,
``tests/test_profiling_shapes.py``, ``tests/test_step_trace.py``).
"""

import csv
import os
from types import SimpleNamespace

import numpy as np
import pytest

from deltaserve_vllm_b200.engine.ft import estimator as est_mod
from deltaserve_vllm_b200.engine.ft.estimator import (MIN_FIT_SAMPLES, REFIT_EVERY, REGIME_DECODE_BWD,
                                                      REGIME_DECODE_ONLY, REGIME_EAGER, REGIME_FT_MIXED,
                                                      REGIME_INF_PREFILL, MergedExecutionEstimator,
                                                      StepFeatures, StepLog)
from deltaserve_vllm_b200.engine.profiling import ProfilingShapeGenerator
from deltaserve_vllm_b200.utils.step_trace import COLUMNS, StepTraceWriter, attach_step_trace

TRUE = {
    REGIME_INF_PREFILL: dict(alpha=2e-9, beta=3e-6, gamma=0.0, delta=4e-5, epsilon=1e-8, c=4e-3),
    REGIME_EAGER: dict(alpha=3e-9, beta=2.5e-6, gamma=6e-6, delta=5e-5, epsilon=2e-8, c=5e-3),
    REGIME_FT_MIXED: dict(alpha=1e-9, beta=2e-6, gamma=9e-6, delta=7e-5, epsilon=3e-8, c=6e-3),
    REGIME_DECODE_ONLY: dict(alpha=0.0, beta=0.0, gamma=0.0, delta=6e-5, epsilon=1.5e-8, c=7e-3),
    REGIME_DECODE_BWD: dict(alpha=0.0, beta=0.0, gamma=0.0, delta=9e-5, epsilon=2.5e-8, c=9e-3),
}


def _t(f: StepFeatures, regime: str) -> float:
    p = TRUE[regime]
    return (p["alpha"] * f.s + p["beta"] * f.t_in + p["gamma"] * f.t_ft + p["delta"] * f.b_d
            + p["epsilon"] * f.k + p["c"])


def _sample(rng, regime: str) -> StepFeatures:
    b_d = int(rng.integers(0, 64))
    k = float(b_d * rng.integers(64, 2048))
    if regime in (REGIME_DECODE_ONLY, REGIME_DECODE_BWD):
        b_d = max(1, b_d)
        return StepFeatures(b_d=b_d, k=float(b_d * rng.integers(64, 2048)), bwd=regime == REGIME_DECODE_BWD)
    lens = [int(x) for x in rng.integers(16, 1024, size=int(rng.integers(1, 6)))]
    if regime == REGIME_INF_PREFILL:
        return StepFeatures(t_in=float(sum(lens)), p=len(lens), b_d=b_d, k=k, prefill_lens=lens)
    ft = [int(x) for x in rng.integers(64, 512, size=int(rng.integers(1, 4)))]
    if regime == REGIME_EAGER:          # FT-only steps: no inference prefill, no decode
        return StepFeatures(t_in=float(sum(ft)), p=len(ft), t_ft=float(sum(ft)), prefill_lens=ft)
    # ft_mixed: FT rows next to inference prefill and decode
    allp = lens + ft
    return StepFeatures(t_in=float(sum(allp)), p=len(allp), t_ft=float(sum(ft)), b_d=b_d, k=k,
                        prefill_lens=allp)


@pytest.fixture
def split_on():
    """The FT-mixed regime split (graph_ft_batches) for the samples and the
    estimators this test makes."""
    return True


def _est(split: bool = False) -> MergedExecutionEstimator:
    e = MergedExecutionEstimator()
    e.split_mixed = split
    return e


def _tracker(rng, per_regime: int, regimes=tuple(TRUE)) -> StepLog:
    tr = StepLog()
    for r in regimes:
        for _ in range(per_regime):
            f = _sample(rng, r)
            assert f.regime(True) == r
            tr.add(f, _t(f, r))
    return tr


def test_fit_recovers_known_coefficients_per_regime(split_on):
    rng = np.random.default_rng(0)
    tr = _tracker(rng, 64)
    est = _est(split_on)
    assert not est.is_ready and est.predict(StepFeatures(b_d=4, k=512.0)) == 0.0
    est.data_fit(tr)
    assert est.is_ready
    for r, true in TRUE.items():
        p = est.params(r)
        assert p.is_fitted, r
        # FT-only steps (the eager regime with the split on) have T_in == T_ft and
        # no decode rows, so only beta + gamma is identifiable there
        names = ("alpha", "c") if r == REGIME_EAGER else tuple(true)
        for name in names:
            got = getattr(p, name)
            assert got == pytest.approx(true[name], rel=1e-5, abs=1e-12), (r, name, got, true[name])
        if r == REGIME_EAGER:
            assert p.beta + p.gamma == pytest.approx(true["beta"] + true["gamma"], rel=1e-5)
        assert est.rmse(r) < 1e-9
    rng2 = np.random.default_rng(1)
    for r in TRUE:
        f = _sample(rng2, r)
        assert est.select_regime(f) == r
        assert est.predict(f, apply_margin=False) == pytest.approx(_t(f, r), rel=1e-6)


def test_contended_prefill_excluded_and_min_samples():
    rng = np.random.default_rng(2)
    tr = StepLog()
    for _ in range(32):                 # prefill while a backward runs: recorded, never fitted
        f = _sample(rng, REGIME_INF_PREFILL)
        f.bwd = True
        assert f.contended
        tr.add(f, 10.0)
    for _ in range(MIN_FIT_SAMPLES - 1):   # one short of the fit threshold
        f = _sample(rng, REGIME_DECODE_ONLY)
        tr.add(f, _t(f, REGIME_DECODE_ONLY))
    est = MergedExecutionEstimator()
    est.data_fit(tr)
    assert not est.is_ready
    f = _sample(rng, REGIME_DECODE_ONLY)
    tr.add(f, _t(f, REGIME_DECODE_ONLY))
    est.data_fit(tr)
    assert est.params(REGIME_DECODE_ONLY).is_fitted
    assert not est.params(REGIME_INF_PREFILL).is_fitted


def test_regime_routing_fallbacks():
    rng = np.random.default_rng(3)
    est = MergedExecutionEstimator()
    est.data_fit(_tracker(rng, 32, regimes=(REGIME_DECODE_ONLY, REGIME_EAGER)))
    # decode with a backward in flight falls back to the decode-only fit
    f = StepFeatures(b_d=8, k=4096.0, bwd=True)
    assert f.regime() == REGIME_DECODE_BWD
    assert est.select_regime(f) == REGIME_DECODE_ONLY
    assert est.predict(f, apply_margin=False) == pytest.approx(_t(f, REGIME_DECODE_ONLY), rel=1e-6)
    # split off: FT next to inference is an eager step
    mixed = StepFeatures(t_in=900.0, p=3, t_ft=300.0, b_d=4, k=2048.0, prefill_lens=[300, 300, 300])
    assert mixed.regime() == REGIME_EAGER
    assert est.select_regime(mixed) == REGIME_EAGER
    # a forced regime with no fit routes to the first fitted one in order
    assert est.select_regime(mixed, REGIME_FT_MIXED) == REGIME_EAGER
    assert est.select_regime(StepFeatures(t_in=64.0, p=1, prefill_lens=[64])) == REGIME_EAGER


def test_refit_cadence_and_tracker_window():
    tr = StepLog(capacity=REFIT_EVERY)
    f = StepFeatures(b_d=1, k=64.0)
    fired = []
    for i in range(1, 3 * REFIT_EVERY + 3):
        tr.add(f, 0.01)
        if tr.due_for_refit():
            fired.append(i)
        assert not tr.due_for_refit()      # at most once per REFIT_EVERY records
    # the cadence keeps going after the ring is full
    assert fired == [REFIT_EVERY, 2 * REFIT_EVERY, 3 * REFIT_EVERY]
    small = StepLog(capacity=10)
    for i in range(25):
        small.add(StepFeatures(b_d=i + 1, k=1.0), float(i))
    assert small.size() == 10 and small.durations[0] == 15.0 and small.feature(0).b_d == 16
    grow = StepLog(capacity=10)
    for i in range(6):
        grow.add(StepFeatures(b_d=1, k=1.0), float(i))
    grow.truncate(4)
    assert grow.size() == 4 and list(grow.durations) == [0.0, 1.0, 2.0, 3.0]


def test_margin_modes():
    rng = np.random.default_rng(4)
    tr = StepLog()
    for _ in range(64):
        f = _sample(rng, REGIME_DECODE_ONLY)
        tr.add(f, _t(f, REGIME_DECODE_ONLY) * (1.0 + 0.05 * rng.standard_normal()))
    est = MergedExecutionEstimator()
    est.data_fit(tr)
    f = StepFeatures(b_d=16, k=16 * 512.0)
    raw = est.predict(f, apply_margin=False)
    rmse, rel = est.rmse(REGIME_DECODE_ONLY), est.rel_rmse(REGIME_DECODE_ONLY)
    assert rmse > 0 and rel > 0
    assert est.predict(f) == pytest.approx(raw * (1 + 1.5 * rmse))          # legacy
    est.set_margin("relative", 2.0)
    assert est.predict(f) == pytest.approx(raw * (1 + 2.0 * rel))
    est.set_margin("absolute", 3.0)
    assert est.predict(f) == pytest.approx(raw + 3.0 * rmse)
    with pytest.raises(ValueError):
        est.set_margin("quadratic")


def test_estimator_and_tracker_state_round_trip(tmp_path, split_on):
    rng = np.random.default_rng(5)
    tr = _tracker(rng, 16)
    est = _est(split_on)
    est.data_fit(tr)
    est2, tr2 = _est(split_on), StepLog()
    est2.import_state(est.export_state())
    tr2.import_state(tr.export_state())
    assert tr2.size() == tr.size()
    assert np.array_equal(tr2.column("s"), tr.column("s"))
    for f in tr.features[::7]:
        assert est2.predict(f) == est.predict(f)
    # predictions are only written for steps that had one
    for i, f in enumerate(tr.features[:5]):
        tr.set_predicted(i, est.predict(f))
    path = tmp_path / "pred" / "stats.csv"
    tr.write_prediction_stats_csv(str(path), split_mixed=True)
    rows = list(csv.DictReader(open(path)))
    assert len(rows) == 5 and rows[0]["regime"] == tr.features[0].regime(True)


def test_profiling_shapes_cover_every_regime(split_on):
    gen = ProfilingShapeGenerator(batch_max_tokens=8192, max_saved_finetuning_tokens=4096,
                                  max_req_len=4096, max_ft_sample=512)
    warm, rec = gen.prepare(with_ft=True)
    assert warm and rec
    kinds = {s.kind for s in rec}
    assert kinds == {"prefill", "decode", "mixed", "coserve", "ft_only"}
    for s in rec:
        total = sum(s.inf_lens) * (0 if s.kind == "decode" else 1) + sum(s.ft_lens) + sum(s.mix_lens)
        assert total <= gen.T, s
        assert all(n <= gen.max_req for n in s.inf_lens + s.mix_lens), s
        assert all(0 < n <= gen.ft_sample + 1 for n in s.ft_lens), s
        assert sum(s.ft_lens) <= gen.ft_cap
    # the FT-free plan has no FT rows at all
    _, rec_inf = gen.prepare(with_ft=False)
    assert not any(s.ft_lens for s in rec_inf)
    # a small token budget still yields a valid (smaller) plan
    small = ProfilingShapeGenerator(batch_max_tokens=512, max_saved_finetuning_tokens=256, max_req_len=512)
    _, rec_s = small.prepare()
    assert all(sum(s.ft_lens) + (sum(s.inf_lens) if s.kind != "decode" else 0) + sum(s.mix_lens) <= 512
               for s in rec_s)


def test_step_trace_rows(tmp_path):
    est = MergedExecutionEstimator()
    rng = np.random.default_rng(6)
    est.data_fit(_tracker(rng, 16, regimes=(REGIME_DECODE_ONLY,)))
    eng = SimpleNamespace(estimator=est, step_listeners=[],
                          last_admit=SimpleNamespace(code="A", baseline=0.01, predicted=0.02))
    path = str(tmp_path / "trace" / "steps.csv")
    w = attach_step_trace(eng, path)
    for i in range(5):
        f = StepFeatures(b_d=i + 1, k=128.0 * (i + 1))
        rec = SimpleNamespace(kind="decode", features=f, predicted=est.predict(f))
        for cb in eng.step_listeners:
            cb(rec, 0.01 * (i + 1))
    w.close()
    rows = list(csv.DictReader(open(path)))
    assert list(rows[0]) == list(COLUMNS)
    assert [int(r["seq"]) for r in rows] == [1, 2, 3, 4, 5]
    assert rows[2]["regime"] == REGIME_DECODE_ONLY and rows[2]["admit_code"] == "A"
    assert float(rows[4]["actual"]) == pytest.approx(0.05)
    assert float(rows[0]["pred_raw"]) <= float(rows[0]["pred"])
    w2 = StepTraceWriter(os.path.join(tmp_path, "plain.csv"))
    w2.put_row(kind="x", regime=None, bwd_in_flight=True)
    w2.close()
    line = open(os.path.join(tmp_path, "plain.csv")).read().splitlines()[1].split(",")
    assert line[COLUMNS.index("bwd_in_flight")] == "1" and line[COLUMNS.index("regime")] == ""
