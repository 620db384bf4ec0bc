"""Composition-based step-time estimator.

One step's time is modelled as ``T = a*S + b*T_in + g*T_ft + d*B_d + e*K + c`` with
``S = sum(n_i^2)`` over prefill chunks, ``T_in`` prefill tokens (FT rows
included), ``T_ft`` FT rows, ``B_d`` decode requests and ``K`` decode KV tokens.
Steps are partitioned by composition into regimes, each fitted by least
squares on its own reduced design matrix (the reference's regime set and fit
procedure, ``deltaserve-plugin/deltaserve/estimator.py:104-579``):

=============  ===================================  =====================
regime         steps                                columns
=============  ===================================  =====================
inf_prefill    prefill, no FT                        S, T_in, B_d, K, 1
eager          FT rows (FT-only, or all FT steps)    S, T_in, T_ft, B_d, K, 1
ft_mixed       FT next to inference (split on)       same as eager
decode_only    decode only                           B_d, K, 1
decode_bwd     decode only, backward in flight       B_d, K, 1
=============  ===================================  =====================

Prefill steps taken while a backward is in flight are recorded but never fitted
("contended"). Refit every 256 recorded steps once a regime has 8 samples.
Margins: ``legacy`` (x(1 + 1.5*RMSE[s])), ``relative`` (x(1 + k*relRMSE)),
``absolute`` (+ k*RMSE).
"""

from __future__ import annotations

import csv
import os
import time
from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np

from ... import dprint

MIN_FIT_SAMPLES = 8
REFIT_EVERY = 256

REGIME_INF_PREFILL = "inf_prefill"
REGIME_EAGER = "eager"
REGIME_DECODE_ONLY = "decode_only"
REGIME_DECODE_BWD = "decode_bwd"
REGIME_FT_MIXED = "ft_mixed"
REGIMES = (REGIME_INF_PREFILL, REGIME_EAGER, REGIME_DECODE_ONLY, REGIME_DECODE_BWD, REGIME_FT_MIXED)

_FT_MIXED_SPLIT = False


def set_ft_mixed_split(enabled: bool) -> None:
    global _FT_MIXED_SPLIT
    _FT_MIXED_SPLIT = bool(enabled)


def ft_mixed_split() -> bool:
    return _FT_MIXED_SPLIT


@dataclass
class StepFeatures:
    t_in: float = 0.0
    p: int = 0
    t_ft: float = 0.0
    b_d: int = 0
    k: float = 0.0
    prefill_lens: Sequence[int] | None = None
    bwd: bool = False
    load_s: float = 0.0

    @property
    def s(self) -> float:
        if self.prefill_lens:
            return float(sum(int(n) * int(n) for n in self.prefill_lens))
        if self.p > 0:
            return float(self.t_in) ** 2 / float(self.p)
        return 0.0

    @property
    def has_ft(self) -> bool:
        return self.t_ft > 0

    def row(self) -> list[float]:
        return [self.s, float(self.t_in), float(self.t_ft), float(self.b_d), float(self.k), 1.0]

    def regime(self) -> str:
        if self.t_ft > 0:
            if _FT_MIXED_SPLIT and (self.t_in > self.t_ft or self.b_d > 0):
                return REGIME_FT_MIXED
            return REGIME_EAGER
        if self.t_in > 0:
            return REGIME_INF_PREFILL
        if self.bwd:
            return REGIME_DECODE_BWD
        return REGIME_DECODE_ONLY

    @property
    def contended(self) -> bool:
        return self.bwd and self.t_in > 0


@dataclass
class StepParams:
    alpha: float | None = None
    beta: float | None = None
    gamma: float | None = None
    delta: float | None = None
    epsilon: float | None = None
    c: float | None = None

    @property
    def is_fitted(self) -> bool:
        return all(v is not None for v in (self.alpha, self.beta, self.gamma, self.delta,
                                           self.epsilon, self.c))

    def eval(self, f: StepFeatures) -> float:
        return (self.alpha * f.s + self.beta * f.t_in + self.gamma * f.t_ft + self.delta * f.b_d
                + self.epsilon * f.k + self.c)


class StepExecutionTracker:
    """Rolling record of served steps: features, measured and predicted time."""

    def __init__(self, max_steps: int = 10240):
        self.max_steps = max_steps
        self.features: list[StepFeatures] = []
        self.durations: list[float] = []
        self.predicted: list[float | None] = []
        self.was_graph: list[bool | None] = []
        self.timestamps: list[float] = []
        self._last_refit_size = 0

    def add(self, features: StepFeatures, duration: float, predicted: float | None = None,
            was_graph: bool | None = None) -> None:
        self.features.append(features)
        self.durations.append(float(duration))
        self.predicted.append(predicted)
        self.was_graph.append(was_graph)
        self.timestamps.append(time.time())
        if len(self.durations) > self.max_steps:
            for lst in (self.features, self.durations, self.predicted, self.was_graph, self.timestamps):
                del lst[0]

    def size(self) -> int:
        return len(self.durations)

    def check_refit(self) -> bool:
        n = self.size()
        if n > 0 and n % REFIT_EVERY == 0 and n > self._last_refit_size:
            self._last_refit_size = n
            return True
        return False

    def export_state(self) -> dict:
        return {"max_steps": self.max_steps, "last_refit_size": self._last_refit_size,
                "samples": [[f.t_in, f.p, f.t_ft, f.b_d, f.k,
                             list(f.prefill_lens) if f.prefill_lens is not None else None,
                             bool(f.bwd), d, wg]
                            for f, d, wg in zip(self.features, self.durations, self.was_graph)]}

    def import_state(self, state: dict) -> None:
        self.features, self.durations, self.predicted, self.was_graph, self.timestamps = [], [], [], [], []
        now = time.time()
        for t_in, p, t_ft, b_d, k, lens, bwd, dur, wg in state["samples"]:
            self.features.append(StepFeatures(t_in=t_in, p=p, t_ft=t_ft, b_d=b_d, k=k,
                                              prefill_lens=lens, bwd=bwd))
            self.durations.append(float(dur))
            self.predicted.append(None)
            self.was_graph.append(wg)
            self.timestamps.append(now)
        while len(self.durations) > self.max_steps:
            for lst in (self.features, self.durations, self.predicted, self.was_graph, self.timestamps):
                del lst[0]
        self._last_refit_size = min(int(state.get("last_refit_size", 0)), self.size())

    def write_prediction_stats_csv(self, path: str | None) -> None:
        if path is None:
            return
        if os.path.dirname(path):
            os.makedirs(os.path.dirname(path), exist_ok=True)
        cols = ["timestamp", "step_index", "regime", "was_graph", "t_in", "p", "t_ft", "b_d", "k",
                "s", "execution_duration", "predicted_duration"]
        with open(path, "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=cols)
            w.writeheader()
            for i in range(self.size()):
                if self.predicted[i] is None:
                    continue
                f = self.features[i]
                w.writerow({"timestamp": self.timestamps[i], "step_index": i, "regime": f.regime(),
                            "was_graph": self.was_graph[i], "t_in": f.t_in, "p": f.p, "t_ft": f.t_ft,
                            "b_d": f.b_d, "k": f.k, "s": f.s,
                            "execution_duration": self.durations[i],
                            "predicted_duration": self.predicted[i]})


_COLS = {
    REGIME_INF_PREFILL: (0, 1, 3, 4, 5),
    REGIME_EAGER: (0, 1, 2, 3, 4, 5),
    REGIME_FT_MIXED: (0, 1, 2, 3, 4, 5),
    REGIME_DECODE_ONLY: (3, 4, 5),
    REGIME_DECODE_BWD: (3, 4, 5),
}
_NAMES = ("alpha", "beta", "gamma", "delta", "epsilon", "c")


class MergedExecutionEstimator:
    MARGIN_MODES = ("legacy", "relative", "absolute")

    def __init__(self):
        self._params = {r: StepParams() for r in REGIMES}
        self._rmse: dict[str, float | None] = {r: None for r in REGIMES}
        self._rel_rmse: dict[str, float | None] = {r: None for r in REGIMES}
        self.margin_mode = "legacy"
        self.margin_k = 1.5

    def set_margin(self, mode: str = "legacy", k: float = 1.5) -> None:
        if mode not in self.MARGIN_MODES:
            raise ValueError(f"slo.admission_margin must be one of {self.MARGIN_MODES}, got {mode!r}")
        self.margin_mode, self.margin_k = mode, float(k)

    def _with_margin(self, pred: float, regime: str) -> float:
        if self.margin_mode == "legacy":
            r = self._rmse[regime]
            return pred * (1.0 + 1.5 * r) if r else pred
        if self.margin_mode == "relative":
            r = self._rel_rmse[regime]
            return pred * (1.0 + self.margin_k * r) if r else pred
        r = self._rmse[regime]
        return pred + self.margin_k * r if r else pred

    @property
    def is_ready(self) -> bool:
        return any(p.is_fitted for p in self._params.values())

    def export_state(self) -> dict:
        return {"ft_mixed_split": ft_mixed_split(),
                "params": {r: {n: getattr(p, n) for n in _NAMES} for r, p in self._params.items()},
                "rmse": dict(self._rmse), "rel_rmse": dict(self._rel_rmse)}

    def import_state(self, state: dict) -> None:
        for r, coefs in (state.get("params") or {}).items():
            if r in self._params:
                self._params[r] = StepParams(**coefs)
                self._rmse[r] = (state.get("rmse") or {}).get(r)
                self._rel_rmse[r] = (state.get("rel_rmse") or {}).get(r)

    @property
    def fit_rmse(self) -> float | None:
        for r in (REGIME_EAGER, REGIME_INF_PREFILL, REGIME_DECODE_ONLY):
            if self._rmse[r] is not None:
                return self._rmse[r]
        return None

    def rmse(self, regime: str) -> float | None:
        return self._rmse[regime]

    def rel_rmse(self, regime: str) -> float | None:
        return self._rel_rmse[regime]

    def params(self, regime: str) -> StepParams:
        return self._params[regime]

    def _select(self, f: StepFeatures, regime: str | None = None):
        regime = regime or f.regime()
        p = self._params[regime]
        if p.is_fitted:
            return regime, p
        order = (REGIME_EAGER, REGIME_FT_MIXED, REGIME_INF_PREFILL, REGIME_DECODE_ONLY)
        if regime == REGIME_DECODE_BWD:
            order = (REGIME_DECODE_ONLY,) + order
        elif regime == REGIME_FT_MIXED:
            order = (REGIME_EAGER,) + order
        for r in order:
            if self._params[r].is_fitted:
                return r, self._params[r]
        return regime, p

    def select_regime(self, f: StepFeatures, regime: str | None = None) -> str | None:
        return self._select(f, regime)[0] if self.is_ready else None

    def predict(self, f: StepFeatures, regime: str | None = None, apply_margin: bool = True) -> float:
        if not self.is_ready:
            return 0.0
        r, p = self._select(f, regime)
        pred = p.eval(f)
        if apply_margin:
            pred = self._with_margin(pred, r)
        return max(0.0, float(pred))

    def data_fit(self, tracker: StepExecutionTracker) -> dict[str, StepParams]:
        buckets: dict[str, tuple[list, list]] = {r: ([], []) for r in REGIMES}
        contended = 0
        for f, dur in zip(tracker.features, tracker.durations):
            if f.contended:
                contended += 1
                continue
            r = f.regime()
            row = f.row()
            buckets[r][0].append([row[i] for i in _COLS[r]])
            buckets[r][1].append(dur)
        msg = [f"excluded {contended} contended prefill"] if contended else []
        for r in REGIMES:
            X, y = buckets[r]
            if len(y) < MIN_FIT_SAMPLES:
                continue
            A, b = np.asarray(X, float), np.asarray(y, float)
            coef, *_ = np.linalg.lstsq(A, b, rcond=None)
            vals = [0.0] * 6
            for c, i in zip(coef, _COLS[r]):
                vals[i] = float(c)
            self._params[r] = StepParams(*vals)
            pred = A @ coef
            self._rmse[r] = float(np.sqrt(np.mean((pred - b) ** 2)))
            pos = b > 1e-6
            self._rel_rmse[r] = (float(np.sqrt(np.mean(((pred[pos] - b[pos]) / b[pos]) ** 2)))
                                 if pos.any() else None)
            msg.append(f"{r}={len(y)}(rmse={self._rmse[r]:.5f})")
        if msg:
            dprint("[estimator] fit: " + ", ".join(msg))
        return self._params
