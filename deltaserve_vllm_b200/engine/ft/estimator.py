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
    s_sum: float | None = None      # sum of squared prefill lengths when known without the lengths

    @property
    def s(self) -> float:
        if self.s_sum is not None:
            return float(self.s_sum)
        if self.prefill_lens:
            return float(sum(int(n) * int(n) for n in self.prefill_lens))
        if self.p > 0:
            return float(self.t_in) ** 2 / float(self.p)
        return 0.0

    @property
    def has_ft(self) -> bool:
        return self.t_ft > 0

    def row(self) -> np.ndarray:
        """The model's feature row: ``[s, T_in, T_ft, B_d, K, 1]``."""
        return np.array((self.s, self.t_in, self.t_ft, self.b_d, self.k, 1.0), np.float64)

    def regime(self, split_mixed: bool = False) -> str:
        """The regime of this step. ``split_mixed`` (the ``graph_ft_batches``
        switch, an attribute of the estimator) gives FT rows that share a step
        with inference work their own regime."""
        return _regime(self.t_in, self.t_ft, self.b_d, self.bwd, split_mixed)

    @property
    def contended(self) -> bool:
        return self.bwd and self.t_in > 0


def _regime(t_in, t_ft, b_d, bwd, split_mixed: bool) -> str:
    if t_ft > 0:
        return REGIME_FT_MIXED if split_mixed and (t_in > t_ft or b_d > 0) else REGIME_EAGER
    if t_in > 0:
        return REGIME_INF_PREFILL
    return REGIME_DECODE_BWD if bwd else REGIME_DECODE_ONLY


_NAMES = ("alpha", "beta", "gamma", "delta", "epsilon", "c")


class StepParams:
    """One regime's fitted model: the coefficient vector ``coef`` over the
    feature row ``[s, T_in, T_ft, B_d, K, 1]`` (named alpha, beta, gamma,
    delta, epsilon, c), or None while the regime has too few samples; and
    the fit's quality on its own samples (``rmse`` in seconds, ``rel_rmse``
    relative), which the admission margins use."""

    __slots__ = ("coef", "rmse", "rel_rmse")

    def __init__(self, *coef, rmse: float | None = None, rel_rmse: float | None = None):
        vals = list(coef[0]) if len(coef) == 1 and isinstance(coef[0], (list, tuple, np.ndarray)) else list(coef)
        self.coef = (np.asarray(vals, np.float64)
                     if len(vals) == len(_NAMES) and all(v is not None for v in vals) else None)
        self.rmse, self.rel_rmse = rmse, rel_rmse

    @property
    def is_fitted(self) -> bool:
        return self.coef is not None

    def eval(self, f: StepFeatures) -> float:
        return float(self.coef @ f.row())

    def as_list(self) -> list:
        return [None] * len(_NAMES) if self.coef is None else [float(v) for v in self.coef]

    def __getattr__(self, name):          # alpha .. c by name
        try:
            i = _NAMES.index(name)
        except ValueError:
            raise AttributeError(name) from None
        return None if self.coef is None else float(self.coef[i])


# When a step's own regime has no fit yet, the first fitted one of these.
_FALLBACK = {
    REGIME_DECODE_BWD: (REGIME_DECODE_ONLY, REGIME_EAGER, REGIME_FT_MIXED, REGIME_INF_PREFILL),
    REGIME_FT_MIXED: (REGIME_EAGER, REGIME_INF_PREFILL, REGIME_DECODE_ONLY),
}
_FALLBACK_DEFAULT = (REGIME_EAGER, REGIME_FT_MIXED, REGIME_INF_PREFILL, REGIME_DECODE_ONLY)


class StepLog:
    """The served steps the estimator learns from: a ring of ``capacity``
    records in numpy columns (features, measured and predicted seconds,
    graph flag, wall time). Appending overwrites the oldest record once the
    ring is full; fits read the columns directly (no per-step objects)."""

    _F = ("t_in", "p", "t_ft", "b_d", "k", "s", "bwd")   # feature columns

    def __init__(self, capacity: int = 10240):
        self.capacity = int(capacity)
        self._col = {c: np.zeros(self.capacity) for c in self._F}
        self._dur = np.zeros(self.capacity)
        self._pred = np.full(self.capacity, np.nan)     # nan = no prediction was made
        self._graph = np.full(self.capacity, -1, dtype=np.int8)   # -1 unknown, 0 eager, 1 graph
        self._wall = np.zeros(self.capacity)
        self.appended = 0          # records ever appended (the write position is appended % capacity)
        self._refit_at = 0         # `appended` when the last refit was signalled

    # ------------------------------------------------------------ records
    def add(self, features: StepFeatures, duration: float, predicted: float | None = None,
            was_graph: bool | None = None) -> None:
        i = self.appended % self.capacity
        f = features
        for c, v in zip(self._F, (f.t_in, f.p, f.t_ft, f.b_d, f.k, f.s, float(bool(f.bwd)))):
            self._col[c][i] = v
        self._dur[i] = duration
        self._pred[i] = np.nan if predicted is None else predicted
        self._graph[i] = -1 if was_graph is None else int(bool(was_graph))
        self._wall[i] = time.time()
        self.appended += 1

    def size(self) -> int:
        return min(self.appended, self.capacity)

    __len__ = size

    def _order(self) -> np.ndarray:
        """Ring slots in chronological order."""
        n = self.size()
        if self.appended <= self.capacity:
            return np.arange(n)
        return (np.arange(n) + self.appended) % self.capacity

    def column(self, name: str) -> np.ndarray:
        """One column in chronological order (copy): a feature name,
        ``duration``, ``predicted`` (nan where none) or ``wall``."""
        src = {"duration": self._dur, "predicted": self._pred, "wall": self._wall}.get(name)
        return (self._col[name] if src is None else src)[self._order()]

    def feature(self, i: int) -> StepFeatures:
        j = self._order()[i]
        c = self._col
        return StepFeatures(t_in=float(c["t_in"][j]), p=int(c["p"][j]), t_ft=float(c["t_ft"][j]),
                            b_d=int(c["b_d"][j]), k=float(c["k"][j]), bwd=bool(c["bwd"][j]),
                            s_sum=float(c["s"][j]))

    @property
    def features(self) -> list[StepFeatures]:
        return [self.feature(i) for i in range(self.size())]

    @property
    def durations(self) -> np.ndarray:
        return self.column("duration")

    def set_predicted(self, i: int, value: float | None) -> None:
        self._pred[self._order()[i]] = np.nan if value is None else value

    def truncate(self, n: int) -> None:
        """Forget every record after the first ``n`` (used before the ring
        has ever wrapped: the launch-time profiling steps)."""
        if not 0 <= n <= self.size() or self.appended > self.capacity:
            raise ValueError("truncate: only before the ring wraps, to a length it has")
        self.appended = n
        self._refit_at = min(self._refit_at, n)

    def due_for_refit(self) -> bool:
        """True once per REFIT_EVERY appended records."""
        mark = self.appended - self.appended % REFIT_EVERY
        if mark > self._refit_at:
            self._refit_at = mark
            return True
        return False

    # ------------------------------------------------------------ state / export
    def export_state(self) -> dict:
        cols = {c: self.column(c).tolist() for c in self._F}
        cols["duration"] = self.column("duration").tolist()
        cols["graph"] = self._graph[self._order()].astype(int).tolist()
        return {"format": "columns", "capacity": self.capacity, "refit_at": self._refit_at,
                "appended": self.appended, "cols": cols}

    def import_state(self, state: dict) -> None:
        self.__init__(self.capacity)
        if "cols" in state:
            cols = state["cols"]
            n = len(cols["duration"])
            for i in range(n):
                f = StepFeatures(t_in=cols["t_in"][i], p=int(cols["p"][i]), t_ft=cols["t_ft"][i],
                                 b_d=int(cols["b_d"][i]), k=cols["k"][i], bwd=bool(cols["bwd"][i]),
                                 s_sum=cols["s"][i])
                g = cols["graph"][i]
                self.add(f, cols["duration"][i], None, None if g < 0 else bool(g))
        else:   # the row-list format of earlier files: one list per step
            for t_in, p, t_ft, b_d, k, lens, bwd, dur, wg in state.get("samples", []):
                self.add(StepFeatures(t_in=t_in, p=p, t_ft=t_ft, b_d=b_d, k=k, prefill_lens=lens, bwd=bwd),
                         dur, None, wg)
        self._refit_at = min(int(state.get("refit_at", state.get("last_refit_size", 0))), self.appended)

    def write_prediction_stats_csv(self, path: str | None, split_mixed: bool = False) -> None:
        """One row per step that had a prediction: features, regime, measured
        and predicted seconds."""
        if path is None:
            return
        if os.path.dirname(path):
            os.makedirs(os.path.dirname(path), exist_ok=True)
        cols = ["timestamp", "step_index", "regime", "was_graph", "t_in", "p", "t_ft", "b_d", "k",
                "s", "execution_duration", "predicted_duration"]
        pred, dur, wall = self.column("predicted"), self.column("duration"), self.column("wall")
        graph = self._graph[self._order()]
        with open(path, "w", newline="") as fh:
            w = csv.writer(fh)
            w.writerow(cols)
            for i in np.flatnonzero(~np.isnan(pred)):
                f = self.feature(int(i))
                w.writerow([wall[i], int(i), f.regime(split_mixed), None if graph[i] < 0 else bool(graph[i]),
                            f.t_in, f.p, f.t_ft, f.b_d, f.k, f.s, dur[i], pred[i]])


_COLS = {
    REGIME_INF_PREFILL: (0, 1, 3, 4, 5),
    REGIME_EAGER: (0, 1, 2, 3, 4, 5),
    REGIME_FT_MIXED: (0, 1, 2, 3, 4, 5),
    REGIME_DECODE_ONLY: (3, 4, 5),
    REGIME_DECODE_BWD: (3, 4, 5),
}
class MergedExecutionEstimator:
    MARGIN_MODES = ("legacy", "relative", "absolute")

    def __init__(self):
        self._params = {r: StepParams() for r in REGIMES}     # per regime: coefficients and fit quality
        self.margin_mode = "legacy"
        self.margin_k = 1.5
        # graph_ft_batches: FT rows that share a step with inference work are
        # their own regime (ft_mixed) instead of the eager one.
        self.split_mixed = False

    def regime_of(self, f: StepFeatures) -> str:
        return f.regime(self.split_mixed)

    def set_margin(self, mode: str = "legacy", k: float = 1.5) -> None:
        if mode not in self.MARGIN_MODES:
            raise ValueError(f"slo.admission_margin must be one of {self.MARGIN_MODES}, got {mode!r}")
        self.margin_mode, self.margin_k = mode, float(k)

    def _with_margin(self, pred: float, regime: str) -> float:
        if self.margin_mode == "legacy":
            r = self._params[regime].rmse
            return pred * (1.0 + 1.5 * r) if r else pred
        if self.margin_mode == "relative":
            r = self._params[regime].rel_rmse
            return pred * (1.0 + self.margin_k * r) if r else pred
        r = self._params[regime].rmse
        return pred + self.margin_k * r if r else pred

    @property
    def is_ready(self) -> bool:
        return any(p.is_fitted for p in self._params.values())

    # ------------------------------------------------------------ state
    def export_state(self) -> dict:
        """Per regime: the six coefficients (alpha .. c, None when unfitted)
        and the fit's RMSE / relative RMSE."""
        return {"split_mixed": self.split_mixed,
                "regimes": {r: {"coef": p.as_list(), "rmse": p.rmse, "rel_rmse": p.rel_rmse}
                            for r, p in self._params.items()}}

    def import_state(self, state: dict) -> None:
        regimes = state.get("regimes")
        if regimes is None:   # files written with per-name coefficient dicts
            regimes = {r: {"coef": [c.get(n) for n in _NAMES],
                           "rmse": (state.get("rmse") or {}).get(r),
                           "rel_rmse": (state.get("rel_rmse") or {}).get(r)}
                       for r, c in (state.get("params") or {}).items()}
        for r, ent in regimes.items():
            if r not in self._params:
                continue
            self._params[r] = StepParams(*ent["coef"], rmse=ent.get("rmse"), rel_rmse=ent.get("rel_rmse"))

    @property
    def fit_rmse(self) -> float | None:
        """RMSE of the most informative fitted regime (FT steps first)."""
        fitted = [self._params[r].rmse for r in (REGIME_EAGER, REGIME_INF_PREFILL, REGIME_DECODE_ONLY)
                  if self._params[r].rmse is not None]
        return fitted[0] if fitted else None

    def rmse(self, regime: str) -> float | None:
        return self._params[regime].rmse

    def rel_rmse(self, regime: str) -> float | None:
        return self._params[regime].rel_rmse

    def params(self, regime: str) -> StepParams:
        return self._params[regime]

    def _select(self, f: StepFeatures, regime: str | None = None):
        regime = regime or self.regime_of(f)
        for r in (regime, *_FALLBACK.get(regime, _FALLBACK_DEFAULT)):
            if self._params[r].is_fitted:
                return r, self._params[r]
        return regime, self._params[regime]

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

    def data_fit(self, log: StepLog) -> dict[str, StepParams]:
        """Least squares per regime over the log's columns (prefill steps
        taken while a backward was in flight are left out: contended)."""
        c = {n: log.column(n) for n in StepLog._F}
        dur = log.column("duration")
        design = np.stack([c["s"], c["t_in"], c["t_ft"], c["b_d"], c["k"], np.ones_like(dur)], axis=1)
        bwd = c["bwd"] > 0
        contended = bwd & (c["t_in"] > 0)
        labels = np.array([_regime(a, b, d, e, self.split_mixed)
                           for a, b, d, e in zip(c["t_in"], c["t_ft"], c["b_d"], bwd)], dtype=object)
        msg = [f"excluded {int(contended.sum())} contended prefill"] if contended.any() else []
        for r in REGIMES:
            sel = (labels == r) & ~contended
            if int(sel.sum()) < MIN_FIT_SAMPLES:
                continue
            cols = list(_COLS[r])
            A, y = design[sel][:, cols], dur[sel]
            coef = np.linalg.lstsq(A, y, rcond=None)[0]
            full = np.zeros(6)
            full[cols] = coef
            err = A @ coef - y
            pos = y > 1e-6
            fit = StepParams(full, rmse=float(np.sqrt(np.mean(err ** 2))),
                             rel_rmse=float(np.sqrt(np.mean((err[pos] / y[pos]) ** 2))) if pos.any() else None)
            self._params[r] = fit
            msg.append(f"{r}={int(sel.sum())}(rmse={fit.rmse:.5f})")
        if msg:
            dprint("[estimator] fit: " + ", ".join(msg))
        return self._params
