"""The routing decision: which adapter, how confident, or the base model.

Sentence embeddings crowd into a narrow cone, so a raw cosine to a centroid
says little on its own. The decision therefore uses two pool-relative signals
(the reference's method, ``deltaserve-plugin/deltaserve/adapter_routing/decision.py:1-147``):

* the *centred* top-1 score: cosine after subtracting the mean of the pool's
  centroids from both request and centroids;
* the *margin* between the best and second-best centred scores.

``confidence = z(top-1) + z(margin)``, with the z statistics taken over the
pool's reference samples; the gate is the ``100 - keep_percent`` percentile
of the reference samples' own confidences, lowered by ``slack``. Candidates
within ``close_band`` of the best are interchangeable; ``prefer`` breaks the
tie (e.g. already in a GPU slot, then most used) to save slot swaps.

Pools smaller than ``min_pool`` cannot be centred (one centroid IS the mean):
they gate on the raw top-1 score z-scored over the reference samples. With no
reference samples nothing is gated.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .index import CentroidIndex, l2_normalize

CENTRED, RAW, UNGATED = "centred", "raw", "ungated"


@dataclass
class Choice:
    adapter: str | None                 # None = base model
    score: float | None = None          # raw cosine of the best adapter
    confidence: float | None = None
    margin: float | None = None
    candidates: list = field(default_factory=list)
    low_confidence: bool = False


def _top2(S: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per row: best value and best - second best (0 for a single column)."""
    if S.shape[1] == 1:
        return S[:, 0], np.zeros(S.shape[0], S.dtype)
    part = np.partition(S, S.shape[1] - 2, axis=1)
    best, second = part[:, -1], part[:, -2]
    return best, best - second


class RoutingModel:
    """Immutable snapshot of a pool's routing geometry (rebuilt on change)."""

    def __init__(self, index: CentroidIndex, keep_percent: float = 90.0, close_band: float = 0.05,
                 min_pool: int = 4, slack: float = 0.0):
        self.names = list(index.names)
        self.keep_percent = float(keep_percent)
        self.close_band = float(close_band)
        self.slack = float(slack)
        self.C = index.matrix.astype(np.float32) if self.names else np.zeros((0, 0), np.float32)
        ref_list = [index.refs[n] for n in self.names if n in index.refs]
        R = np.concatenate(ref_list).astype(np.float32) if ref_list else None
        self.n_refs = 0 if R is None else len(R)
        self.mode, self.threshold, self.mu, self.Cc = UNGATED, None, None, None
        self.stats = (0.0, 1.0, 0.0, 1.0)           # mean/std of top-1, mean/std of margin
        conf = None
        if R is not None and len(self.names) >= max(2, int(min_pool)):
            self.mode = CENTRED
            self.mu = self.C.mean(0)
            self.Cc = l2_normalize(self.C - self.mu)
            top, margin = self._centred_signals(R)
            self.stats = (float(top.mean()), float(top.std()) or 1.0,
                          float(margin.mean()), float(margin.std()) or 1.0)
            conf = self._confidence(top, margin)
        elif R is not None and self.names:
            self.mode = RAW
            top = (R @ self.C.T).max(1)
            self.stats = (float(top.mean()), float(top.std()) or 1.0, 0.0, 1.0)
            conf = (top - self.stats[0]) / self.stats[1]
        if conf is not None and self.keep_percent < 100.0:
            self.threshold = float(np.percentile(conf, 100.0 - self.keep_percent)) - self.slack

    def _centred_signals(self, E: np.ndarray):
        return _top2(l2_normalize(E - self.mu) @ self.Cc.T)

    def _confidence(self, top, margin):
        m1, s1, m2, s2 = self.stats
        return (top - m1) / s1 + (margin - m2) / s2

    def describe(self) -> dict:
        return {"mode": self.mode, "adapters": len(self.names), "reference_samples": self.n_refs,
                "threshold": self.threshold, "keep_percent": self.keep_percent,
                "slack": self.slack, "close_band": self.close_band}

    def decide(self, emb, prefer=None, raw_floor: float = -1.0) -> Choice:
        """``prefer(name)`` returns a sortable key (higher wins among close
        candidates); ``raw_floor`` is an absolute cut on the raw cosine."""
        if not self.names:
            return Choice(None)
        e = l2_normalize(np.asarray(emb, np.float32).reshape(1, -1))
        raw = (e @ self.C.T)[0]
        s = (l2_normalize(e - self.mu) @ self.Cc.T)[0] if self.mode == CENTRED else raw
        order = np.argsort(-s, kind="stable")
        b = int(order[0])
        margin = float(s[b] - s[order[1]]) if len(order) > 1 else None
        if self.mode == CENTRED:
            conf = float(self._confidence(s[b], margin if margin is not None else 0.0))
            close = [self.names[i] for i in order if s[i] >= s[b] - self.close_band]
        else:
            conf = float((raw[b] - self.stats[0]) / self.stats[1]) if self.mode == RAW else None
            close = [self.names[b]]
        score = float(raw[b])
        if score < raw_floor:
            return Choice(None, score, conf, margin, close)
        if self.threshold is not None and conf is not None and conf < self.threshold:
            return Choice(None, score, conf, margin, close, low_confidence=True)
        pick = close[0]
        if len(close) > 1 and prefer is not None:
            rank = {n: i for i, n in enumerate(close)}
            pick = max(close, key=lambda n: (prefer(n), -rank[n]))
        return Choice(pick, score, conf, margin, close)


def admission_report(index: CentroidIndex, name: str, centroid, refs=None, min_pool: int = 4) -> dict:
    """What adding ``name`` to the active pool ``index`` would do, measured on
    reference samples only (no encoding):

    * ``self_recall`` — share of the candidate's reference samples the new
      pool sends to it;
    * ``stolen`` / ``stolen_max`` / ``stolen_from`` — per existing adapter,
      the share of its reference samples the candidate would take;
    * ``nearest`` / ``nearest_cosine`` — the closest existing centroid.
    """
    c = l2_normalize(np.asarray(centroid, np.float32).reshape(-1))
    others = [n for n in index.names if n != name]
    rep = {"pool_before": len(others), "self_recall": None, "stolen": {}, "stolen_max": 0.0,
           "stolen_from": None, "nearest": None, "nearest_cosine": None}
    if not others:
        return rep
    C = np.vstack([index.centroid_of(n) for n in others] + [c])
    if len(C) >= max(2, int(min_pool)):
        mu = C.mean(0)
        Cc = l2_normalize(C - mu)
        proj = lambda X: l2_normalize(np.asarray(X, np.float32) - mu)  # noqa: E731
    else:
        Cc = C
        proj = lambda X: np.asarray(X, np.float32)  # noqa: E731
    me = len(C) - 1
    sims = Cc[:me] @ Cc[me]
    j = int(np.argmax(sims))
    rep["nearest"], rep["nearest_cosine"] = others[j], round(float(sims[j]), 4)
    if refs is not None and len(refs):
        rep["self_recall"] = round(float(((proj(refs) @ Cc.T).argmax(1) == me).mean()), 4)
    for i, n in enumerate(others):
        r = index.refs.get(n)
        if r is None or not len(r):
            continue
        S = proj(r) @ Cc.T
        mine_before = S[:, :me].argmax(1) == i
        taken = mine_before & (S.argmax(1) == me)
        share = float(taken.sum()) / max(1, int(mine_before.sum()))
        if share > 0:
            rep["stolen"][n] = round(share, 4)
        if share > rep["stolen_max"]:
            rep["stolen_max"], rep["stolen_from"] = round(share, 4), n
    return rep
