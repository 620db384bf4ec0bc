"""The routing decision: which adapter serves a request, how sure the router
is, or the base model when it is not sure enough.

The quantities follow the reference (``deltaserve-plugin/deltaserve/adapter_routing/decision.py:1-147``):
sentence embeddings crowd into a narrow cone, so a raw cosine to a centroid
says little by itself, and the router scores pool-relative signals instead:

* ``top``    — the best cosine after centring (the mean of the pool's
  centroids subtracted from request and centroids alike);
* ``margin`` — best minus second-best centred cosine;
* ``confidence = z(top) + z(margin)``, the z statistics taken over the pool's
  reference samples; the gate is the ``100 - keep_percent`` percentile of the
  reference samples' own confidences, lowered by ``slack``;
* candidates within ``close_band`` of the best are interchangeable and a
  ``prefer`` key picks among them (saves slot swaps).

Pools smaller than ``min_pool`` cannot be centred (one centroid IS the mean):
they gate on the z-scored raw best cosine. Without reference samples nothing
is gated.

Implementation: :class:`PoolGeometry` is an immutable snapshot that scores a
whole batch of embeddings with one matrix product (:meth:`PoolGeometry.score`);
the calibration runs the same scorer over the reference samples.
:func:`admission_report` measures a candidate's effect on the pool with one
assignment pass over every reference sample.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .index import CentroidIndex, l2_normalize

CENTRED, RAW, UNGATED = "centred", "raw", "ungated"


@dataclass
class RouteChoice:
    adapter: str | None                     # None = the base model
    raw_cosine: float | None = None         # raw cosine of the best adapter
    confidence: float | None = None
    margin: float | None = None
    shortlist: list = field(default_factory=list)   # the close candidates, best first
    below_gate: bool = False                # confidence under the pool's gate


@dataclass
class _Scores:
    """Batch scores: ``S`` [B, n] the gating scores (centred or raw), ``raw``
    [B, n] raw cosines, ``best`` [B] index, ``top`` / ``margin`` /
    ``confidence`` [B] (confidence None when the pool has no calibration)."""
    S: np.ndarray
    raw: np.ndarray
    best: np.ndarray
    top: np.ndarray
    margin: np.ndarray
    confidence: np.ndarray | None


class PoolGeometry:
    """Routing geometry of one pool snapshot (rebuilt whenever the pool changes)."""

    def __init__(self, index: CentroidIndex, keep_percent: float = 90.0, close_band: float = 0.05,
                 min_pool: int = 4, slack: float = 0.0):
        self.names = list(index.names)
        self.keep_percent, self.close_band, self.slack = float(keep_percent), float(close_band), float(slack)
        self.C = index.matrix.astype(np.float32) if self.names else np.zeros((0, 0), np.float32)
        refs = [index.refs[n] for n in self.names if n in index.refs]
        R = np.concatenate(refs).astype(np.float32) if refs else np.zeros((0, self.C.shape[1] or 1), np.float32)
        self.n_refs = len(R)
        centre = self.n_refs > 0 and len(self.names) >= max(2, int(min_pool))
        self.mode = CENTRED if centre else (RAW if self.n_refs and self.names else UNGATED)
        self.mu = self.C.mean(0) if centre else None
        self.G = l2_normalize(self.C - self.mu) if centre else self.C   # the gating centroids
        # z statistics of (top, margin) over the reference samples, then the gate
        self.z = np.array([0.0, 1.0, 0.0, 1.0])
        self.threshold = None
        if self.mode != UNGATED:
            sc = self.score(R, calibrated=False)
            z_top = (sc.top.mean(), sc.top.std() or 1.0)
            z_mar = (sc.margin.mean(), sc.margin.std() or 1.0) if self.mode == CENTRED else (0.0, 1.0)
            self.z = np.array([z_top[0], z_top[1], z_mar[0], z_mar[1]], dtype=np.float64)
            if self.keep_percent < 100.0:
                conf = self._confidence(sc.top, sc.margin)
                self.threshold = float(np.percentile(conf, 100.0 - self.keep_percent)) - self.slack

    # ------------------------------------------------------------ scoring
    def _project(self, E: np.ndarray) -> np.ndarray:
        return l2_normalize(E - self.mu) if self.mode == CENTRED else E

    def _confidence(self, top: np.ndarray, margin: np.ndarray) -> np.ndarray:
        z = (top - self.z[0]) / self.z[1]
        return z + (margin - self.z[2]) / self.z[3] if self.mode == CENTRED else z

    def score(self, E, calibrated: bool = True) -> _Scores:
        """Scores of a batch of embeddings [B, d] (normalised here)."""
        E = l2_normalize(np.asarray(E, np.float32).reshape(-1, self.C.shape[1]))
        raw = E @ self.C.T
        S = self._project(E) @ self.G.T if self.mode == CENTRED else raw
        best = np.argmax(S, axis=1)
        rows = np.arange(len(S))
        top = S[rows, best]
        if S.shape[1] > 1:
            second = np.partition(S, S.shape[1] - 2, axis=1)[:, -2]
            margin = top - second
        else:
            margin = np.zeros_like(top)
        conf = self._confidence(top, margin) if (calibrated and self.mode != UNGATED) else None
        return _Scores(S, raw, best, top, margin, conf)

    def describe(self) -> dict:
        return {"mode": self.mode, "adapters": len(self.names), "reference_samples": self.n_refs,
                "threshold": self.threshold, "keep_percent": self.keep_percent,
                "slack": self.slack, "close_band": self.close_band}

    def decide(self, emb, prefer=None, raw_floor: float = -1.0) -> RouteChoice:
        """Route one embedding. ``prefer(name)`` gives a sortable key (higher
        wins among the close candidates); ``raw_floor`` is an absolute cut on
        the best raw cosine."""
        if not self.names:
            return RouteChoice(None)
        sc = self.score(emb)
        s, b = sc.S[0], int(sc.best[0])
        ranked = np.argsort(-s, kind="stable")
        margin = float(sc.margin[0]) if len(self.names) > 1 else None
        conf = float(sc.confidence[0]) if sc.confidence is not None else None
        band = self.close_band if self.mode == CENTRED else -np.inf
        shortlist = [self.names[i] for i in ranked if s[i] >= s[b] - band] if band != -np.inf \
            else [self.names[b]]
        raw_best = float(sc.raw[0, b])
        out = RouteChoice(None, raw_best, conf, margin, shortlist)
        if raw_best < raw_floor:
            return out
        if self.threshold is not None and conf is not None and conf < self.threshold:
            out.below_gate = True
            return out
        out.adapter = shortlist[0]
        if len(shortlist) > 1 and prefer is not None:
            # highest preference; among equal preferences the better score
            keyed = sorted(enumerate(shortlist), key=lambda t: (prefer(t[1]), -t[0]), reverse=True)
            out.adapter = keyed[0][1]
        return out


def admission_report(index: CentroidIndex, name: str, centroid, refs=None, min_pool: int = 4) -> dict:
    """What adding ``name`` (``centroid``, reference samples ``refs``) to the
    active pool ``index`` would do, on reference samples only (no encoding):

    * ``self_recall`` — share of the candidate's reference samples the new
      pool routes to it;
    * ``stolen`` / ``stolen_max`` / ``stolen_from`` — per existing adapter,
      the share of its own reference samples the candidate would take;
    * ``nearest`` / ``nearest_cosine`` — the closest existing centroid.
    """
    others = [n for n in index.names if n != name]
    rep = {"pool_before": len(others), "self_recall": None, "stolen": {}, "stolen_max": 0.0,
           "stolen_from": None, "nearest": None, "nearest_cosine": None}
    if not others:
        return rep
    cand = l2_normalize(np.asarray(centroid, np.float32).reshape(1, -1))
    C = np.concatenate([np.stack([index.centroid_of(n) for n in others]), cand]).astype(np.float32)
    new = len(C) - 1                               # the candidate's column
    if len(C) >= max(2, int(min_pool)):
        mu = C.mean(0)
        G = l2_normalize(C - mu)
        proj = lambda X: l2_normalize(np.asarray(X, np.float32) - mu)  # noqa: E731
    else:
        G = C
        proj = lambda X: np.asarray(X, np.float32)  # noqa: E731
    near = G[:new] @ G[new]
    j = int(np.argmax(near))
    rep["nearest"], rep["nearest_cosine"] = others[j], round(float(near[j]), 4)
    if refs is not None and len(refs):
        rep["self_recall"] = round(float(np.mean(np.argmax(proj(refs) @ G.T, axis=1) == new)), 4)
    # every existing adapter's reference samples in one pass, labelled by owner
    owned = [(i, index.refs[n]) for i, n in enumerate(others) if n in index.refs and len(index.refs[n])]
    if not owned:
        return rep
    X = np.concatenate([r for _, r in owned])
    owner = np.concatenate([np.full(len(r), i) for i, r in owned])
    S = proj(X) @ G.T
    before = np.argmax(S[:, :new], axis=1)
    after = np.argmax(S, axis=1)
    kept_own = before == owner                     # samples their owner wins today
    lost = kept_own & (after == new)               # ... and the candidate wins tomorrow
    n_own = np.bincount(owner[kept_own], minlength=len(others))
    n_lost = np.bincount(owner[lost], minlength=len(others))
    share = n_lost / np.maximum(1, n_own)
    for i in np.flatnonzero(share > 0):
        rep["stolen"][others[i]] = round(float(share[i]), 4)
    if share.max() > 0:
        k = int(np.argmax(share))                  # first adapter with the largest share
        rep["stolen_max"], rep["stolen_from"] = round(float(share[k]), 4), others[k]
    return rep

