"""``Router``: centroid index + decision model -> :class:`RouteDecision`.

The decision reaches the client as response headers (same names and meaning
as the reference's ``deltaserve-plugin/deltaserve/route_middleware.py:27-36``)::

    x-deltaserve-routing: routed | fallback
    x-deltaserve-adapter: <adapter>                  (routed)
    x-deltaserve-routing-score: <best cosine>
    x-deltaserve-routing-confidence: <pool-relative confidence>
    x-deltaserve-routing-candidates: <a,b,...>       (several were close)
    x-deltaserve-routing-reason: <why>               (fallback)
    x-deltaserve-routing-message: <sentence>         (fallback)
"""

from __future__ import annotations

import json
import time
from dataclasses import dataclass

from .decision import PoolGeometry
from .index import CentroidIndex

ROUTED, FALLBACK = "routed", "fallback"
BELOW_THRESHOLD = "below-threshold"
LOW_CONFIDENCE = "low-confidence"
NO_ADAPTERS = "no-adapters"
NO_TEXT = "no-text"
UNAVAILABLE = "router-unavailable"
DISABLED = "adapter-routing-disabled"
MESSAGES = {
    BELOW_THRESHOLD: "no adapter matched this request closely enough; served by the base model",
    LOW_CONFIDENCE: "the best adapter is not a confident match for this request; served by the base model",
    NO_ADAPTERS: "no routable adapter is available; served by the base model",
    NO_TEXT: "the request has no text to route on; served by the base model",
    UNAVAILABLE: "the adapter router is unavailable; served by the base model",
    DISABLED: "adapter routing is not enabled on this server; served by the base model",
}


@dataclass
class RouteDecision:
    adapter: str | None
    score: float | None = None
    reason: str = ""
    confidence: float | None = None
    candidates: tuple = ()

    @property
    def outcome(self) -> str:
        return ROUTED if self.adapter else FALLBACK

    def headers(self) -> dict[str, str]:
        h = {"x-deltaserve-routing": self.outcome}
        if self.adapter:
            h["x-deltaserve-adapter"] = self.adapter
        if self.score is not None:
            h["x-deltaserve-routing-score"] = f"{self.score:.4f}"
        if self.confidence is not None:
            h["x-deltaserve-routing-confidence"] = f"{self.confidence:.3f}"
        if len(self.candidates) > 1:
            h["x-deltaserve-routing-candidates"] = ",".join(self.candidates)
        if self.reason:
            h["x-deltaserve-routing-reason"] = self.reason
            if self.reason in MESSAGES:
                h["x-deltaserve-routing-message"] = MESSAGES[self.reason]
        return h


def extract_text(body: dict) -> str | None:
    """The text a request is routed on: the last user message of a chat, the
    prompt string of a completion (first of a list); None for token ids."""
    msgs = body.get("messages")
    if msgs is None and "input" in body:
        if isinstance(body["input"], str):
            return body["input"] or None
        msgs = body["input"]
    if isinstance(msgs, list):
        for m in reversed(msgs):
            if isinstance(m, dict) and m.get("role") == "user":
                c = m.get("content")
                if isinstance(c, list):
                    c = "\n".join(p.get("text", "") for p in c if isinstance(p, dict)
                                  and p.get("type") in ("text", "input_text"))
                if isinstance(c, str) and c.strip():
                    return c
        return None
    p = body.get("prompt")
    if isinstance(p, str):
        return p or None
    if isinstance(p, list) and p and isinstance(p[0], str):
        return p[0] or None
    return None


class Router:
    def __init__(self, encoder, keep_percent: float = 90.0, close_band: float = 0.05,
                 min_pool: int = 4, slack: float = 0.0, raw_floor: float = -1.0,
                 decision_log: str | None = None, tier_of=None):
        self.encoder = encoder
        self._args = (float(keep_percent), float(close_band), int(min_pool), float(slack))
        self.raw_floor = float(raw_floor)
        self.decision_log = decision_log
        self.tier_of = tier_of or (lambda name: "")
        self.index = CentroidIndex()
        self.model = PoolGeometry(self.index, *self._args)
        self.routed: dict[str, int] = {}
        self.requests = 0

    def set_index(self, index: CentroidIndex) -> None:
        """Rebuild the decision model from a pool snapshot (one assignment,
        so a batch being routed keeps the model it started with)."""
        snap = index.snapshot()
        self.index, self.model = snap, PoolGeometry(snap, *self._args)

    def _prefer(self, name: str):
        return (self.tier_of(name) == "gpu", self.routed.get(name, 0))

    def _decide(self, model: PoolGeometry, emb) -> RouteDecision:
        c = model.decide(emb, prefer=self._prefer, raw_floor=self.raw_floor)
        reason = "" if c.adapter else (LOW_CONFIDENCE if c.below_gate else BELOW_THRESHOLD)
        if c.adapter:
            self.routed[c.adapter] = self.routed.get(c.adapter, 0) + 1
        d = RouteDecision(c.adapter, c.raw_cosine, reason, c.confidence, tuple(c.shortlist))
        if self.decision_log:
            try:
                with open(self.decision_log, "a") as f:
                    f.write(json.dumps({"t": round(time.time(), 3), "outcome": d.outcome,
                                        "adapter": d.adapter, "reason": d.reason, "score": d.score,
                                        "confidence": d.confidence, "margin": c.margin,
                                        "candidates": list(d.candidates)}) + "\n")
            except OSError:
                pass
        return d

    def route_many(self, texts: list) -> list[RouteDecision]:
        """One decision per text with ONE encoder call for the batch."""
        self.requests += len(texts)
        model = self.model                 # one snapshot for the whole batch
        has_text = [bool(t) and bool(str(t).strip()) for t in texts]
        if not model.names:
            return [RouteDecision(None, None, NO_ADAPTERS if ok else NO_TEXT) for ok in has_text]
        wanted = [t for t, ok in zip(texts, has_text) if ok]
        embs = iter(self.encoder.encode(wanted) if wanted else ())
        return [self._decide(model, next(embs)) if ok else RouteDecision(None, None, NO_TEXT)
                for ok in has_text]

    def route_embeddings(self, embs: list) -> list[RouteDecision]:
        self.requests += len(embs)
        model = self.model
        return [RouteDecision(None, None, UNAVAILABLE) if e is None else
                RouteDecision(None, None, NO_ADAPTERS) if not model.names else self._decide(model, e)
                for e in embs]

    def route(self, text: str | None) -> RouteDecision:
        return self.route_many([text])[0]
