"""Adapter routing: a request sent to the routing model name (``auto``) is
served by the pool adapter whose training data it resembles most, or by the
base model when no adapter is a confident match.

* ``index``     — per-adapter centroids (mean unit embedding of its training
  inputs) plus a few reference-sample embeddings; resumable indexing;
* ``decision``  — centred-score + margin confidence, keep-percent threshold,
  close band; admission report for a candidate adapter;
* ``encoder``   — sentence encoders (a local HF encoder, or an offline hashing
  encoder when no encoder weights are on disk);
* ``pool``      — tiers gpu / cpu / disk, active / retired, decayed-hit GPU
  slot policy, admission rules, persistent registry;
* ``router``    — index + decision model -> ``RouteDecision`` and headers;
* ``engine``    — the pool wired to the engine's LoRA slots, the encode step
  and held requests;
* ``stages``    — the ``indexing`` and ``admission`` finetuning-job stages.

Reference: ``deltaserve-plugin/deltaserve/adapter_routing/`` (3.2k lines) and
``deltaserve-plugin/deltaserve/route_middleware.py``.
"""

from .service import AdapterRouter  # noqa: E402

__all__ = ["AdapterRouter"]
