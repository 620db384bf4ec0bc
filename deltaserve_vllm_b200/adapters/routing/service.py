"""Adapter routing inside the engine: pool + router + the engine's LoRA slots.

Requests for the routing model name (or for a pool adapter by name) go
through :meth:`AdapterRouter.submit`, which queues them. At the start of
every engine step :meth:`AdapterRouter.tick` runs the *encode step*: all
queued texts are embedded in one encoder call, decided, and each request
either enters the scheduler at once (base model, or its adapter already holds
a GPU slot) or is *held* until the pool can give its adapter a slot (evicting
the least-used slot holder that no running request uses). The request keeps
its real arrival time throughout, so TTFT includes the hold.

With ``route_encode_async`` (default) the encoder call runs on a worker
thread: ``tick`` hands the batch over and applies its decisions on the first
tick after they are ready, so the engine keeps stepping (and its GPU work
keeps flowing) while the encoder tokenizes and runs; at most one batch is in
flight and the next one collects the requests that arrived meanwhile.

Reference: ``deltaserve-plugin/deltaserve/adapter_routing/engine.py:37-391``
and ``engine_router.py:178-380`` (held routed requests, encode step, slot
placement), re-built around this engine's own slot table.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import time
from collections import deque

from ... import dprint
from .. import peft_io
from .encoder import SentenceEncoder, encoder_identity, make_encoder
from .index import CentroidIndex
from .indexing import index_dir, make_indexing_service, prepare_indexing, store_centroid
from .pool import GPU, AdapterPool
from .router import NO_TEXT, RouteDecision, Router


class EngineSlotBackend:
    """Pool tiers mapped onto the engine: ``cpu`` = host tensors read from
    the PEFT directory, ``gpu`` = a LoRA slot of the engine."""

    def __init__(self, engine):
        self.eng = engine
        self.host: dict[str, tuple] = {}

    def load(self, e) -> None:
        tensors, acfg = peft_io.read_adapter(e.path)
        rank, alpha = peft_io.adapter_rank_alpha(acfg)
        self.host[e.name] = (tensors, rank, alpha)

    def activate(self, e) -> None:
        if e.name not in self.host:
            self.load(e)
        tensors, rank, alpha = self.host[e.name]
        self.eng.load_inference_adapter(e.name, path=e.path, tensors=tensors, rank=rank, alpha=alpha)

    def deactivate(self, e) -> None:
        if e.name in self.eng.adapter_slots:
            self.eng.unload_inference_adapter(e.name)

    def unload(self, e) -> None:
        self.host.pop(e.name, None)


class AdapterRouter:
    def __init__(self, engine, cfg, backend=None):
        self.eng, self.cfg = engine, cfg
        dev = str(engine.device) if getattr(engine, "cuda", False) else "cpu"
        self.encoder = make_encoder(cfg, dev)
        # Indexing encodes in processes of its own (started with the first
        # job): a CPU copy of the encoder, and a GPU process on the route
        # encoder's own weights while the engine is idle.
        self.index_encoder = (make_encoder(cfg, "cpu") if isinstance(self.encoder, SentenceEncoder)
                              else self.encoder)
        self.indexer_service = None
        self.enc_id = encoder_identity(self.encoder)
        self.dir = index_dir(cfg)
        used = set(engine.adapter_slots.values())
        free = (engine.lora.slots - len(used)) if engine.lora is not None else 0
        if free < 1:
            raise RuntimeError("adapter routing needs at least one free LoRA slot (raise max_loras)")
        self.pool = AdapterPool(
            backend or EngineSlotBackend(engine),
            CentroidIndex(self.enc_id, cfg.encoder_query_prefix, cfg.encoder_max_tokens),
            capacity=cfg.max_active_adapters, gpu_slots=free, protected=cfg.pool_protected_slots,
            half_life_s=cfg.pool_hit_half_life_s, directory=os.path.join(self.dir, "pool"),
            when_full=cfg.when_full, grace_s=cfg.retire_grace_s, min_pool=cfg.route_min_pool,
            min_self_recall=cfg.admission_min_self_recall, max_stolen=cfg.admission_max_stolen)
        log = os.path.join(self.dir, "decisions.jsonl") if cfg.route_decision_log else None
        self.router = Router(self.encoder, cfg.route_keep_percent, cfg.route_close_band, cfg.route_min_pool,
                             cfg.route_confidence_slack, cfg.fallback_score_threshold, log,
                             tier_of=lambda n: self.pool.entries[n].tier if n in self.pool.entries else "")
        self.pool.listeners.append(lambda p: self.router.set_index(p.index))
        self.pending: deque = deque()   # (rid, ids, params, text, adapter, arrival, future)
        self._encode_pool = (cf.ThreadPoolExecutor(1, thread_name_prefix="dsv-route-encode")
                             if cfg.route_encode_async else None)
        self._inflight = None           # (batch, future of the decisions, t0) of the async encode step
        self._cancelled: set = set()    # requests cancelled while their batch is being encoded
        self.held: deque = deque()      # (rid, ids, params, adapter, arrival)
        self.indexing: dict[str, tuple] = {}     # name -> (job, path, fingerprint)
        engine.request_listeners.append(self._on_request)
        self.stats = {"routed": 0, "fallback": 0, "held": 0, "encode_calls": 0, "encode_ms": 0.0}
        for a in cfg.adapters or []:
            self.add(a.get("name") or os.path.basename(os.path.normpath(a["path"])), a["path"],
                     data_path=a.get("data_path"), centroid_path=a.get("centroid_path"),
                     prewarm=bool(a.get("prewarm", False)))

    # ------------------------------------------------------------ pool entry
    def add(self, name: str, path: str, data_path: str | None = None, centroid_path: str | None = None,
            prewarm: bool = False) -> dict:
        """Put an adapter in the pool: with a saved centroid it is admitted
        at once; with a dataset it is indexed in the background (servable by
        name meanwhile) and admitted when the centroid is ready."""
        if centroid_path:
            idx = CentroidIndex.load(centroid_path)
            src = name if name in idx else (idx.names[0] if len(idx) == 1 else None)
            if src is None:
                raise KeyError(f"{centroid_path} has no centroid for '{name}'")
            return self.pool.admit(name, path, idx.centroid_of(src), idx.refs.get(src), load=True,
                                   prewarm=prewarm)
        if name not in self.pool:
            self.pool.register(name, path, load=True, prewarm=prewarm)
        if data_path:
            return self.start_indexing(name, path, data_path)
        return {"name": name, "level": self.pool.entries[name].level, "indexed": False}

    def start_indexing(self, name: str, path: str, data_path: str) -> dict:
        job, hit = self.index_job(name, data_path)
        if hit is not None:
            return self.pool.admit(name, path, hit[0], hit[1], load=True)
        self.indexing[name] = (job, path, job.fp)
        return {"name": name, "indexing": job.describe()}

    def index_job(self, name: str, data_path: str):
        """(indexing job, None) or (None, cached (centroid, refs)); the job
        carries its fingerprint as ``job.fp``."""
        ix, hit, fp = prepare_indexing(self.cfg, self.enc_id, name, data_path)
        if hit is not None:
            return None, hit
        if self.indexer_service is None:
            self.indexer_service = make_indexing_service(self.cfg, self.index_encoder, self.encoder)
            if self.eng.has_unfinished():
                self.indexer_service.placement.note_inference()
        job = self.indexer_service.submit(name, ix)
        job.fp = fp
        return job, None

    def _on_request(self, what: str, _req) -> None:
        if what == "add" and self.indexer_service is not None:
            self.indexer_service.placement.note_inference()

    def _poll_indexing(self) -> None:
        for name, (job, path, fp) in list(self.indexing.items()):
            if job.error:
                dprint(f"[indexing] {name} failed: {job.error}")
                del self.indexing[name]
            elif job.done:
                del self.indexing[name]
                c, r = job.indexer.centroid(), job.indexer.references()
                store_centroid(self.dir, name, fp, c, r, self.enc_id, self.cfg.encoder_query_prefix,
                               self.cfg.encoder_max_tokens)
                if name in self.pool:
                    self.pool.admit(name, path, c, r)

    def centroid_ready(self, name: str) -> bool:
        e = self.pool.entries.get(name)
        return e is not None and e.centroid is not None

    def names(self) -> list[str]:
        return self.pool.names()

    # ------------------------------------------------------------ requests
    def submit(self, rid: str, ids: list[int], params, text: str | None = None,
               adapter: str | None = None, arrival: float | None = None) -> cf.Future:
        """Queue a routed request (``adapter`` None: decide from ``text``) or
        a request naming a pool adapter. The future resolves with the
        :class:`RouteDecision` at the next encode step."""
        fut: cf.Future = cf.Future()
        if self.indexer_service is not None:
            self.indexer_service.placement.note_inference()
        self.pending.append((rid, list(ids), params, text, adapter,
                             arrival if arrival is not None else time.perf_counter(), fut))
        self.eng.arrival_flag = True
        return fut

    def has_pending(self) -> bool:
        return bool(self.pending or self.held or self._inflight is not None)

    def cancel(self, rid: str) -> bool:
        """Drop a request still waiting for its route decision or for its
        adapter's slot (its client went away)."""
        for q in (self.pending, self.held):
            for item in list(q):
                if item[0] == rid:
                    q.remove(item)
                    if q is self.pending and not item[-1].done():
                        item[-1].cancel()
                    return True
        if self._inflight is not None and any(item[0] == rid for item in self._inflight[0]):
            self._cancelled.add(rid)    # dropped when its batch's decisions are applied
            return True
        return False

    def _in_use(self) -> set[str]:
        return {r.adapter for r in self.eng.requests.values() if r.adapter}

    def _enter(self, rid, ids, params, adapter, arrival) -> None:
        self.eng.add_request(rid, ids, params, adapter, arrival_time=arrival)

    def tick(self) -> None:
        """The encode step plus slot placement; runs on the engine thread."""
        if self.indexer_service is not None and (self.pending or self.held or self.eng.scheduler.has_unfinished()):
            self.indexer_service.placement.note_inference()
        if self.indexing:
            self._poll_indexing()
        if self._inflight is not None and self._inflight[1].done():
            batch, fut_dec, t0 = self._inflight
            self._inflight = None
            try:
                decisions = fut_dec.result()
            except Exception as e:  # the encoder failed: every request of the batch gets the error
                for item in batch:
                    self._cancelled.discard(item[0])
                    if not item[-1].done():
                        item[-1].set_exception(e)
                decisions = None
            if decisions is not None:
                self._apply(batch, decisions, t0)
        if self.pending and self._inflight is None:
            batch = list(self.pending)
            self.pending.clear()
            texts = [b[3] for b in batch if b[4] is None]
            t0 = time.perf_counter()
            if texts and self._encode_pool is not None:
                self._inflight = (batch, self._encode_pool.submit(self.router.route_many, texts), t0)
            else:
                self._apply(batch, self.router.route_many(texts) if texts else [], t0)
        if self.held:
            keep = deque()
            while self.held:
                rid, ids, params, adapter, arrival = self.held.popleft()
                if adapter not in self.pool:
                    self._enter(rid, ids, params, None, arrival)        # removed meanwhile
                elif self.pool.ensure_gpu(adapter, self._in_use()):
                    self._enter(rid, ids, params, adapter, arrival)
                else:
                    keep.append((rid, ids, params, adapter, arrival))
            self.held = keep

    def _apply(self, batch, decisions, t0: float) -> None:
        """Enter, hold or fall back every request of an encoded batch."""
        if any(b[4] is None for b in batch):
            self.stats["encode_calls"] += 1
            self.stats["encode_ms"] += (time.perf_counter() - t0) * 1e3
        it = iter(decisions)
        for rid, ids, params, text, named, arrival, fut in batch:
            d = RouteDecision(named) if named is not None else next(it)
            if rid in self._cancelled:
                self._cancelled.discard(rid)
                if not fut.done():
                    fut.cancel()
                continue
            try:
                if d.adapter is None:
                    self.stats["fallback"] += 1
                    self._enter(rid, ids, params, None, arrival)
                else:
                    self.stats["routed"] += 1
                    self.pool.note_hit(d.adapter, self._in_use(), place=True)
                    if self.pool.entries[d.adapter].tier == GPU:
                        self._enter(rid, ids, params, d.adapter, arrival)
                    else:
                        self.stats["held"] += 1
                        self.held.append((rid, ids, params, d.adapter, arrival))
                fut.set_result(d)
            except Exception as e:  # reported to the HTTP handler
                fut.set_exception(e)

    def status(self) -> dict:
        return {"pool": self.pool.status(), "model": self.router.model.describe(),
                "pending": len(self.pending), "held": len(self.held), "stats": dict(self.stats),
                "indexing": {n: j.describe() for n, (j, _, _) in self.indexing.items()},
                "indexer": self.indexer_service.describe() if self.indexer_service is not None else None}

    def stop(self) -> None:
        if self._encode_pool is not None:
            self._encode_pool.shutdown(wait=True)
            self._encode_pool = None
        for job, _, _ in self.indexing.values():
            job.stop()
        if self.indexer_service is not None:
            self.indexer_service.stop()
            self.indexer_service = None


NO_TEXT_DECISION = RouteDecision(None, None, NO_TEXT)
