"""Background indexing: build an adapter's centroid from its dataset while
the engine serves, and the on-disk centroid cache that lets a restart (or the
same dataset listed again) skip encoding.

* :class:`IndexingPlacement` -- where indexing may run, from the engine's
  inference activity: **busy** while an inference request is present (and
  for ``gpu_after_quiet_s`` after the last one): the GPU is off limits and
  the CPU process gets ``busy_threads``; **idle** otherwise: the GPU process
  may compute and the CPU process gets ``idle_threads``. The engine reports
  activity (:meth:`IndexingPlacement.note_inference`) on every arrival and
  every step that still has requests; the grant byte the GPU process obeys
  is cleared in that same call, so an arrival takes the GPU back at the
  indexer's next encoder layer.
* :class:`IndexingService` -- one thread that runs the indexing jobs in
  arrival order, each chunk on the executor the placement picks (the CPU and
  GPU processes of ``index_process``), one chunk in flight. A GPU chunk cut
  short by an arrival is encoded again on the CPU; a GPU failure moves
  indexing to the CPU for a while.

Reference behaviour: ``deltaserve-plugin/deltaserve/adapter_routing/runner.py:40-230``.
"""

from __future__ import annotations

import json
import os
import tempfile
import threading
import time

from ... import dprint
from .index import CentroidIndex, Indexer, fingerprint, select_samples
from .index_process import Preempted

CENTROIDS_FILE = "centroids.npz"
FINGERPRINTS_FILE = "centroids.json"
_CACHE_LOCK = threading.Lock()


def index_dir(cfg) -> str:
    return cfg.index_path or os.path.join(tempfile.gettempdir(), f"deltaserve-b200-index-{os.getuid()}")


def _fingerprints(directory: str) -> dict:
    try:
        with open(os.path.join(directory, FINGERPRINTS_FILE)) as f:
            d = json.load(f)
        return d if isinstance(d, dict) else {}
    except (OSError, ValueError):
        return {}


def cached_centroid(directory: str, name: str, fp: str):
    """(centroid, refs) of ``name`` if it was built from exactly this data
    and encoder, else None."""
    if _fingerprints(directory).get(name) != fp:
        return None
    idx = CentroidIndex.load_or_none(os.path.join(directory, CENTROIDS_FILE))
    if idx is None or name not in idx:
        return None
    return idx.centroid_of(name), idx.refs.get(name)


def store_centroid(directory: str, name: str, fp: str, centroid, refs, enc_id: str, prefix: str,
                   max_tokens: int) -> None:
    with _CACHE_LOCK:
        os.makedirs(directory, exist_ok=True)
        path = os.path.join(directory, CENTROIDS_FILE)
        idx = CentroidIndex.load_or_none(path) or CentroidIndex(enc_id, prefix, max_tokens)
        if len(idx) and (idx.encoder, idx.prefix, idx.max_tokens) != (enc_id, prefix, int(max_tokens)):
            raise RuntimeError(f"{path} was built with encoder '{idx.encoder}', not '{enc_id}'; "
                               "centroids of different encoders cannot mix")
        idx.add(name, centroid, refs=refs)
        idx.save(path)
        fps = _fingerprints(directory)
        fps[name] = fp
        tmp = os.path.join(directory, FINGERPRINTS_FILE + ".tmp")
        with open(tmp, "w") as f:
            json.dump(fps, f, indent=1)
        os.replace(tmp, os.path.join(directory, FINGERPRINTS_FILE))


IDLE, BUSY = "idle", "busy"


class IndexingPlacement:
    """Busy/idle level of the engine for indexing, and the GPU grant."""

    def __init__(self, gpu_after_quiet_s: float = 3.0, grant=None, idle_threads: int = 8,
                 busy_threads: int = 2, clock=time.monotonic):
        self.gpu_after_quiet_s = float(gpu_after_quiet_s)
        self.grant = grant
        self.idle_threads, self.busy_threads = int(idle_threads), int(busy_threads)
        self.clock = clock
        self._last: float | None = None
        self._level = IDLE
        self.changes = 0
        # The level and the grant change together under this lock: otherwise
        # the indexing thread could set the grant from a stale look just after
        # an arrival cleared it.
        self._lock = threading.Lock()
        if grant is not None:
            grant.set(False)                  # nothing is granted before the first look

    def _apply(self, level: str) -> None:
        if level != self._level:
            self._level = level
            self.changes += 1
        if self.grant is not None and self.grant.granted != (level == IDLE):
            self.grant.set(level == IDLE)

    def note_inference(self) -> None:
        """Inference work is present (an arrival, a step with requests)."""
        with self._lock:
            self._last = self.clock()
            self._apply(BUSY)

    def level(self) -> str:
        with self._lock:
            quiet = self._last is None or self.clock() - self._last >= self.gpu_after_quiet_s
            self._apply(IDLE if quiet else BUSY)
            return self._level

    def cpu_threads(self) -> int:
        return self.idle_threads if self.level() == IDLE else self.busy_threads

    def use_gpu(self, gpu_ready: bool) -> bool:
        return gpu_ready and self.level() == IDLE


class IndexingJob:
    """One adapter's indexing: progress, where its chunks ran, and the outcome."""

    def __init__(self, name: str, indexer: Indexer):
        self.name, self.indexer = name, indexer
        self.state = "pending"                # pending / cpu / gpu / paused / done / failed / stopped
        self.chunks = {"cpu": 0, "gpu": 0}
        self.discarded = self.preempted = 0
        self.error: str | None = None
        self.t0 = time.time()
        self.t1: float | None = None
        self.stopped = False

    @property
    def done(self) -> bool:
        return self.indexer.done and self.state == "done"

    @property
    def finished(self) -> bool:
        return self.state in ("done", "failed", "stopped")

    def stop(self) -> None:
        self.stopped = True

    def describe(self) -> dict:
        done, total = self.indexer.progress
        return {"name": self.name, "state": self.state, "done": done, "total": total,
                "chunks": dict(self.chunks), "discarded": self.discarded, "preempted": self.preempted,
                "resumed_from": self.indexer.resumed_from, "error": self.error,
                "seconds": round((self.t1 or time.time()) - self.t0, 3)}


class IndexingService:
    """Runs indexing jobs on one thread over shared executors.

    ``executors`` maps ``"cpu"`` (required) and optionally ``"gpu"`` to
    executors of :mod:`index_process` (``submit`` / ``poll`` / ``cancel`` /
    ``stop``); ``chunk`` gives the samples per chunk of each."""

    GPU_BACKOFF_S = 30.0

    def __init__(self, executors: dict, placement: IndexingPlacement, chunk: dict | int = 16,
                 poll_s: float = 0.05, recheck_s: float = 0.25):
        if "cpu" not in executors:
            raise ValueError("indexing needs a CPU executor")
        self.executors, self.placement = dict(executors), placement
        self.chunk = chunk if isinstance(chunk, dict) else {d: int(chunk) for d in self.executors}
        self.poll_s, self.recheck_s = float(poll_s), float(recheck_s)
        self.jobs: list[IndexingJob] = []
        self._inflight: tuple[str, int, IndexingJob] | None = None
        self._gpu_off_until = 0.0
        self._wake = threading.Event()
        self._stop = threading.Event()
        self._lock = threading.Lock()
        self._thread = threading.Thread(target=self._loop, daemon=True, name="dsv-indexing")
        self._thread.start()

    def submit(self, name: str, indexer: Indexer) -> IndexingJob:
        job = IndexingJob(name, indexer)
        with self._lock:
            self.jobs.append(job)
        self._wake.set()
        return job

    def _current(self) -> IndexingJob | None:
        with self._lock:
            self.jobs = [j for j in self.jobs if not j.finished]
            return self.jobs[0] if self.jobs else None

    def _device(self) -> str:
        gpu = self.executors.get("gpu")
        ok = gpu is not None and gpu.ready and time.monotonic() >= self._gpu_off_until
        return "gpu" if self.placement.use_gpu(ok) else "cpu"

    def step(self) -> float:
        """One action; returns how long the thread may wait before the next."""
        if self._inflight is not None:
            return self._collect()
        job = self._current()
        if job is None:
            return -1.0                                   # nothing to do: wait for a submit
        if job.stopped:
            job.state, job.t1 = "stopped", time.time()
            return 0.0
        if job.indexer.done:
            job.state, job.t1 = "done", time.time()
            return 0.0
        dev = self._device()
        threads = 0
        if dev == "cpu":
            threads = self.placement.cpu_threads()
            if threads < 1:
                job.state = "paused"
                return self.recheck_s
        job.state = dev
        start, texts = job.indexer.next_chunk(self.chunk.get(dev, 16))
        try:
            self.executors[dev].submit(texts, threads)
        except Exception as e:  # noqa: BLE001
            return self._failed(job, dev, e)
        self._inflight = (dev, start, job)
        return 0.0

    def _collect(self) -> float:
        dev, start, job = self._inflight
        ex = self.executors[dev]
        if dev == "gpu" and self._device() != "gpu":
            # Inference is back: the GPU chunk is abandoned at the child's next
            # layer (its grant is cleared); the samples go to the CPU.
            ex.cancel()
            self._inflight = None
            job.discarded += 1
            return 0.0
        try:
            emb = ex.poll(self.poll_s)
        except Preempted:
            self._inflight = None
            job.preempted += 1
            job.discarded += 1
            return 0.0
        except Exception as e:  # noqa: BLE001
            self._inflight = None
            return self._failed(job, dev, e)
        if emb is None:
            return 0.0
        self._inflight = None
        if job.indexer.commit(start, emb):
            job.chunks[dev] += 1
        else:
            job.discarded += 1
        if job.indexer.done:
            job.state, job.t1 = "done", time.time()
        return 0.0

    def _failed(self, job: IndexingJob, dev: str, e: Exception) -> float:
        if dev == "gpu":
            dprint(f"[indexing] {job.name}: GPU chunk failed ({e}); CPU for {self.GPU_BACKOFF_S:.0f} s")
            self._gpu_off_until = time.monotonic() + self.GPU_BACKOFF_S
            job.discarded += 1
            return 0.0
        job.error = f"{type(e).__name__}: {e}" if not isinstance(e, RuntimeError) else str(e)
        job.state, job.t1 = "failed", time.time()
        return 0.0

    def _loop(self) -> None:
        while not self._stop.is_set():
            try:
                wait = self.step()
            except Exception as e:  # noqa: BLE001 -- a bug here must not end indexing silently
                job = self._inflight[2] if self._inflight else self._current()
                self._inflight = None
                if job is not None:
                    job.error, job.state, job.t1 = f"{type(e).__name__}: {e}", "failed", time.time()
                wait = 0.0
            if wait < 0:
                self._wake.wait(1.0)
                self._wake.clear()
            elif wait > 0:
                self._stop.wait(wait)

    def describe(self) -> dict:
        return {"level": self.placement.level(),
                "executors": {d: ex.describe() for d, ex in self.executors.items()},
                "jobs": [j.describe() for j in list(self.jobs)]}

    def stop(self) -> None:
        self._stop.set()
        self._wake.set()
        self._thread.join(timeout=5.0)
        for ex in self.executors.values():
            try:
                ex.stop()
            except Exception:  # noqa: BLE001
                pass


def make_indexing_service(cfg, index_encoder, route_encoder=None, engine_busy=None) -> IndexingService:
    """The service an :class:`AdapterRouting` config asks for: a CPU process
    (or the in-thread executor when ``indexing_process`` is off) and, with
    ``indexing_on_gpu`` and a route encoder on a CUDA device, the GPU process
    sharing that encoder's weights."""
    from .encoder import SentenceEncoder
    from .index_process import EncoderProcess, IndexGrant, InlineExecutor
    grant = IndexGrant()
    placement = IndexingPlacement(cfg.indexing_gpu_after_quiet_s, grant, cfg.indexing_cpu_max_threads,
                                  cfg.indexing_cpu_busy_threads)
    if cfg.indexing_process:
        cpu = EncoderProcess(index_encoder, "cpu", cpus=cfg.indexing_cpus, name="cpu").start()
    else:
        cpu = InlineExecutor(index_encoder)
    executors = {"cpu": cpu}
    chunk = {"cpu": cfg.indexing_chunk_samples, "gpu": cfg.indexing_gpu_chunk_samples}
    if (cfg.indexing_on_gpu and cfg.indexing_process and isinstance(route_encoder, SentenceEncoder)
            and str(route_encoder.device).startswith("cuda")):
        desc = SentenceEncoder(route_encoder.path, route_encoder.prefix, route_encoder.max_tokens,
                               route_encoder.device)
        try:
            executors["gpu"] = EncoderProcess(desc, route_encoder.device, shared=route_encoder.shared_state(),
                                              grant=grant, low_priority=False, name="gpu").start()
        except Exception as e:  # noqa: BLE001 -- the CPU process still indexes
            dprint(f"[indexing] no GPU indexing process: {e}")
    return IndexingService(executors, placement, chunk)


def prepare_indexing(cfg, enc_id: str, name: str, data_path: str):
    """(Indexer or None, cached (centroid, refs) or None, fingerprint)."""
    texts = select_samples(data_path, cfg.indexing_max_samples, input_until=cfg.indexing_input_until)
    if not texts:
        raise RuntimeError(f"no sample to index in {data_path}")
    texts.sort(key=len)                  # similar lengths per chunk: less padding
    fp = fingerprint(texts, enc_id, cfg.encoder_query_prefix, cfg.encoder_max_tokens)
    d = index_dir(cfg)
    hit = cached_centroid(d, name, fp)
    if hit is not None:
        dprint(f"[indexing] {name}: centroid already built from this dataset")
        return None, hit, fp
    ix = Indexer(texts, fp, os.path.join(d, "checkpoints", f"{name}.npz"),
                 reference_samples=int(cfg.route_reference_samples))
    return ix, None, fp
