"""Background indexing: build an adapter's centroid from its dataset on a
host thread while the engine serves, and the on-disk centroid cache that
lets a restart (or the same dataset listed again) skip encoding.

The reference runs a CPU indexer process under ``SCHED_IDLE`` and moves to a
GPU executor after a quiet period
(``deltaserve-plugin/deltaserve/adapter_routing/runner.py:40-230``). Here the
indexer is a daemon thread: the serving loop spends its host time waiting on
the GPU, so a thread that encodes smaller chunks (and yields between them)
while requests are in flight costs the serving path little, and larger
chunks when the engine is idle.
"""

from __future__ import annotations

import json
import os
import tempfile
import threading
import time

from ... import dprint
from .index import CentroidIndex, Indexer, fingerprint, select_samples

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
    path = os.path.join(directory, CENTROIDS_FILE)
    if not os.path.exists(path):
        return None
    idx = CentroidIndex.load(path)
    if name not in idx:
        return None
    return idx.centroid_of(name), idx.refs.get(name)


def store_centroid(directory: str, name: str, fp: str, centroid, refs, enc_id: str, prefix: str,
                   max_tokens: int) -> None:
    with _CACHE_LOCK:
        os.makedirs(directory, exist_ok=True)
        path = os.path.join(directory, CENTROIDS_FILE)
        idx = CentroidIndex.load(path) if os.path.exists(path) else CentroidIndex(enc_id, prefix, max_tokens)
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


class IndexingRunner:
    """Encodes an :class:`Indexer`'s chunks on a daemon thread."""

    def __init__(self, indexer: Indexer, encoder, name: str, chunk_idle: int = 16, chunk_busy: int = 4,
                 busy=lambda: False, busy_pause_s: float = 0.002):
        self.indexer, self.encoder, self.name = indexer, encoder, name
        self.chunk_idle, self.chunk_busy = max(1, int(chunk_idle)), max(1, int(chunk_busy))
        self.busy, self.busy_pause_s = busy, busy_pause_s
        self.error: str | None = None
        self.chunks = 0
        self.t0 = time.time()
        self.t1: float | None = None
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True, name=f"dsv-index-{name}")

    def start(self) -> "IndexingRunner":
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()

    @property
    def done(self) -> bool:
        return self.indexer.done

    def _run(self) -> None:
        try:
            while not self.indexer.done and not self._stop.is_set():
                busy = bool(self.busy())
                start, texts = self.indexer.next_chunk(self.chunk_busy if busy else self.chunk_idle)
                emb = self.encoder.encode(texts)
                self.indexer.commit(start, emb)
                self.chunks += 1
                if busy:
                    time.sleep(self.busy_pause_s)
        except Exception as e:  # reported through the job / pool
            self.error = f"{type(e).__name__}: {e}"
        self.t1 = time.time()

    def describe(self) -> dict:
        done, total = self.indexer.progress
        return {"name": self.name, "done": done, "total": total, "chunks": self.chunks,
                "resumed_from": self.indexer.resumed_from, "error": self.error,
                "seconds": round((self.t1 or time.time()) - self.t0, 3)}


def start_indexing(cfg, encoder, enc_id: str, name: str, data_path: str, busy=lambda: False):
    """(runner or None, cached (centroid, refs) or None, fingerprint)."""
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
    runner = IndexingRunner(ix, encoder, name, cfg.indexing_chunk_samples,
                            max(1, cfg.indexing_chunk_samples // 4), busy=busy).start()
    return runner, None, fp
