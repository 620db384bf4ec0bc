"""Adapter centroids and the resumable indexing job.

An adapter is placed for routing by one unit vector, its *centroid*: the
re-normalised mean of the unit embeddings of its training inputs, plus a few
*reference samples* (the embeddings of inputs at evenly spaced positions of
the sample list) that calibrate the routing confidence later. The centroid
definition and the reference-sample placement are the reference's
(``deltaserve-plugin/deltaserve/adapter_routing/index.py``); the data layout,
the job's state and the file formats here are this package's own.

* :class:`CentroidIndex` holds one record per adapter in insertion order and
  builds the stacked centroid matrix only when it is asked for it (scoring a
  query is one matrix-vector product);
* :class:`Indexer` is the job: the sample list is consumed in chunks whose
  embeddings are folded into a float64 sum. Its state -- position, rows seen,
  the sum, the reference rows met so far -- is checkpointed after every
  accepted chunk; a chunk whose embeddings never come back is simply handed
  out again, and a restart with the same samples and encoder (same
  fingerprint) continues at the checkpoint.
"""

from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass, field

import numpy as np


def l2_normalize(x) -> np.ndarray:
    """Rows of ``x`` scaled to unit length (all-zero rows stay zero)."""
    x = np.asarray(x)
    norm = np.sqrt((x * x).sum(axis=-1, keepdims=True))
    return np.divide(x, norm, out=np.zeros_like(x, dtype=np.result_type(x, np.float32)), where=norm > 0)


def _write_npz(path: str, **arrays) -> None:
    """``np.savez`` into a sibling file, then one rename over ``path``."""
    folder = os.path.dirname(os.path.abspath(path))
    os.makedirs(folder, exist_ok=True)
    part = os.path.join(folder, f".{os.path.basename(path)}.{os.getpid()}.part.npz")
    np.savez(part, **arrays)
    os.replace(part, path)


def select_samples(data_path: str, max_samples: int, seed: int = 0,
                   input_until: str | None = None) -> list[str]:
    """The inputs a centroid is built from: one sample per non-blank corpus
    line, cut before ``input_until`` when given (a served request carries only
    that part), and at most ``max_samples`` of them, drawn without
    replacement by a seeded generator when the corpus is larger."""
    with open(data_path, encoding="utf-8") as f:
        raw = f.read().splitlines()
    inputs = []
    for line in raw:
        text = line.partition(input_until)[0] if input_until else line
        text = text.strip()
        if text:
            inputs.append(text)
    if len(inputs) <= max_samples:
        return inputs
    order = np.random.default_rng(seed).permutation(len(inputs))
    return [inputs[i] for i in order[:max_samples]]


def fingerprint(texts: list[str], encoder: str, prefix: str, max_tokens: int) -> str:
    """Identity of an indexing job: the encoder settings and every sample,
    each field length-prefixed so that no two different jobs hash alike."""
    h = hashlib.blake2b(digest_size=32)
    for part in (encoder, prefix, str(int(max_tokens)), str(len(texts)), *texts):
        b = part.encode("utf-8", "replace")
        h.update(len(b).to_bytes(8, "little"))
        h.update(b)
    return h.hexdigest()


# ---------------------------------------------------------------- the job
@dataclass
class _Progress:
    pos: int = 0                        # next sample to hand out
    seen: int = 0                       # rows folded into ``acc``
    acc: np.ndarray | None = None       # float64 sum of unit embeddings
    ref_rows: dict = field(default_factory=dict)    # reference slot -> unit embedding


class Indexer:
    """One adapter's indexing job over ``texts``, resumable chunk by chunk."""

    def __init__(self, texts: list[str], fp: str, checkpoint_path: str | None = None,
                 reference_samples: int = 0):
        self.texts = list(texts)
        self.fp = fp
        self.checkpoint_path = checkpoint_path
        n = len(self.texts)
        want = min(max(int(reference_samples), 0), n)
        # positions of the reference samples: evenly spread, first and last included
        self._ref_pos = (np.unique(np.rint(np.linspace(0, n - 1, want)).astype(np.int64))
                         if want else np.zeros(0, np.int64))
        self._p = _Progress()
        self.resumed_from = 0
        if checkpoint_path and os.path.exists(checkpoint_path):
            self._load(checkpoint_path)

    # state ---------------------------------------------------------------
    @property
    def cursor(self) -> int:
        return self._p.pos

    @property
    def count(self) -> int:
        return self._p.seen

    @property
    def done(self) -> bool:
        return self._p.pos >= len(self.texts)

    @property
    def progress(self) -> tuple[int, int]:
        return self._p.pos, len(self.texts)

    def _save(self) -> None:
        slots = np.array(sorted(self._p.ref_rows), np.int64)
        rows = (np.stack([self._p.ref_rows[s] for s in slots]).astype(np.float32) if len(slots)
                else np.zeros((0, 0), np.float32))
        _write_npz(self.checkpoint_path, job=np.array([self.fp]),
                   counters=np.array([self._p.pos, self._p.seen, len(self.texts), len(self._ref_pos)], np.int64),
                   acc=self._p.acc if self._p.acc is not None else np.zeros(0),
                   ref_slots=slots, ref_rows=rows)

    def _load(self, path: str) -> None:
        try:
            with np.load(path, allow_pickle=False) as z:
                job = str(z["job"][0])
                pos, seen, total, n_refs = (int(v) for v in z["counters"])
                acc, slots, rows = z["acc"], z["ref_slots"], z["ref_rows"]
        except (OSError, KeyError, ValueError, IndexError):
            return
        if job != self.fp or total != len(self.texts) or n_refs != len(self._ref_pos) or not 0 <= pos <= total:
            return                         # another dataset, encoder or reference setting: start over
        self._p = _Progress(pos, seen, acc.astype(np.float64) if acc.size else None,
                            {int(s): rows[i].astype(np.float32) for i, s in enumerate(slots)})
        self.resumed_from = pos

    # chunks --------------------------------------------------------------
    def next_chunk(self, n: int) -> tuple[int, list[str]]:
        """``(start, texts)`` of the next chunk; the same until it is committed."""
        start = self._p.pos
        return start, self.texts[start:start + max(1, int(n))]

    def commit(self, start: int, embeddings) -> bool:
        """Fold in the embeddings of the chunk starting at ``start``. Anything
        but the current chunk (a late result of an abandoned one) is refused
        and changes nothing."""
        e = np.asarray(embeddings, np.float64)
        if start != self._p.pos or e.ndim != 2 or e.shape[0] == 0 or start + e.shape[0] > len(self.texts):
            return False
        u = l2_normalize(e)
        end = start + u.shape[0]
        lo, hi = np.searchsorted(self._ref_pos, [start, end])
        for slot in range(int(lo), int(hi)):
            self._p.ref_rows[slot] = u[int(self._ref_pos[slot]) - start].astype(np.float32)
        total = u.sum(axis=0)
        self._p.acc = total if self._p.acc is None else self._p.acc + total
        self._p.seen += u.shape[0]
        self._p.pos = end
        if self.checkpoint_path:
            self._save()
        return True

    # results -------------------------------------------------------------
    def centroid(self) -> np.ndarray:
        if not self.done or self._p.acc is None:
            raise RuntimeError("indexing is not finished")
        return l2_normalize(self._p.acc / self._p.seen).astype(np.float32)

    def references(self) -> np.ndarray | None:
        if not self.done:
            raise RuntimeError("indexing is not finished")
        if not self._p.ref_rows:
            return None
        return np.stack([self._p.ref_rows[s] for s in sorted(self._p.ref_rows)]).astype(np.float32)


# ---------------------------------------------------------------- the index
class CentroidIndex:
    """The routable adapters: per name a unit centroid and optional reference
    samples, tagged with the encoder settings (``encoder``, ``prefix``,
    ``max_tokens``) that produced them."""

    def __init__(self, encoder: str = "", prefix: str = "", max_tokens: int = 0):
        self.encoder, self.prefix, self.max_tokens = encoder, prefix, int(max_tokens)
        self._cent: dict[str, np.ndarray] = {}
        self._refs: dict[str, np.ndarray] = {}
        self._stacked: np.ndarray | None = None

    def __len__(self) -> int:
        return len(self._cent)

    def __contains__(self, name: str) -> bool:
        return name in self._cent

    @property
    def names(self) -> list[str]:
        return list(self._cent)

    @property
    def refs(self) -> dict[str, np.ndarray]:
        return self._refs

    @property
    def dim(self) -> int:
        return next(iter(self._cent.values())).shape[0] if self._cent else 0

    @property
    def matrix(self) -> np.ndarray:
        """``[len, dim]`` float32 centroids in ``names`` order."""
        if self._stacked is None:
            self._stacked = (np.stack(list(self._cent.values())) if self._cent
                             else np.zeros((0, 0), np.float32))
        return self._stacked

    def add(self, name: str, centroid, refs=None) -> None:
        """Insert or replace ``name`` (a replaced adapter keeps its position)."""
        c = l2_normalize(np.asarray(centroid, np.float32).reshape(-1)).astype(np.float32)
        others = [v for k, v in self._cent.items() if k != name]
        if others and c.shape[0] != others[0].shape[0]:
            raise ValueError(f"centroid dim {c.shape[0]} != index dim {others[0].shape[0]}")
        self._cent[name] = c
        if refs is not None and len(refs):
            self._refs[name] = np.asarray(refs, np.float32)
        else:
            self._refs.pop(name, None)
        self._stacked = None

    def remove(self, name: str) -> bool:
        if self._cent.pop(name, None) is None:
            return False
        self._refs.pop(name, None)
        self._stacked = None
        return True

    def centroid_of(self, name: str) -> np.ndarray:
        return self._cent[name].copy()

    def scores(self, embedding) -> np.ndarray:
        """Cosine of one embedding with every centroid, in ``names`` order."""
        if not self._cent:
            return np.zeros(0, np.float32)
        return self.matrix @ l2_normalize(np.asarray(embedding, np.float32).reshape(-1))

    def snapshot(self) -> "CentroidIndex":
        """An independent copy: later changes to this index do not reach it."""
        snap = CentroidIndex(self.encoder, self.prefix, self.max_tokens)
        snap._cent = {n: c.copy() for n, c in self._cent.items()}
        snap._refs = {n: r.copy() for n, r in self._refs.items()}
        return snap

    # file: tag [encoder, prefix, max_tokens], names, centroids, per-name
    # reference row counts and all reference rows concatenated
    def save(self, path: str) -> None:
        names = self.names
        counts = np.array([len(self._refs.get(n, ())) for n in names], np.int64)
        rows = [self._refs[n] for n in names if n in self._refs]
        _write_npz(path, tag=np.array([self.encoder, self.prefix, str(self.max_tokens)]),
                   names=np.array(names, dtype=np.str_), centroids=self.matrix,
                   ref_counts=counts,
                   ref_data=np.concatenate(rows).astype(np.float32) if rows else np.zeros((0, 0), np.float32))

    @classmethod
    def load_or_none(cls, path: str) -> "CentroidIndex | None":
        """:meth:`load`, or None when the file is missing or not an index of
        this layout (a cache written by another version is rebuilt)."""
        try:
            return cls.load(path)
        except (OSError, KeyError, ValueError):
            return None

    @classmethod
    def load(cls, path: str) -> "CentroidIndex":
        with np.load(path, allow_pickle=False) as z:
            enc, prefix, max_tokens = (str(v) for v in z["tag"])
            idx = cls(enc, prefix, int(max_tokens))
            names = [str(n) for n in z["names"]]
            cents = z["centroids"].astype(np.float32)
            counts = z["ref_counts"]
            data = z["ref_data"].astype(np.float32)
        bounds = np.concatenate([[0], np.cumsum(counts)])
        for i, n in enumerate(names):
            idx._cent[n] = cents[i]
            if counts[i]:
                idx._refs[n] = data[bounds[i]:bounds[i + 1]]
        return idx
