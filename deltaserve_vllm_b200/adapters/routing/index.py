"""Adapter centroids and the resumable indexing job.

An adapter's centroid is the re-normalised mean of the unit embeddings of its
training inputs. Indexing keeps a running sum, so its whole state is
``(sum, count, cursor)`` plus a handful of *reference samples* (embeddings of
samples at evenly spaced positions) that later calibrate the routing
confidence. The state is checkpointed after every committed chunk; a chunk
whose result never arrives is simply handed out again, and a restart resumes
at the checkpoint if the dataset and encoder are unchanged (fingerprint).

Behaviour follows ``deltaserve-plugin/deltaserve/adapter_routing/index.py:1-267``
(centroid definition, reference-sample placement, resumable chunks); the file
layout is this package's own.
"""

from __future__ import annotations

import hashlib
import json
import os

import numpy as np


def l2_normalize(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x)
    n = np.linalg.norm(x, axis=-1, keepdims=True)
    return x / np.maximum(n, 1e-30) * (n > 0)


def _save_npz(path: str, **arrays) -> None:
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + ".partial.npz"
    np.savez(tmp, **arrays)
    os.replace(tmp, path)


def select_samples(data_path: str, max_samples: int, seed: int = 0,
                   input_until: str | None = None) -> list[str]:
    """The texts a centroid is built from: non-empty corpus lines (one sample
    per line), cut at ``input_until`` (requests carry only the input part),
    at most ``max_samples`` of them in a seeded random order."""
    with open(data_path, encoding="utf-8") as f:
        lines = [ln.strip() for ln in f]
    if input_until:
        lines = [ln.split(input_until, 1)[0].strip() for ln in lines]
    lines = [ln for ln in lines if ln]
    if len(lines) > max_samples:
        keep = np.random.default_rng(seed).permutation(len(lines))[:max_samples]
        lines = [lines[i] for i in keep]
    return lines


def fingerprint(texts: list[str], encoder: str, prefix: str, max_tokens: int) -> str:
    """Identity of an indexing job: the samples and the encoder settings."""
    h = hashlib.sha256(json.dumps([encoder, prefix, int(max_tokens), len(texts)]).encode())
    for t in texts:
        h.update(t.encode("utf-8", "replace") + b"\0")
    return h.hexdigest()


class Indexer:
    """One adapter's indexing job, resumable chunk by chunk."""

    def __init__(self, texts: list[str], fp: str, checkpoint_path: str | None = None,
                 reference_samples: int = 0):
        self.texts = list(texts)
        self.fp = fp
        self.checkpoint_path = checkpoint_path
        n = len(self.texts)
        k = max(0, min(int(reference_samples), n))
        pos = sorted(set(np.linspace(0, n - 1, k).round().astype(int).tolist())) if k else []
        self._ref_slot = {p: i for i, p in enumerate(pos)}
        self.cursor, self.count = 0, 0
        self.sum: np.ndarray | None = None
        self.refs: np.ndarray | None = None
        self.resumed_from = 0
        if checkpoint_path and os.path.exists(checkpoint_path):
            self._resume(checkpoint_path)

    def _resume(self, path: str) -> None:
        try:
            with np.load(path, allow_pickle=False) as z:
                fp = str(z["fp"])
                cursor, count, total = (int(v) for v in z["progress"])
                s = z["sum"]
                refs = z["refs"]
        except (OSError, KeyError, ValueError):
            return
        if fp != self.fp or total != len(self.texts) or not 0 <= cursor <= total:
            return                                   # another dataset / encoder
        if cursor > 0 and refs.shape[0] != len(self._ref_slot):
            return                                   # another reference setting
        self.cursor, self.count = cursor, count
        self.sum = s.astype(np.float64) if s.size else None
        self.refs = refs.astype(np.float32) if refs.size else None
        self.resumed_from = cursor

    @property
    def done(self) -> bool:
        return self.cursor >= len(self.texts)

    @property
    def progress(self) -> tuple[int, int]:
        return self.cursor, len(self.texts)

    def next_chunk(self, n: int) -> tuple[int, list[str]]:
        """The next ``n`` texts and their start position; repeated until committed."""
        return self.cursor, self.texts[self.cursor:self.cursor + max(1, int(n))]

    def commit(self, start: int, embeddings) -> bool:
        """Fold in one chunk's embeddings. A chunk that is not the current one
        (a late result of an abandoned chunk) is refused and changes nothing."""
        e = np.asarray(embeddings, np.float64)
        if start != self.cursor or e.ndim != 2 or not len(e) or start + len(e) > len(self.texts):
            return False
        e = l2_normalize(e)
        if self._ref_slot:
            if self.refs is None:
                self.refs = np.zeros((len(self._ref_slot), e.shape[1]), np.float32)
            for j in range(len(e)):
                slot = self._ref_slot.get(start + j)
                if slot is not None:
                    self.refs[slot] = e[j]
        self.sum = e.sum(0) if self.sum is None else self.sum + e.sum(0)
        self.count += len(e)
        self.cursor += len(e)
        if self.checkpoint_path:
            _save_npz(self.checkpoint_path, fp=np.array(self.fp),
                      progress=np.array([self.cursor, self.count, len(self.texts)], np.int64),
                      sum=self.sum if self.sum is not None else np.zeros(0),
                      refs=self.refs if self.refs is not None else np.zeros((0, 0), np.float32))
        return True

    def centroid(self) -> np.ndarray:
        if not self.done or self.sum is None:
            raise RuntimeError("indexing is not finished")
        return l2_normalize(self.sum / self.count).astype(np.float32)

    def references(self) -> np.ndarray | None:
        if not self.done:
            raise RuntimeError("indexing is not finished")
        return None if self.refs is None else self.refs.copy()


class CentroidIndex:
    """One unit centroid per routable adapter (+ optional reference samples),
    tagged with the encoder settings that produced them."""

    def __init__(self, encoder: str = "", prefix: str = "", max_tokens: int = 0):
        self.encoder, self.prefix, self.max_tokens = encoder, prefix, int(max_tokens)
        self.names: list[str] = []
        self.matrix = np.zeros((0, 0), np.float32)
        self.refs: dict[str, np.ndarray] = {}

    def __len__(self) -> int:
        return len(self.names)

    def __contains__(self, name: str) -> bool:
        return name in self.names

    @property
    def dim(self) -> int:
        return int(self.matrix.shape[1]) if len(self.names) else 0

    def add(self, name: str, centroid, refs=None) -> None:
        c = l2_normalize(np.asarray(centroid, np.float32).reshape(-1)).astype(np.float32)
        if self.names and c.shape[0] != self.dim:
            raise ValueError(f"centroid dim {c.shape[0]} != index dim {self.dim}")
        if refs is not None and len(refs):
            self.refs[name] = np.asarray(refs, np.float32)
        else:
            self.refs.pop(name, None)
        if name in self.names:
            self.matrix[self.names.index(name)] = c
        else:
            self.matrix = c[None] if not self.names else np.vstack([self.matrix, c[None]])
            self.names.append(name)

    def remove(self, name: str) -> bool:
        if name not in self.names:
            return False
        i = self.names.index(name)
        del self.names[i]
        self.matrix = np.delete(self.matrix, i, axis=0)
        self.refs.pop(name, None)
        return True

    def centroid_of(self, name: str) -> np.ndarray:
        return self.matrix[self.names.index(name)].copy()

    def scores(self, embedding) -> np.ndarray:
        """Cosine of one embedding with every centroid (``names`` order)."""
        if not self.names:
            return np.zeros(0, np.float32)
        e = l2_normalize(np.asarray(embedding, np.float32).reshape(-1))
        return self.matrix @ e

    def route(self, embedding, threshold: float = -1.0) -> tuple[str | None, float]:
        """Plain top-1 (no confidence gating): (adapter or None, best cosine)."""
        s = self.scores(embedding)
        if not s.size:
            return None, float("nan")
        i = int(np.argmax(s))
        return (self.names[i] if s[i] >= threshold else None), float(s[i])

    def save(self, path: str) -> None:
        with_refs = [n for n in self.names if n in self.refs]
        meta = {"encoder": self.encoder, "prefix": self.prefix, "max_tokens": self.max_tokens,
                "names": self.names, "with_refs": with_refs}
        _save_npz(path, meta=np.array(json.dumps(meta)), matrix=self.matrix,
                  **{f"refs{i}": self.refs[n] for i, n in enumerate(with_refs)})

    @classmethod
    def load(cls, path: str) -> "CentroidIndex":
        with np.load(path, allow_pickle=False) as z:
            meta = json.loads(str(z["meta"]))
            idx = cls(meta["encoder"], meta["prefix"], meta["max_tokens"])
            idx.names = list(meta["names"])
            idx.matrix = z["matrix"].astype(np.float32)
            for i, n in enumerate(meta.get("with_refs", [])):
                idx.refs[n] = z[f"refs{i}"].astype(np.float32)
        return idx
