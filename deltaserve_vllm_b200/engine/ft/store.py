"""Finetuning sample store: tokenized corpus, length-bucketed selection,
claim / commit / release around in-flight steps, epochs.

Same contract as the reference store (``deltaserve-plugin/deltaserve/finetuning_store.py:51-312``):

* ``pop_best_under(n)`` — the untrained sample with the largest length <= n;
  ``pop_next()`` — the smallest untrained sample (the admission loop goes
  smallest-first); neither marks anything;
* ``claim`` removes samples from the selectable pool for an in-flight step,
  ``commit_claimed`` marks them trained after their backward, and
  ``release_claimed`` puts them back (a pre-empted FT step);
* ``advance_epoch`` refuses while anything is claimed;
* samples longer than the activation buffer are dropped at load (they could
  never be admitted and would wedge admission).
"""

from __future__ import annotations

import uuid
from bisect import bisect_left, bisect_right, insort
from collections import defaultdict, deque
from dataclasses import dataclass
from typing import Callable, Iterable

import numpy as np

from ... import dprint


@dataclass
class FinetuningSample:
    request_id: str
    prompt_ids: list[int]
    text: str = ""
    adapter: str | None = None

    @property
    def input_len(self) -> int:
        return len(self.prompt_ids)


class FinetuningStore:
    def __init__(self, data_path: str | None = None, tokenize: Callable[[str], list[int]] | None = None,
                 adapter: str | None = None, total_epochs: int = 1,
                 max_saved_finetuning_tokens: int = 256, max_prepare: int | None = None):
        self.data_path = data_path
        self.tokenize = tokenize
        self.adapter = adapter
        self.total_epochs = int(total_epochs)
        self.cap = int(max_saved_finetuning_tokens)
        self.max_prepare = max_prepare
        self.samples: list[FinetuningSample] = []
        self.id2idx: dict[str, int] = {}
        self.trained: list[bool] = []
        self.current_epoch = 0
        self.buckets: dict[int, deque] = defaultdict(deque)
        self.lengths: list[int] = []       # sorted distinct lengths with untrained samples
        self._claimed: set[int] = set()
        self.dropped = 0

    # ------------------------------------------------------------ loading
    def load(self) -> int:
        if self.data_path is None:
            return 0
        if self.tokenize is None:
            raise ValueError("store needs a tokenizer to load a text corpus")
        texts = []
        with open(self.data_path, encoding="utf-8") as f:
            for line in f:
                t = line.strip()
                if t:
                    texts.append(t)
                if self.max_prepare is not None and len(texts) >= self.max_prepare:
                    break
        return self.add_samples((self.tokenize(t), t) for t in texts)

    def add_samples(self, items: Iterable[tuple[list[int], str]]) -> int:
        n = 0
        dropped = []
        for ids, text in items:
            ids = list(ids)
            if len(ids) > self.cap or len(ids) == 0:
                dropped.append(len(ids))
                continue
            s = FinetuningSample(uuid.uuid4().hex, ids, text, self.adapter)
            self.id2idx[s.request_id] = len(self.samples)
            self.samples.append(s)
            self.trained.append(False)
            n += 1
        self.dropped += len(dropped)
        if dropped:
            dprint(f"[store] dropped {len(dropped)} sample(s) longer than the activation buffer "
                   f"({self.cap} tokens); longest {max(dropped)}")
        self._rebuild()
        return n

    @classmethod
    def synthetic(cls, vocab: int, num: int, min_len: int, max_len: int, seed: int = 0,
                  **kw) -> "FinetuningStore":
        """Uniform-random token sequences with uniform lengths (benchmarks)."""
        st = cls(**kw)
        rng = np.random.default_rng(seed)
        lens = rng.integers(min_len, max_len + 1, size=num)
        st.add_samples((rng.integers(0, vocab, size=int(n)).tolist(), "") for n in lens)
        return st

    def _rebuild(self) -> None:
        self.buckets = defaultdict(deque)
        for i, s in enumerate(self.samples):
            if not self.trained[i] and i not in self._claimed:
                self.buckets[s.input_len].append(i)
        self.lengths = sorted(k for k, v in self.buckets.items() if v)

    # ------------------------------------------------------------ selection
    def __len__(self) -> int:
        return len(self.samples)

    def has_next(self) -> bool:
        return bool(self.lengths)

    def num_untrained(self) -> int:
        return sum(len(self.buckets[k]) for k in self.lengths)

    def _peek_len(self, ln: int, exclude: set[int]):
        for i in self.buckets[ln]:
            if i not in exclude:
                return i
        return None

    def pop_best_under(self, max_tokens: int, exclude=()) -> FinetuningSample | None:
        ex = {self.id2idx[s.request_id] for s in exclude}
        pos = bisect_right(self.lengths, max_tokens)
        for j in range(pos - 1, -1, -1):
            i = self._peek_len(self.lengths[j], ex)
            if i is not None:
                return self.samples[i]
        return None

    def pop_next(self, exclude=()) -> FinetuningSample | None:
        ex = {self.id2idx[s.request_id] for s in exclude}
        for ln in self.lengths:
            i = self._peek_len(ln, ex)
            if i is not None:
                return self.samples[i]
        return None

    def min_len(self) -> int | None:
        return self.lengths[0] if self.lengths else None

    # ------------------------------------------------------------ claims
    def claim(self, samples: list[FinetuningSample]) -> None:
        for s in samples:
            i = self.id2idx[s.request_id]
            if i in self._claimed or self.trained[i]:
                raise ValueError(f"sample {s.request_id} already claimed or trained")
            self._claimed.add(i)
            b = self.buckets[s.input_len]
            b.remove(i)
            if not b:
                k = bisect_left(self.lengths, s.input_len)
                if k < len(self.lengths) and self.lengths[k] == s.input_len:
                    del self.lengths[k]

    def commit_claimed(self, samples: list[FinetuningSample]) -> None:
        for s in samples:
            i = self.id2idx[s.request_id]
            self._claimed.discard(i)
            self.trained[i] = True

    def release_claimed(self, samples: list[FinetuningSample]) -> None:
        for s in samples:
            i = self.id2idx[s.request_id]
            if i not in self._claimed:
                continue
            self._claimed.discard(i)
            b = self.buckets[s.input_len]
            if not b:
                insort(self.lengths, s.input_len)
            b.appendleft(i)

    @property
    def num_claimed(self) -> int:
        return len(self._claimed)

    def advance_epoch(self) -> bool:
        """Start the next pass once every sample of this one is reconciled."""
        if self._claimed or self.has_next():
            return False
        if self.current_epoch + 1 >= self.total_epochs:
            return False
        self.current_epoch += 1
        self.trained = [False] * len(self.samples)
        self._rebuild()
        dprint(f"[store] epoch {self.current_epoch} started ({len(self.samples)} samples)")
        return True

    def finished(self) -> bool:
        return (not self.has_next() and not self._claimed
                and self.current_epoch >= self.total_epochs - 1)

    def total_tokens(self) -> int:
        return sum(s.input_len for s in self.samples)
