"""Continuous-batching scheduler with chunked prefill and paged KV.

Every step is built in three parts, in batch order:

1. **decode** — every running request past its prompt gets one token (a new
   page when it crosses a page boundary; when pages run out the newest running
   request is pre-empted by recompute: pages freed, request back to the front
   of the waiting queue);
2. **prefill** — running requests in the middle of a chunked prompt, then
   waiting requests in arrival order, under ``max_num_batched_tokens`` and
   ``max_num_seqs`` (the last one is chunked when chunked prefill is on);
3. **finetuning** — whole FT samples handed in by the finetuning admission
   layer for this step (never chunked; their pages are freed at the end of
   the step).

FT rows therefore form one contiguous range at the end of the batch.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field

from .kv_cache import BlockAllocator, PrefixCachingAllocator, block_hash, blocks_needed
from .request import Request, Status


@dataclass
class ScheduledSeq:
    req: Request
    num_new: int
    is_decode: bool
    sample: bool

    @property
    def start(self) -> int:
        return self.req.num_computed


@dataclass
class SchedulerOutput:
    decode: list[ScheduledSeq] = field(default_factory=list)
    prefill: list[ScheduledSeq] = field(default_factory=list)
    ft: list[ScheduledSeq] = field(default_factory=list)
    preempted: list[Request] = field(default_factory=list)

    @property
    def seqs(self) -> list[ScheduledSeq]:
        return self.decode + self.prefill + self.ft

    @property
    def num_tokens(self) -> int:
        return sum(s.num_new for s in self.seqs)

    @property
    def t_in(self) -> int:
        """Prefill tokens (inference + FT)."""
        return sum(s.num_new for s in self.prefill) + sum(s.num_new for s in self.ft)

    @property
    def t_ft(self) -> int:
        return sum(s.num_new for s in self.ft)

    @property
    def b_d(self) -> int:
        return len(self.decode)

    @property
    def k_decode(self) -> int:
        return sum(s.req.num_computed + 1 for s in self.decode)

    def prefill_lens(self) -> list[int]:
        return [s.num_new for s in self.prefill] + [s.num_new for s in self.ft]

    def is_empty(self) -> bool:
        return not (self.decode or self.prefill or self.ft)


class Scheduler:
    def __init__(self, allocator: BlockAllocator, block_size: int, max_num_seqs: int = 256,
                 max_num_batched_tokens: int = 8192, max_model_len: int = 4096,
                 enable_chunked_prefill: bool = True, cache_key=None):
        self.alloc = allocator
        # Automatic prefix caching when the allocator supports it: a waiting
        # request starts after the longest run of cached full pages of its
        # tokens. ``cache_key(req)`` identifies what else shaped the K/V (its
        # LoRA slot and version); None = the request neither uses nor feeds
        # the cache (finetuning rows, the adapter being trained).
        self.caching = isinstance(allocator, PrefixCachingAllocator)
        self.cache_key = cache_key or (lambda req: ())
        self.block_size = block_size
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.chunked = enable_chunked_prefill
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.finished: list[Request] = []

    # ------------------------------------------------------------ queue ops
    def add(self, req: Request) -> None:
        if req.num_prompt == 0:
            raise ValueError("empty prompt")
        if req.num_prompt + (0 if req.is_ft else req.params.max_tokens) > self.max_model_len:
            raise ValueError(f"request {req.request_id}: prompt + max_tokens exceeds "
                             f"max_model_len={self.max_model_len}")
        req.status = Status.WAITING
        self.waiting.append(req)

    def abort(self, request_id: str) -> Request | None:
        for q in (self.running, self.waiting):
            for r in list(q):
                if r.request_id == request_id:
                    q.remove(r)
                    self._free(r)
                    r.status = Status.ABORTED
                    return r
        return None

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running)

    def num_waiting(self) -> int:
        return len(self.waiting)

    def _free(self, req: Request) -> None:
        if req.block_ids:
            self.alloc.free(req.block_ids)
            req.block_ids = []

    def _ensure_blocks(self, req: Request, total_tokens: int) -> bool:
        need = blocks_needed(total_tokens, self.block_size) - len(req.block_ids)
        if need <= 0:
            return True
        if need > self.alloc.num_free:
            return False
        req.block_ids.extend(self.alloc.allocate(need))
        return True

    # ------------------------------------------------------------ prefix cache
    def _key(self, req: Request):
        if not self.caching or req.is_ft:
            return None
        return self.cache_key(req)

    def _hashes(self, req: Request, key, n_pages: int) -> list:
        bs = self.block_size
        ids = req.all_ids
        hs = req.block_hashes
        while len(hs) < n_pages:
            j = len(hs)
            hs.append(block_hash(hs[-1] if hs else b"", ids[j * bs:(j + 1) * bs], key))
        return hs

    def _attach_prefix(self, req: Request) -> None:
        """Reuse cached pages for the request's leading full pages (at least
        one token is always left to compute: its logits give the next token)."""
        key = self._key(req)
        if key is None or req.num_computed or req.block_ids:
            return
        req.block_hashes, req.num_registered = [], 0
        n_pages = (req.num_tokens - 1) // self.block_size
        if n_pages <= 0:
            return
        pages = self.alloc.lookup(self._hashes(req, key, n_pages))
        if pages:
            req.block_ids = pages
            req.num_registered = len(pages)
            req.num_computed = len(pages) * self.block_size
            req.num_cached_tokens = req.num_computed

    def _detach_prefix(self, req: Request) -> None:
        """Give back cached pages of a request that could not be admitted."""
        if req.block_ids:
            self.alloc.free(req.block_ids)
            req.block_ids = []
        req.num_computed = 0
        req.num_registered = 0
        req.num_cached_tokens = 0

    def _register(self, req: Request) -> None:
        """Publish the request's newly completed full pages to the cache."""
        key = self._key(req)
        if key is None:
            return
        full = min(req.num_computed // self.block_size, len(req.block_ids))
        if full <= req.num_registered:
            return
        hs = self._hashes(req, key, full)
        for j in range(req.num_registered, full):
            self.alloc.register(req.block_ids[j], hs[j])
        req.num_registered = full

    def cache_stats(self) -> dict:
        if not self.caching:
            return {"enabled": False}
        return {"enabled": True, "queried_pages": self.alloc.queries, "hit_pages": self.alloc.hits,
                "cached_pages": len(self.alloc.hash_of), "evictable_pages": len(self.alloc.evictable)}

    def _preempt_one(self, out: SchedulerOutput, protect: Request) -> bool:
        for victim in reversed(self.running):
            if victim is protect:
                continue
            self.running.remove(victim)
            self._free(victim)
            victim.num_computed = 0
            victim.num_registered = 0
            victim.status = Status.WAITING
            self.waiting.appendleft(victim)
            out.preempted.append(victim)
            out.decode = [s for s in out.decode if s.req is not victim]
            return True
        return False

    # ------------------------------------------------------------ schedule
    def schedule(self) -> SchedulerOutput:
        """Inference part of the next step (decode + prefill)."""
        out = SchedulerOutput()
        budget = self.max_num_batched_tokens
        # 1. decode for running requests that finished their prompt
        gone: set[int] = set()     # ids of requests pre-empted during this loop
        for req in list(self.running):
            if req.in_prefill or id(req) in gone:
                continue
            while not self._ensure_blocks(req, req.num_computed + 1):
                if not self._preempt_one(out, req):
                    break
                gone.add(id(out.preempted[-1]))
            if id(req) in gone:
                continue
            if blocks_needed(req.num_computed + 1, self.block_size) > len(req.block_ids):
                continue  # could not get a page even after pre-emption
            out.decode.append(ScheduledSeq(req, 1, True, True))
            budget -= 1
        # 2a. running requests in the middle of a chunked prompt
        for req in self.running:
            if not req.in_prefill or budget <= 0:
                continue
            n = min(req.remaining_prefill, budget)
            if not self._ensure_blocks(req, req.num_computed + n):
                continue
            out.prefill.append(ScheduledSeq(req, n, False, n == req.remaining_prefill))
            budget -= n
        # 2b. waiting requests
        while self.waiting and budget > 0 and len(self.running) < self.max_num_seqs:
            req = self.waiting[0]
            if self.caching:
                self._attach_prefix(req)
            n = req.remaining_prefill
            if n > budget:
                if not self.chunked:
                    if self.caching:
                        self._detach_prefix(req)
                    break
                n = budget
            if not self._ensure_blocks(req, req.num_computed + n):
                if self.caching:
                    self._detach_prefix(req)
                break
            self.waiting.popleft()
            req.status = Status.RUNNING
            self.running.append(req)
            out.prefill.append(ScheduledSeq(req, n, False, n == req.remaining_prefill))
            budget -= n
        return out

    def finish(self, req: Request, now: float | None = None) -> None:
        """End a running request early (a stop string matched)."""
        if req in self.running:
            self.running.remove(req)
        req.status = Status.FINISHED
        req.finish_time = time.perf_counter() if now is None else now
        if self.caching:
            self._register(req)
        self._free(req)
        self.finished.append(req)

    def add_ft(self, out: SchedulerOutput, reqs: list[Request]) -> list[Request]:
        """Append whole FT samples to ``out``; returns the ones that did not fit
        (token budget or pages) so the caller can release them."""
        budget = self.max_num_batched_tokens - out.num_tokens
        rejected = []
        for r in reqs:
            n = r.num_prompt
            if n > budget or not self._ensure_blocks(r, n):
                rejected.append(r)
                continue
            r.status = Status.RUNNING
            out.ft.append(ScheduledSeq(r, n, False, False))
            budget -= n
        return rejected

    def rollback_ft(self, out: SchedulerOutput) -> list[Request]:
        """Drop the FT part of a step that will not run (pre-empted before launch)."""
        reqs = [s.req for s in out.ft]
        for r in reqs:
            self._free(r)
            r.status = Status.ABORTED
        out.ft = []
        return reqs

    def update(self, out: SchedulerOutput, sampled: dict[int, int], now: float | None = None,
               eos_id=None) -> list[Request]:
        """Apply a finished step: advance computed counts, append sampled tokens,
        retire finished requests. ``sampled`` maps Request.seq_no -> token."""
        now = time.perf_counter() if now is None else now
        eos = (() if eos_id is None else (eos_id,) if isinstance(eos_id, int) else tuple(eos_id))
        done: list[Request] = []
        for s in out.decode + out.prefill:
            r = s.req
            r.num_computed += s.num_new
            if self.caching:
                self._register(r)
            if not s.sample:
                continue
            tok = sampled.get(r.seq_no)
            if tok is None:
                continue
            r.output_ids.append(int(tok))
            if r.first_token_time is None:
                r.first_token_time = now
            else:
                r.token_times.append(now)
            stop = (len(r.output_ids) >= r.params.max_tokens
                    or (not r.params.ignore_eos and tok in eos)
                    or tok in r.params.stop_token_ids
                    or r.num_tokens >= self.max_model_len)
            if stop:
                r.status = Status.FINISHED
                r.finish_time = now
                self.running.remove(r)
                self._free(r)
                done.append(r)
        for s in out.ft:
            s.req.num_computed += s.num_new
            s.req.status = Status.FINISHED
            s.req.finish_time = now
            self._free(s.req)
        self.finished.extend(done)
        return done
