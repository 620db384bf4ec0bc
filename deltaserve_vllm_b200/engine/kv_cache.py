"""Paged KV cache: page allocator and the per-layer cache tensors.

Each layer owns ``k`` and ``v`` tensors of shape ``[num_blocks, Hkv_local,
block_size, head_dim]`` (bf16): one (page, head) is a contiguous
``block_size x head_dim`` tile, the unit the attention kernels load. A request
holds a list of page ids; token ``t`` of the request lives in page
``block_ids[t // block_size]`` at offset ``t % block_size``.

Pages are sized from the HBM left after weights, LoRA buffers and the
activation-capture buffers (``gpu_memory_utilization`` of the total).
"""

from __future__ import annotations

import hashlib
from collections import OrderedDict

import torch


class BlockAllocator:
    """LIFO free list of page ids (recently freed pages are reused first, which
    keeps the working set of the cache warm in L2)."""

    def __init__(self, num_blocks: int):
        self.num_blocks = num_blocks
        self._free = list(range(num_blocks - 1, -1, -1))

    @property
    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> list[int]:
        if n > len(self._free):
            raise MemoryError(f"KV cache out of pages: need {n}, have {len(self._free)}")
        out = self._free[-n:] if n else []
        del self._free[len(self._free) - n:]
        return out[::-1]

    def free(self, ids: list[int]) -> None:
        self._free.extend(reversed(ids))

    def usage(self) -> float:
        return 1.0 - len(self._free) / max(1, self.num_blocks)


def blocks_needed(num_tokens: int, block_size: int) -> int:
    return -(-num_tokens // block_size)


def block_hash(parent: bytes, tokens, extra: tuple = ()) -> bytes:
    """Hash of a full page given its parent page's hash, its token ids and the
    identity of whatever else shaped its KV (the LoRA slot and its version)."""
    h = hashlib.blake2b(digest_size=16)
    h.update(parent)
    h.update(repr(tuple(extra)).encode())
    h.update(b",".join(str(int(t)).encode() for t in tokens))
    return h.digest()


class PrefixCachingAllocator(BlockAllocator):
    """Page allocator with automatic prefix caching (vLLM's semantics): every
    full page of a request is registered under a chained hash of its tokens
    (and the LoRA slot version that produced its K/V); a later request whose
    prompt starts with the same pages reuses them instead of recomputing.
    Pages are reference counted; a released page that holds a registered
    prefix stays cached (evictable, least recently used first) until its id
    is needed for a new allocation."""

    def __init__(self, num_blocks: int):
        super().__init__(num_blocks)
        self.ref = [0] * num_blocks
        self.hash_of: dict[int, bytes] = {}     # page -> registered hash
        self.page_of: dict[bytes, int] = {}     # hash -> page
        self.evictable: OrderedDict[int, None] = OrderedDict()  # cached pages with ref 0, LRU first
        self.hits = 0
        self.queries = 0

    @property
    def num_free(self) -> int:
        return len(self._free) + len(self.evictable)

    def _evict(self, page: int) -> None:
        del self.evictable[page]
        h = self.hash_of.pop(page)
        if self.page_of.get(h) == page:
            del self.page_of[h]

    def allocate(self, n: int) -> list[int]:
        if n > self.num_free:
            raise MemoryError(f"KV cache out of pages: need {n}, have {self.num_free}")
        take = min(n, len(self._free))
        out = super().allocate(take)
        while len(out) < n:                      # reuse the least recently used cached pages
            page = next(iter(self.evictable))
            self._evict(page)
            out.append(page)
        for p in out:
            self.ref[p] = 1
        return out

    def free(self, ids: list[int]) -> None:
        plain = []
        for p in ids:
            self.ref[p] -= 1
            if self.ref[p] > 0:
                continue
            if p in self.hash_of:
                self.evictable[p] = None         # most recently used at the end
            else:
                plain.append(p)
        super().free(plain)

    def lookup(self, hashes: list[bytes]) -> list[int]:
        """Pages holding the longest cached run of ``hashes`` (each gets a
        reference)."""
        out = []
        self.queries += len(hashes)
        for h in hashes:
            p = self.page_of.get(h)
            if p is None:
                break
            if self.ref[p] == 0:
                del self.evictable[p]
            self.ref[p] += 1
            out.append(p)
        self.hits += len(out)
        return out

    def usage(self) -> float:
        return 1.0 - self.num_free / max(1, self.num_blocks)

    def register(self, page: int, h: bytes) -> None:
        """Record that ``page`` (full) holds the prefix hashed ``h``."""
        if page in self.hash_of:
            return
        if h in self.page_of:                    # the same prefix already lives elsewhere
            return
        self.hash_of[page] = h
        self.page_of[h] = page


class KVCache:
    def __init__(self, num_layers: int, num_blocks: int, num_kv_heads_local: int, block_size: int,
                 head_dim: int, device, dtype=torch.bfloat16, prefix_caching: bool = False):
        self.block_size = block_size
        self.num_blocks = num_blocks
        shape = (num_blocks, num_kv_heads_local, block_size, head_dim)
        self.k = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.v = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.allocator = PrefixCachingAllocator(num_blocks) if prefix_caching else BlockAllocator(num_blocks)

    @staticmethod
    def bytes_per_block(num_layers: int, num_kv_heads_local: int, block_size: int, head_dim: int,
                        elem: int = 2) -> int:
        return 2 * num_layers * num_kv_heads_local * block_size * head_dim * elem

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)
