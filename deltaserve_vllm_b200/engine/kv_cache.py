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


class KVCache:
    def __init__(self, num_layers: int, num_blocks: int, num_kv_heads_local: int, block_size: int,
                 head_dim: int, device, dtype=torch.bfloat16):
        self.block_size = block_size
        self.num_blocks = num_blocks
        shape = (num_blocks, num_kv_heads_local, block_size, head_dim)
        self.k = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.v = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        self.allocator = BlockAllocator(num_blocks)

    @staticmethod
    def bytes_per_block(num_layers: int, num_kv_heads_local: int, block_size: int, head_dim: int,
                        elem: int = 2) -> int:
        return 2 * num_layers * num_kv_heads_local * block_size * head_dim * elem

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)
