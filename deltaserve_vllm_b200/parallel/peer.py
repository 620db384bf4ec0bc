"""Peer-mapped workspaces for the fused GEMM + all-reduce kernel.

One cudaMalloc'd block per rank, exported as a CUDA IPC handle and opened by
every other rank (plain P2P mappings over NVLink / NVSwitch: no multicast
object, so a rank that exits cannot leave a multicast binding behind). The
block holds, for output width ``n_cols`` and up to ``max_rows`` rows:

* ``recv``  — ``world x owned_cap`` partial tiles of 128 x 128 bf16: the slots
  other ranks push the tiles this rank owns into (tile ``L`` belongs to rank
  ``L % world``);
* ``out``   — the reduced ``[max_rows, n_cols]`` bf16 result;
* ``rflag`` — per owned tile, how many ranks have pushed (reset by the owner);
* ``fflag`` — per output tile, set by its owner once the result is written
  here (reset by this rank);
* ``tile_cnt`` — this rank's split-K tickets (the last split reduces).

``ops.gemm_ar`` drives the kernel; the workspace is reused by every call on
the forward stream (each call's result is consumed before the next call's
pushes can reach it: a peer only pushes after this rank's partial of the
same tile arrived, which comes after this rank consumed the previous output).
"""

from __future__ import annotations

import math
import os

import torch

TILE = 128
_ALIGN = 256


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class PeerWorkspace:
    def __init__(self, comm, max_rows: int, n_cols: int, device=None):
        from .. import ops
        ext = ops.native_ext()
        if ext is None:
            raise RuntimeError("the fused all-reduce needs the CUDA extension")
        if n_cols % TILE:
            raise ValueError("n_cols must be a multiple of 128")
        self.comm = comm
        self.world = comm.size if comm is not None else 1
        self.rank = comm.rank if comm is not None else 0
        if self.world > 8:
            raise ValueError("the fused all-reduce supports up to 8 ranks")
        self.n_cols = n_cols
        m_tiles = math.ceil(max_rows / TILE)
        self.max_rows = m_tiles * TILE
        self.tiles = m_tiles * (n_cols // TILE)
        self.owned_cap = math.ceil(self.tiles / self.world)
        sizes = [self.world * self.owned_cap * TILE * TILE * 2,   # recv
                 self.max_rows * n_cols * 2,                         # out
                 self.owned_cap * 4,                                 # rflag
                 self.tiles * 4,                                     # fflag
                 self.tiles * 4]                                     # tile_cnt
        self.offsets = []
        off = 0
        for sz in sizes:
            self.offsets.append(off)
            off += _align(sz)
        self.bytes = off
        self._ext = ext
        self.base, handle = ext.peer_alloc(self.bytes)
        handles = comm.all_gather_object(handle) if self.world > 1 else [handle]
        self.ptrs = [self.base if r == self.rank else ext.peer_open(h) for r, h in enumerate(handles)]
        self.table = torch.tensor([[p + self.offsets[k] for p in self.ptrs] for k in range(4)],
                                  dtype=torch.int64)
        self.tile_cnt = self.base + self.offsets[4]
        self.calls = 0
        # Measured (ar_bench, Llama-3-8B o / down shapes): at TP=2 GEMM + NCCL
        # wins above 2048 rows; at TP=4 the fused kernel wins up to 4096 rows
        # (1.03-1.33x) and NCCL at 8192 rows (0.82-0.91x).
        default_max = 2048 if self.world <= 2 else 4096
        self.fused_max_rows = int(os.environ.get("DSV_FUSED_AR_MAX_ROWS", str(default_max)))
        if comm is not None and self.world > 1:
            comm.barrier()        # every rank mapped every block before first use

    def fits(self, rows: int, n_cols: int) -> bool:
        return rows <= self.max_rows and n_cols == self.n_cols

    def prefer(self, rows: int, n_cols: int) -> bool:
        """Whether the fused kernel should take this call: measured at TP=2 it
        beats GEMM + NCCL from 256 to 2048 rows (1.2-1.5x) and at 4096 rows
        for o_proj, not for down_proj at 4096 rows; calls above
        ``fused_max_rows`` go to NCCL."""
        return self.fits(rows, n_cols) and rows <= self.fused_max_rows

    def close(self) -> None:
        """Unmap the peers' blocks and free this rank's (after a barrier, so no
        peer is still writing into it)."""
        if self.base is None:
            return
        torch.cuda.synchronize()
        if self.comm is not None and self.world > 1:
            self.comm.barrier()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self._ext.peer_close(p)
        self._ext.peer_free(self.base)
        self.base = None


class PeerTable:
    """A row-sharded table (the vocabulary-parallel embedding) in peer-mapped
    memory: rank ``r``'s shard holds rows ``[r * rows, (r + 1) * rows)`` of a
    ``vocab``-row table, and every rank can read every shard directly
    (``ops.embedding_peer``). ``local`` is this rank's shard (it replaces the
    weight tensor, so nothing is stored twice)."""

    def __init__(self, comm, shard: torch.Tensor, vocab: int):
        from .. import ops
        ext = ops.native_ext()
        if ext is None:
            raise RuntimeError("the peer table needs the CUDA extension")
        self.comm = comm
        self.world, self.rank = comm.size, comm.rank
        if self.world > 8:
            raise ValueError("peer tables support up to 8 ranks")
        self.rows, self.vocab = int(shard.shape[0]), int(vocab)
        self._ext = ext
        self.base, handle = ext.peer_alloc(_align(shard.numel() * shard.element_size()))
        handles = comm.all_gather_object(handle)
        self.ptrs = [self.base if r == self.rank else ext.peer_open(h) for r, h in enumerate(handles)]
        self.local = _from_ptr(self.base, shard.shape, shard.dtype, shard.device.index)
        self.local.copy_(shard)
        self.table = torch.tensor(self.ptrs, dtype=torch.int64, device=shard.device)
        torch.cuda.synchronize()
        comm.barrier()            # every shard filled and mapped before the first read

    def close(self) -> None:
        if self.base is None:
            return
        torch.cuda.synchronize()
        self.comm.barrier()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self._ext.peer_close(p)
        self.local = None
        self._ext.peer_free(self.base)
        self.base = None


class AGPeerWorkspace:
    """Row shards of an activation in peer-mapped memory, for the all-gather
    -> column-parallel GEMM (``ops.gemm_ag``): rank ``r`` writes its rows into
    ``local`` ([max_rows_per_rank, cols] bf16). The GEMM reads its own row
    blocks in place (TMA through ``maps[rank]``) and, by default, first copies
    every remote row block once into ``gathered`` (P2P loads by the epilogue
    warps of all its CTAs, counted per block in ``cnt``) and reads those from
    there, so each remote row crosses NVLink once whatever the number of N
    tiles; ``copy_once=False`` reads every tile from its owner instead."""

    def __init__(self, comm, max_rows_per_rank: int, cols: int, device=None):
        from .. import ops
        ext = ops.native_ext()
        if ext is None:
            raise RuntimeError("the all-gather GEMM workspace needs the CUDA extension")
        self.comm = comm
        self.world = comm.size if comm is not None else 1
        self.rank = comm.rank if comm is not None else 0
        if self.world > 8:
            raise ValueError("up to 8 ranks")
        self.rows_cap = -(-int(max_rows_per_rank) // TILE) * TILE
        self.cols = int(cols)
        self._ext = ext
        self.base, handle = ext.peer_alloc(_align(self.rows_cap * self.cols * 2))
        handles = comm.all_gather_object(handle) if self.world > 1 else [handle]
        self.ptrs = [self.base if r == self.rank else ext.peer_open(h) for r, h in enumerate(handles)]
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.local = _from_ptr(self.base, (self.rows_cap, self.cols), torch.bfloat16, dev.index)
        host_maps = ext.peer_tmaps(torch.tensor(self.ptrs, dtype=torch.int64), self.rows_cap, self.cols, self.cols)
        self.maps = host_maps.to(dev)           # 128 B per map, from a 256-byte aligned allocation
        self.src = torch.tensor(self.ptrs, dtype=torch.int64)
        # Copy-once gather: this rank's copy of every shard's rows (its own
        # rows stay unused there) and the per-128-row-block unit counters.
        self.gathered = torch.empty(self.world * self.rows_cap, self.cols, dtype=torch.bfloat16, device=dev)
        self.cnt = torch.zeros(self.world * self.rows_cap // TILE + 1, dtype=torch.int32, device=dev)  # + ticket
        if comm is not None and self.world > 1:
            comm.barrier()

    def close(self) -> None:
        if self.base is None:
            return
        torch.cuda.synchronize()
        if self.comm is not None and self.world > 1:
            self.comm.barrier()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self._ext.peer_close(p)
        self.local = None
        self._ext.peer_free(self.base)
        self.base = None


class BwdPeerWorkspace:
    """Peer-mapped buffers of the tensor-parallel backward's residual-gradient
    reductions (``ops.gemm_push`` + ``ops.tp_reduce_rows``): the dX GEMM
    pushes each 128-row block's bf16 partial to the block's owner
    (block ``mt`` -> rank ``mt % world``), the owner sums, applies the RMSNorm
    backward and writes the bf16 rows into every rank's gather buffer.

    One cudaMalloc'd block per rank, opened by every peer (CUDA IPC, plain P2P
    mappings, no multicast object), holding:

    * ``recv``  — ``[world][blocks_cap][128][ld]`` bf16 partial rows pushed to
      this rank (``blocks_cap`` = owned row blocks at ``max_rows``);
    * ``gather`` x 2 — ``[max_rows][ld]`` bf16 reduced rows (two, so the
      result of one reduction is still readable while the next is gathered);
    * ``cnt``   — per owned block, columns arrived (reset by this rank);
    * ``gcnt``  — per row block, rows arrived from its owner (reset by this rank).
    """

    def __init__(self, comm, max_rows: int, ld: int):
        from .. import ops
        ext = ops.native_ext()
        if ext is None:
            raise RuntimeError("the tensor-parallel backward workspace needs the CUDA extension")
        if ld % 32:
            raise ValueError("the row width must be a multiple of 32")
        self.comm = comm
        self.world = comm.size
        self.rank = comm.rank
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self.ld = ld
        self.m_blocks = math.ceil(max_rows / TILE)
        self.max_rows = self.m_blocks * TILE
        self.blocks_cap = math.ceil(self.m_blocks / self.world)
        sizes = [self.world * self.blocks_cap * TILE * ld * 2,   # recv
                 self.max_rows * ld * 2,                          # gather 0
                 self.max_rows * ld * 2,                          # gather 1
                 self.blocks_cap * 4,                             # cnt
                 self.m_blocks * 4]                               # gcnt
        self.offsets = []
        off = 0
        for sz in sizes:
            self.offsets.append(off)
            off += _align(sz)
        self.bytes = off
        self._ext = ext
        self.base, handle = ext.peer_alloc(self.bytes)
        handles = comm.all_gather_object(handle)
        self.ptrs = [self.base if r == self.rank else ext.peer_open(h) for r, h in enumerate(handles)]
        at = lambda k: [p + self.offsets[k] for p in self.ptrs]
        self.push_table = torch.tensor([at(0), at(3)], dtype=torch.int64)
        self.gather_tables = [torch.tensor([at(1), at(4)], dtype=torch.int64),
                              torch.tensor([at(2), at(4)], dtype=torch.int64)]
        self.recv_addr = self.base + self.offsets[0]
        self.cnt_addr = self.base + self.offsets[3]
        self.gcnt_addr = self.base + self.offsets[4]
        self._views = {}
        comm.barrier()        # every rank mapped every block before first use

    def gather_view(self, buf: int, rows: int) -> torch.Tensor:
        """This rank's gather buffer ``buf`` as a bf16 [rows, ld] tensor."""
        key = (buf, rows)
        t = self._views.get(key)
        if t is None:
            full = self._views.get((buf, None))
            if full is None:
                full = _from_ptr(self.base + self.offsets[1 + buf], (self.max_rows, self.ld),
                                 torch.bfloat16, torch.cuda.current_device())
                self._views[(buf, None)] = full
            t = full[:rows]
            self._views[key] = t
        return t

    def close(self) -> None:
        if self.base is None:
            return
        torch.cuda.synchronize()
        self.comm.barrier()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self._ext.peer_close(p)
        self._ext.peer_free(self.base)
        self.base = None
        self._views.clear()


def _from_ptr(addr: int, shape, dtype, device) -> torch.Tensor:
    """A tensor over ``addr`` (memory owned by the workspace, not by PyTorch)."""
    from .. import ops
    return ops.native_ext().peer_view(int(addr), list(shape), dtype, int(device))


class OptPeerWorkspace:
    """Peer-mapped buffers of the fused optimizer for the TP-replicated LoRA
    factors (``ops.push_slices`` ... ``ops.adamw_slice_bcast``): rank ``r``
    owns elements ``[r * slice, (r + 1) * slice)`` of the replicated block,
    receives every rank's partial gradients of them, sums them, runs AdamW
    with per-layer clipping on them and sends the updated values to every
    rank. One IPC-exported block per rank (plain P2P mappings) holding:

    * ``recv``   — ``[world][slice]`` fp32 partial gradients pushed to this rank;
    * ``pstage`` — ``[total]`` fp32 updated parameters from the other owners;
    * ``rows``   — ``[world][layers]`` fp32 per-layer sums of squares of every rank;
    * three counters (gradient elements, rows, parameter elements arrived).
    """

    def __init__(self, comm, total: int, layers: int):
        from .. import ops
        ext = ops.native_ext()
        if ext is None:
            raise RuntimeError("the fused optimizer workspace needs the CUDA extension")
        self.comm = comm
        self.world, self.rank = comm.size, comm.rank
        self.total, self.layers = int(total), int(layers)
        self.slice = -(-self.total // self.world)
        self.slice = -(-self.slice // 64) * 64
        self.first = self.rank * self.slice
        self.len = max(0, min(self.slice, self.total - self.first))
        sizes = [self.world * self.slice * 4, self.total * 4, self.world * self.layers * 4, 4, 4, 4]
        self.offsets, off = [], 0
        for sz in sizes:
            self.offsets.append(off)
            off += _align(sz)
        self._ext = ext
        self.base, handle = ext.peer_alloc(off)
        handles = comm.all_gather_object(handle)
        self.ptrs = [self.base if r == self.rank else ext.peer_open(h) for r, h in enumerate(handles)]
        at = lambda k: [p + self.offsets[k] for p in self.ptrs]
        self.push_table = torch.tensor([at(0), at(3)], dtype=torch.int64)
        self.param_table = torch.tensor([at(1), at(5)], dtype=torch.int64)
        self.row_table = torch.tensor([at(2), at(4)], dtype=torch.int64)
        self.recv_addr = self.base + self.offsets[0]
        self.cnt_push = self.base + self.offsets[3]
        self.cnt_rows = self.base + self.offsets[4]
        self.cnt_param = self.base + self.offsets[5]
        dev = torch.cuda.current_device()
        self.pstage = _from_ptr(self.base + self.offsets[1], (self.total,), torch.float32, dev)
        self.rows = _from_ptr(self.base + self.offsets[2], (self.world, self.layers), torch.float32, dev)
        comm.barrier()

    def close(self) -> None:
        if self.base is None:
            return
        torch.cuda.synchronize()
        self.comm.barrier()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self._ext.peer_close(p)
        self._ext.peer_free(self.base)
        self.base = None
