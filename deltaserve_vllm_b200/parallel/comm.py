"""Tensor-parallel communicators.

* :class:`TPComm` — ``torch.distributed`` collectives on one process group:
  NCCL over NVLink/NVSwitch on GPUs (the baseline path), gloo for CPU ranks in
  tests. In-place all-reduce of activations and gradients, column all-gather of
  vocab-parallel logits, object gather for checkpoint merges, and a CPU-side
  group for host votes.
* :func:`init_tp` — one process per GPU, rendezvous from the torchrun env
  (``RANK``/``WORLD_SIZE``/``MASTER_ADDR``/``MASTER_PORT``) with a short timeout so
  ranks that wait on a dead peer fail instead of hanging.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


class TPComm:
    def __init__(self, group=None, cpu_group=None):
        self.group = group
        self.cpu_group = cpu_group
        self.size = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.num_collectives = 0

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(t, group=self.group)
            self.num_collectives += 1
        return t

    def all_gather_cols(self, t: torch.Tensor) -> torch.Tensor:
        """[R, V/tp] per rank -> [R, V] (rank-major columns)."""
        if self.size == 1:
            return t
        parts = [torch.empty_like(t) for _ in range(self.size)]
        dist.all_gather(parts, t.contiguous(), group=self.group)
        self.num_collectives += 1
        return torch.cat(parts, dim=1)

    def all_gather_into(self, out: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """``out`` [size, *t.shape] = every rank's ``t`` (rank-major)."""
        if self.size == 1:
            out[0].copy_(t)
            return out
        flat = out.view((self.size * t.shape[0],) + tuple(t.shape[1:]))   # gloo wants rank-major rows
        dist.all_gather_into_tensor(flat, t.contiguous(), group=self.group)
        self.num_collectives += 1
        return out

    def all_gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return t
        out = torch.empty((self.size * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        flat = out.view((self.size * t.shape[0],) + tuple(t.shape[1:]))   # gloo wants rank-major rows
        dist.all_gather_into_tensor(flat, t.contiguous(), group=self.group)
        self.num_collectives += 1
        return out

    def broadcast_object(self, obj, src: int = 0):
        if self.size == 1:
            return obj
        box = [obj]
        dist.broadcast_object_list(box, src=src, group=self.cpu_group or self.group)
        return box[0]

    def gather_objects(self, obj, dst: int = 0):
        if self.size == 1:
            return [obj]
        out = [None] * self.size if self.rank == dst else None
        dist.gather_object(obj, out, dst=dst, group=self.cpu_group or self.group)
        return out

    def all_gather_object(self, obj) -> list:
        if self.size == 1:
            return [obj]
        out = [None] * self.size
        dist.all_gather_object(out, obj, group=self.cpu_group or self.group)
        return out

    def all_reduce_max_int(self, v: int) -> int:
        """Host vote: every rank gets the max (used for rank-symmetric decisions)."""
        if self.size == 1:
            return int(v)
        t = torch.tensor([int(v)], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.cpu_group or self.group)
        return int(t.item())

    def barrier(self) -> None:
        if self.size > 1:
            dist.barrier(group=self.cpu_group or self.group)


# SM budget of the collectives that can run at the same time on one GPU. Every
# kernel that waits on other ranks must be able to be resident together with
# the others, or two ranks could each hold the SMs the other's partner needs:
#   forward stream: the fused GEMM + all-reduce (at most SMs - 20 CTAs) or an
#     NCCL collective of the default group (at most FWD_NCCL_MAX_CTAS), never
#     both at once (one stream);
#   backward stream: NCCL collectives of the backward's own group (at most
#     BWD_NCCL_MAX_CTAS) and the one-CTA waits of its peer-memory reductions.
# 128 + 16 + 1 and 64 + 16 + 1 both fit in 148 SMs. The forward's group also
# runs on a high-priority NCCL stream, ahead of the backward's kernels.
FWD_NCCL_MAX_CTAS = int(os.environ.get("DSV_FWD_NCCL_CTAS", "64"))
BWD_NCCL_MAX_CTAS = 16


def nccl_options(max_ctas: int, high_priority: bool):
    """ProcessGroupNCCL options with a CTA cap and stream priority."""
    opts = dist.ProcessGroupNCCL.Options()
    opts.is_high_priority_stream = high_priority
    opts.config.max_ctas = int(max_ctas)
    return opts


def new_backward_group(comm: "TPComm") -> "TPComm":
    """The backward's own communicator (its collectives run on another
    stream than the forward's and must never share an NCCL queue), capped at
    BWD_NCCL_MAX_CTAS CTAs on a normal-priority stream."""
    ranks = list(range(comm.size))
    if dist.get_backend() == "nccl":
        g = dist.new_group(ranks, pg_options=nccl_options(BWD_NCCL_MAX_CTAS, high_priority=False))
    else:
        g = dist.new_group(ranks)
    return TPComm(g, comm.cpu_group)


def init_tp(backend: str | None = None, timeout_s: float = 120.0) -> TPComm:
    """Initialise the default process group from the torchrun environment."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws == 1 and not dist.is_initialized():
        return TPComm()
    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":
            local = int(os.environ.get("LOCAL_RANK", os.environ.get("RANK", "0")))
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
            kw["pg_options"] = nccl_options(FWD_NCCL_MAX_CTAS, high_priority=True)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    cpu_group = dist.new_group(backend="gloo") if backend == "nccl" else None
    return TPComm(None, cpu_group)
