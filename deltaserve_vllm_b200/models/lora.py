"""Multi-LoRA serving buffers and adapter tensors.

The seven LoRA targets are served in four *groups* of projections that share
an input (and one base GEMM):

=========  ===  ================  ==================================
group      P    input (K)         output rows (N), projection of row
=========  ===  ================  ==================================
qkv        3    hidden            q | k | v (row boundaries)
o          1    q heads (local)   hidden
gate_up    2    hidden            gate/up interleaved in 64-row blocks
down       1    intermediate (l)  hidden
=========  ===  ================  ==================================

Per layer and group, for ``slots`` adapters of padded rank ``R``:

* ``A``  [slots, P*R, K]   bf16 — the shrink weights (row ``p*R + j``)
* ``B2`` [N, slots*SEG]    bf16 — the expand weights, ``SEG = ceil(P*R/64)*64``
  columns per slot; row ``n`` of projection ``p`` keeps ``B_p[n, j] * alpha/r``
  in column ``slot*SEG + p*R + j`` and zeros elsewhere.

The scaling ``alpha/r`` is folded into ``B2`` exactly once, at load or
publish (the reference does the same for the served slot,
``bwd_services/common/trainer.py:766-777``). Column-parallel groups keep the
full ``A`` and the local rows of ``B``; row-parallel groups keep the local
input columns of ``A`` and the full ``B`` (``bwd_services/common/tp.py:37-57``),
so every LoRA term composes with the layer's single all-reduce.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..config import LORA_PROJS, PEFT_MODULE
from .configs import ModelArch
from .weights import TPInfo

GROUPS = ("qkv", "o", "gate_up", "down")
GROUP_PROJS = {"qkv": ("q", "k", "v"), "o": ("o",), "gate_up": ("gate", "up"), "down": ("down",)}
PROJ_GROUP = {p: g for g, ps in GROUP_PROJS.items() for p in ps}
COLUMN_PARALLEL = ("q", "k", "v", "gate", "up")


def seg_width(P: int, R: int) -> int:
    return -(-(P * R) // 64) * 64


@dataclass(frozen=True)
class GroupGeom:
    name: str
    P: int
    K: int          # local input width
    N: int          # local output rows
    b1: int         # row boundaries for qkv (q | k | v)
    b2: int
    interleave: bool

    def proj_rows(self, p: int) -> torch.Tensor:
        """Local row indices of projection p inside the group's output."""
        if self.interleave:
            n = torch.arange(self.N)
            return n[(n // 64) % 2 == p]
        bounds = [0, self.b1, self.b2, self.N][: self.P + 1] if self.P == 3 else [0, self.N]
        return torch.arange(bounds[p], bounds[p + 1])


def group_geoms(arch: ModelArch, tp: TPInfo) -> dict[str, GroupGeom]:
    D = arch.hidden
    ql, kl, il = arch.q_size // tp.size, arch.kv_size // tp.size, arch.intermediate // tp.size
    return {
        "qkv": GroupGeom("qkv", 3, D, ql + 2 * kl, ql, ql + kl, False),
        "o": GroupGeom("o", 1, ql, D, D, D, False),
        "gate_up": GroupGeom("gate_up", 2, D, 2 * il, 0, 0, True),
        "down": GroupGeom("down", 1, il, D, D, D, False),
    }


def peft_key(layer: int, proj: str, ab: str) -> str:
    return f"base_model.model.model.layers.{layer}.{PEFT_MODULE[proj]}.lora_{ab}.weight"


def shard_lora_factor(arch: ModelArch, proj: str, ab: str, t: torch.Tensor, tp: TPInfo) -> torch.Tensor:
    """Full PEFT factor -> this rank's shard (identity at tp=1)."""
    if tp.size == 1:
        return t
    if proj in COLUMN_PARALLEL and ab == "B":
        n = t.shape[0] // tp.size
        return t[tp.rank * n:(tp.rank + 1) * n]
    if proj in ("o", "down") and ab == "A":
        n = t.shape[1] // tp.size
        return t[:, tp.rank * n:(tp.rank + 1) * n]
    return t


def random_adapter(arch: ModelArch, rank: int, seed: int, targets=LORA_PROJS,
                   b_std: float = 0.01, dtype=torch.float32) -> dict[str, torch.Tensor]:
    """PEFT-named LoRA tensors: A kaiming-uniform (a=sqrt(5), as PEFT), B ~ N(0, b_std)."""
    g = torch.Generator().manual_seed(seed)
    dims = {"q": (arch.hidden, arch.q_size), "k": (arch.hidden, arch.kv_size),
            "v": (arch.hidden, arch.kv_size), "o": (arch.q_size, arch.hidden),
            "gate": (arch.hidden, arch.intermediate), "up": (arch.hidden, arch.intermediate),
            "down": (arch.intermediate, arch.hidden)}
    out = {}
    for i in range(arch.num_layers):
        for p in targets:
            fin, fout = dims[p]
            bound = 1.0 / math.sqrt(fin)  # kaiming_uniform(a=sqrt(5)) on [r, fin]
            out[peft_key(i, p, "A")] = (torch.rand(rank, fin, generator=g) * 2 - 1).mul_(bound).to(dtype)
            out[peft_key(i, p, "B")] = (torch.randn(fout, rank, generator=g) * b_std).to(dtype)
    return out


class LoraServeBuffers:
    """Per-layer ``A`` / ``B2`` slot buffers for every group."""

    def __init__(self, arch: ModelArch, tp: TPInfo, slots: int, max_rank: int, device,
                 dtype=torch.bfloat16):
        if slots > 32:
            raise ValueError("at most 32 LoRA slots per batch")
        self.arch, self.tp, self.slots, self.R = arch, tp, slots, max_rank
        self.geom = group_geoms(arch, tp)
        self.seg = {g: seg_width(self.geom[g].P, max_rank) for g in GROUPS}
        self.A: list[dict[str, torch.Tensor]] = []
        self.B2: list[dict[str, torch.Tensor]] = []
        for _ in range(arch.num_layers):
            a, b = {}, {}
            for g in GROUPS:
                gg = self.geom[g]
                a[g] = torch.zeros(slots, gg.P * max_rank, gg.K, dtype=dtype, device=device)
                b[g] = torch.zeros(gg.N, slots * self.seg[g], dtype=dtype, device=device)
            self.A.append(a)
            self.B2.append(b)
        self.slot_rank = [0] * slots
        # Bumped whenever a slot's weights are replaced: cached K/V computed
        # with an older version of the slot is never reused.
        self.version = [0] * slots

    def clear_slot(self, slot: int) -> None:
        self.version[slot] += 1
        for i in range(self.arch.num_layers):
            for g in GROUPS:
                self.A[i][g][slot].zero_()
                s = self.seg[g]
                self.B2[i][g][:, slot * s:(slot + 1) * s].zero_()
        self.slot_rank[slot] = 0

    @torch.no_grad()
    def load_slot(self, slot: int, tensors: dict[str, torch.Tensor], rank: int, alpha: float) -> None:
        """Write a full PEFT adapter (all layers) into ``slot``, sharding for TP."""
        if rank > self.R:
            raise ValueError(f"adapter rank {rank} > max_lora_rank {self.R}")
        self.clear_slot(slot)           # (bumps the version)
        scale = alpha / rank
        for i in range(self.arch.num_layers):
            for g in GROUPS:
                gg = self.geom[g]
                A = self.A[i][g]
                B2 = self.B2[i][g]
                s = self.seg[g]
                for p, proj in enumerate(GROUP_PROJS[g]):
                    ka, kb = peft_key(i, proj, "A"), peft_key(i, proj, "B")
                    if ka not in tensors:
                        continue
                    a = shard_lora_factor(self.arch, proj, "A", tensors[ka].float(), self.tp)
                    b = shard_lora_factor(self.arch, proj, "B", tensors[kb].float(), self.tp)
                    A[slot, p * self.R:p * self.R + rank] = a.to(A.dtype, copy=False).to(A.device)
                    rows = gg.proj_rows(p).to(B2.device)
                    cols = slot * s + p * self.R + torch.arange(rank, device=B2.device)
                    vals = (b.to(B2.device) * scale).clamp(-65504, 65504).to(B2.dtype)
                    B2[rows[:, None], cols[None, :]] = vals
        self.slot_rank[slot] = rank
