"""Weight containers, random initialisation and tensor-parallel shard geometry.

Per-rank layout of one decoder layer (``tp`` ranks, rank ``r``):

* ``qkv``     [q_l + 2*kv_l, D]   column-parallel: this rank's q heads, then k, then v
* ``o``       [D, q_l]            row-parallel: input columns of this rank's heads
* ``gate_up`` [2*I_l, D]          column-parallel, gate and up rows interleaved in
                                  blocks of 64 ([g0..g63, u0..u63, g64..]) so the
                                  GEMM epilogue sees matching gate/up columns in
                                  one tile and emits silu(g)*u directly
* ``down``    [D, I_l]            row-parallel
* norms: ``in_ln``, ``post_ln`` [D]; Qwen3 ``q_norm``, ``k_norm`` [head_dim]

Embedding and LM head are vocab-parallel ([V/tp, D] per rank); the finetuning
head additionally keeps the full LM head (the reference all-gathers it for its
backward, ``deltaserve-plugin/deltaserve/worker.py:207-224``).

Random init draws every FULL tensor from a generator seeded by (seed, name),
then slices, so any TP degree sees the same model.
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass, field

import torch

from .configs import ModelArch
from ..ops.reference import interleave64


@dataclass
class TPInfo:
    rank: int = 0
    size: int = 1

    def split(self, n: int) -> tuple[int, int]:
        if n % self.size:
            raise ValueError(f"dimension {n} is not divisible by tp={self.size}")
        w = n // self.size
        return self.rank * w, w


@dataclass
class LayerWeights:
    qkv: torch.Tensor
    o: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    in_ln: torch.Tensor
    post_ln: torch.Tensor
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None


@dataclass
class ModelWeights:
    arch: ModelArch
    tp: TPInfo
    embed: torch.Tensor           # [V_l, D]
    lm_head: torch.Tensor         # [V_l, D] (aliases embed when tied)
    final_norm: torch.Tensor
    layers: list[LayerWeights] = field(default_factory=list)
    lm_head_full: torch.Tensor | None = None  # [V, D], for the finetuning head

    def to(self, device, dtype) -> "ModelWeights":
        """Copy of every tensor on ``device`` in ``dtype`` (tied heads stay tied)."""
        cv = lambda t: None if t is None else t.to(device=device, dtype=dtype).contiguous()
        embed = cv(self.embed)
        lm_head = embed if self.lm_head.data_ptr() == self.embed.data_ptr() else cv(self.lm_head)
        out = ModelWeights(self.arch, self.tp, embed, lm_head, cv(self.final_norm),
                           lm_head_full=cv(self.lm_head_full))
        for L in self.layers:
            out.layers.append(LayerWeights(*(cv(getattr(L, f)) for f in
                                             ("qkv", "o", "gate_up", "down", "in_ln", "post_ln",
                                              "q_norm", "k_norm"))))
        return out

    @property
    def q_local(self) -> int:
        return self.arch.q_size // self.tp.size

    @property
    def kv_local(self) -> int:
        return self.arch.kv_size // self.tp.size

    @property
    def i_local(self) -> int:
        return self.arch.intermediate // self.tp.size

    @property
    def v_local(self) -> int:
        return self.arch.vocab // self.tp.size


def _gen(seed: int, name: str, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFF)
    return g


def _randn(shape, seed, name, device, std=0.02, dtype=torch.bfloat16):
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=_gen(seed, name, device))
    return t.to(dtype)


def _norm_w(n, seed, name, device, dtype):
    # Near-one norm weights (exactly one would hide layout bugs in tests).
    t = torch.empty(n, dtype=torch.float32, device=device)
    t.uniform_(0.9, 1.1, generator=_gen(seed, name, device))
    return t.to(dtype)


def full_layer_tensors(arch: ModelArch, i: int, seed: int, device, dtype=torch.bfloat16,
                       std: float = 0.02) -> dict[str, torch.Tensor]:
    """The unsharded weights of layer ``i`` in HF orientation ([out, in])."""
    D, I = arch.hidden, arch.intermediate
    p = f"layers.{i}."
    t = {
        "q": _randn((arch.q_size, D), seed, p + "q", device, std, dtype),
        "k": _randn((arch.kv_size, D), seed, p + "k", device, std, dtype),
        "v": _randn((arch.kv_size, D), seed, p + "v", device, std, dtype),
        "o": _randn((D, arch.q_size), seed, p + "o", device, std, dtype),
        "gate": _randn((I, D), seed, p + "gate", device, std, dtype),
        "up": _randn((I, D), seed, p + "up", device, std, dtype),
        "down": _randn((D, I), seed, p + "down", device, std, dtype),
        "in_ln": _norm_w(D, seed, p + "in_ln", device, dtype),
        "post_ln": _norm_w(D, seed, p + "post_ln", device, dtype),
    }
    if arch.qk_norm:
        t["q_norm"] = _norm_w(arch.head_dim, seed, p + "q_norm", device, dtype)
        t["k_norm"] = _norm_w(arch.head_dim, seed, p + "k_norm", device, dtype)
    return t


def _layer_from(arch: ModelArch, get, tp: TPInfo) -> LayerWeights:
    """One rank's layer from ``get(name, dim, start, length)``, which returns
    the slice ``[start, start + length)`` along ``dim`` of the full HF-orientation
    tensor ``name`` (``dim`` None: the whole tensor)."""
    q0, ql = tp.split(arch.q_size)
    k0, kl = tp.split(arch.kv_size)
    i0, il = tp.split(arch.intermediate)
    qkv = torch.cat([get("q", 0, q0, ql), get("k", 0, k0, kl), get("v", 0, k0, kl)], 0).contiguous()
    gate_up = interleave64(get("gate", 0, i0, il).t(), get("up", 0, i0, il).t()).t().contiguous()
    norms = {n: get(n, None, 0, 0) for n in ("q_norm", "k_norm")} if arch.qk_norm else {}
    return LayerWeights(
        qkv=qkv, o=get("o", 1, q0, ql).contiguous(), gate_up=gate_up,
        down=get("down", 1, i0, il).contiguous(), in_ln=get("in_ln", None, 0, 0),
        post_ln=get("post_ln", None, 0, 0), q_norm=norms.get("q_norm"), k_norm=norms.get("k_norm"))


def shard_layer(arch: ModelArch, t: dict[str, torch.Tensor], tp: TPInfo) -> LayerWeights:
    return _layer_from(arch, lambda n, d, s, l: t[n] if d is None else t[n].narrow(d, s, l), tp)


def init_weights(arch: ModelArch, tp: TPInfo | None = None, seed: int = 0, device="cpu",
                 dtype=torch.bfloat16, std: float = 0.02, keep_full_head: bool = True) -> ModelWeights:
    tp = tp or TPInfo()
    if arch.num_kv_heads % tp.size or arch.num_heads % tp.size:
        raise ValueError("heads must divide evenly across tensor-parallel ranks")
    if (arch.intermediate // tp.size) % 64:
        raise ValueError("intermediate / tp must be a multiple of 64")
    v0, vl = tp.split(arch.vocab)
    emb_full = _randn((arch.vocab, arch.hidden), seed, "embed", device, std, dtype)
    embed = emb_full[v0:v0 + vl].contiguous()
    if arch.tie_embeddings:
        head_full = emb_full
        lm_head = embed
    else:
        head_full = _randn((arch.vocab, arch.hidden), seed, "lm_head", device, std, dtype)
        lm_head = head_full[v0:v0 + vl].contiguous()
    w = ModelWeights(arch=arch, tp=tp, embed=embed, lm_head=lm_head,
                     final_norm=_norm_w(arch.hidden, seed, "final_norm", device, dtype),
                     lm_head_full=head_full.contiguous() if keep_full_head else None)
    del emb_full
    for i in range(arch.num_layers):
        w.layers.append(shard_layer(arch, full_layer_tensors(arch, i, seed, device, dtype, std), tp))
    return w


def unshard_qkv(arch: ModelArch, qkv: torch.Tensor, tp_size: int = 1):
    """Split a per-rank fused qkv weight back into (q, k, v)."""
    ql, kl = arch.q_size // tp_size, arch.kv_size // tp_size
    return qkv[:ql], qkv[ql:ql + kl], qkv[ql + kl:]
