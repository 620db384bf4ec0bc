"""Base weights from an HF safetensors checkpoint, sharded for tensor parallelism.

A model directory with ``config.json`` and ``*.safetensors`` (single file or
sharded with ``model.safetensors.index.json``) loads with HF tensor names
(Llama-3 and Qwen3 dense):

=====================================================  =========================
HF tensor                                              engine tensor (per rank)
=====================================================  =========================
``model.embed_tokens.weight``                          ``embed`` rows of this rank
``lm_head.weight`` (absent when tied)                  ``lm_head`` rows of this rank
``model.norm.weight``                                  ``final_norm``
``model.layers.i.self_attn.{q,k,v}_proj.weight``       ``qkv`` (this rank's heads)
``model.layers.i.self_attn.o_proj.weight``             ``o`` (this rank's columns)
``model.layers.i.mlp.{gate,up}_proj.weight``           ``gate_up`` (64-row interleave)
``model.layers.i.mlp.down_proj.weight``                ``down`` (this rank's columns)
``model.layers.i.{input,post_attention}_layernorm``    ``in_ln`` / ``post_ln``
``model.layers.i.self_attn.{q,k}_norm.weight``         ``q_norm`` / ``k_norm`` (Qwen3)
=====================================================  =========================

Each rank reads only its own slice of every sharded tensor (``safe_open``
slices are read from the file, not materialised in full), so a 70B model at
TP=8 moves 1/8 of the projection bytes per rank. The reference gets the same
layout from vLLM's loaders (``QKVParallelLinear`` / ``MergedColumnParallelLinear`` /
``RowParallelLinear`` weight loaders, as mirrored by its shard helper
``tests/bwd_harness.py:110-129``).
"""

from __future__ import annotations

import glob
import json
import os

import torch

from .configs import ModelArch
from .weights import ModelWeights, TPInfo, _layer_from

_LAYER_NAMES = {
    "q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
    "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
    "down": "mlp.down_proj.weight", "in_ln": "input_layernorm.weight",
    "post_ln": "post_attention_layernorm.weight", "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
}


def checkpoint_files(path: str) -> list[str]:
    """The safetensors files of an HF model directory ([] if it has none)."""
    if not path or not os.path.isdir(path):
        return []
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.isfile(idx):
        with open(idx) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, x) for x in files]
    return sorted(glob.glob(os.path.join(path, "*.safetensors")))


class _Reader:
    """Name → open safetensors handle, with sliced reads."""

    def __init__(self, files: list[str]):
        from safetensors import safe_open
        self.handles = [safe_open(f, framework="pt", device="cpu") for f in files]
        self.where: dict[str, object] = {}
        for h in self.handles:
            for k in h.keys():
                self.where[k] = h

    def has(self, name: str) -> bool:
        return name in self.where

    def get(self, name: str, dim: int | None = None, start: int = 0, length: int = 0) -> torch.Tensor:
        h = self.where.get(name)
        if h is None:
            raise KeyError(f"checkpoint has no tensor {name!r}")
        if dim is None:
            return h.get_tensor(name)
        sl = h.get_slice(name)
        if dim == 0:
            return sl[start:start + length]
        return sl[:, start:start + length]


def load_hf_weights(arch: ModelArch, path: str, tp: TPInfo | None = None, device="cpu",
                    dtype=torch.bfloat16, keep_full_head: bool = True) -> ModelWeights:
    """This rank's :class:`ModelWeights` from the safetensors files under ``path``."""
    tp = tp or TPInfo()
    files = checkpoint_files(path)
    if not files:
        raise FileNotFoundError(f"{path!r} has no *.safetensors checkpoint")
    rd = _Reader(files)
    cv = lambda t: t.to(device=device, dtype=dtype).contiguous()

    def check(name: str, t: torch.Tensor, shape: tuple) -> torch.Tensor:
        if tuple(t.shape) != shape:
            raise ValueError(f"{name}: checkpoint shape {tuple(t.shape)} != expected {shape}")
        return t

    D, V = arch.hidden, arch.vocab
    v0, vl = tp.split(V)
    embed = cv(check("model.embed_tokens.weight", rd.get("model.embed_tokens.weight", 0, v0, vl), (vl, D)))
    tied = arch.tie_embeddings or not rd.has("lm_head.weight")
    head_name = "model.embed_tokens.weight" if tied else "lm_head.weight"
    lm_head = embed if tied else cv(rd.get(head_name, 0, v0, vl))
    head_full = None
    if keep_full_head:
        head_full = embed if (tied and tp.size == 1) else cv(rd.get(head_name))
    w = ModelWeights(arch=arch, tp=tp, embed=embed, lm_head=lm_head,
                     final_norm=cv(rd.get("model.norm.weight")), lm_head_full=head_full)
    shapes = {"q": (arch.q_size, D), "k": (arch.kv_size, D), "v": (arch.kv_size, D), "o": (D, arch.q_size),
              "gate": (arch.intermediate, D), "up": (arch.intermediate, D), "down": (D, arch.intermediate)}
    for i in range(arch.num_layers):
        pre = f"model.layers.{i}."

        def get(n, d, s, l, pre=pre):
            t = rd.get(pre + _LAYER_NAMES[n], d, s, l)
            if n in shapes:
                full = shapes[n]
                want = full if d is None else tuple(l if j == d else full[j] for j in range(2))
                check(pre + _LAYER_NAMES[n], t, want)
            return cv(t)
        w.layers.append(_layer_from(arch, get, tp))
    return w
