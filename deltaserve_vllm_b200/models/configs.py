"""Decoder architectures the engine serves and trains.

Two families, as in the reference (``deltaserve-plugin/deltaserve/bwd_services/registry.py:15-25``):
``llama`` (Llama-3) and ``qwen3`` (Qwen3 dense: per-head q/k RMSNorm).
Weights are random-initialised from the architecture alone (no checkpoints
are needed), or the architecture is read from an HF ``config.json``.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, replace


@dataclass(frozen=True)
class ModelArch:
    name: str
    family: str                 # "llama" | "qwen3"
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None
    tie_embeddings: bool = False
    max_position: int = 8192

    @property
    def qk_norm(self) -> bool:
        return self.family == "qwen3"

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def params(self) -> int:
        D, I = self.hidden, self.intermediate
        per_layer = D * (self.q_size + 2 * self.kv_size) + self.q_size * D + 3 * D * I
        emb = self.vocab * D * (1 if self.tie_embeddings else 2)
        return self.num_layers * per_layer + emb

    def flops_per_token(self) -> float:
        """Dense forward FLOPs per token excluding attention scores."""
        D, I = self.hidden, self.intermediate
        per_layer = 2 * D * (self.q_size + 2 * self.kv_size) + 2 * self.q_size * D + 6 * D * I
        return float(self.num_layers * per_layer + 2 * self.vocab * D)


PRESETS: dict[str, ModelArch] = {
    # The CPU/gloo plumbing model (tiny Qwen3-style decoder, fp32 checks).
    "qwen3-tiny": ModelArch("qwen3-tiny", "qwen3", 2, 256, 4, 2, 64, 512, 1024,
                            rms_eps=1e-6, rope_theta=1e6, tie_embeddings=True),
    "llama3-tiny": ModelArch("llama3-tiny", "llama", 2, 256, 4, 2, 64, 512, 1024,
                             rms_eps=1e-5, rope_theta=5e5),
    # Tiny GQA model whose heads split over 4 tensor-parallel ranks (CPU rank tests).
    "llama3-tiny-kv4": ModelArch("llama3-tiny-kv4", "llama", 2, 256, 8, 4, 32, 1024, 1024,
                                 rms_eps=1e-5, rope_theta=5e5),
    # Small head_dim-128 models for GPU tests of the full engine path.
    "qwen3-test": ModelArch("qwen3-test", "qwen3", 2, 512, 4, 2, 128, 1024, 4096,
                            rms_eps=1e-6, rope_theta=1e6, tie_embeddings=True),
    "llama3-test": ModelArch("llama3-test", "llama", 2, 512, 4, 2, 128, 1024, 4096,
                             rms_eps=1e-5, rope_theta=5e5),
    # Llama-3-8B layer geometry with 2 layers and a small vocab (GPU smoke / tests).
    "llama3-8b-2l": ModelArch("llama3-8b-2l", "llama", 2, 4096, 32, 8, 128, 14336, 8192,
                              rms_eps=1e-5, rope_theta=5e5),
    "qwen3-0.6b": ModelArch("qwen3-0.6b", "qwen3", 28, 1024, 16, 8, 128, 3072, 151936,
                            rms_eps=1e-6, rope_theta=1e6, tie_embeddings=True,
                            max_position=40960),
    "llama3-8b": ModelArch("llama3-8b", "llama", 32, 4096, 32, 8, 128, 14336, 128256,
                           rms_eps=1e-5, rope_theta=5e5),
    "qwen3-14b": ModelArch("qwen3-14b", "qwen3", 40, 5120, 40, 8, 128, 17408, 151936,
                           rms_eps=1e-6, rope_theta=1e6, max_position=40960),
    "llama3-70b": ModelArch("llama3-70b", "llama", 80, 8192, 64, 8, 128, 28672, 128256,
                            rms_eps=1e-5, rope_theta=5e5),
}

ALIASES = {
    "meta-llama/Meta-Llama-3-8B": "llama3-8b",
    "meta-llama/Meta-Llama-3-8B-Instruct": "llama3-8b",
    "meta-llama/Llama-3.1-8B": "llama3-8b",
    "meta-llama/Meta-Llama-3-70B": "llama3-70b",
    "Qwen/Qwen3-0.6B": "qwen3-0.6b",
    "Qwen/Qwen3-0.6B-Base": "qwen3-0.6b",
    "Qwen/Qwen3-14B": "qwen3-14b",
    "Qwen/Qwen3-14B-Base": "qwen3-14b",
}

_SUPPORTED_ROPE = ("default", "linear", "llama3")


def arch_from_hf_config(cfg: dict, name: str = "hf") -> ModelArch:
    """Architecture from an HF ``config.json`` dict (Llama / Qwen3 only).

    RoPE variants the backward cannot reproduce are refused here, at launch,
    as the reference does (``deltaserve-plugin/deltaserve/ft_meta.py:46-86``)."""
    archs = cfg.get("architectures") or []
    arch = archs[0] if archs else cfg.get("model_type", "")
    if "Qwen3" in arch or cfg.get("model_type") == "qwen3":
        family = "qwen3"
    elif "Llama" in arch or cfg.get("model_type") == "llama":
        family = "llama"
    else:
        raise ValueError(f"unsupported architecture {arch!r} (Llama-3 and Qwen3 dense only)")
    heads = int(cfg["num_attention_heads"])
    hidden = int(cfg["hidden_size"])
    head_dim = int(cfg.get("head_dim") or hidden // heads)
    # Older configs carry ``rope_theta`` + ``rope_scaling``; newer ones one
    # ``rope_parameters`` dict holding both (``rope_type`` "default" = none).
    rp = cfg.get("rope_parameters") or {}
    theta = float(cfg.get("rope_theta") or rp.get("rope_theta") or 10000.0)
    rs = cfg.get("rope_scaling") or {k: v for k, v in rp.items() if k != "rope_theta"}
    if rs and rs.get("rope_type", rs.get("type", "default")) == "default" and len(rs) <= 1:
        rs = None
    if rs:
        rtype = rs.get("rope_type", rs.get("type", "default"))
        if rtype not in _SUPPORTED_ROPE:
            raise ValueError(f"RoPE type {rtype!r} is not supported "
                             f"(supported: {', '.join(_SUPPORTED_ROPE)})")
        rs = dict(rs, rope_type=rtype)
    return ModelArch(
        name=name, family=family,
        num_layers=int(cfg["num_hidden_layers"]), hidden=hidden,
        num_heads=heads, num_kv_heads=int(cfg.get("num_key_value_heads", heads)),
        head_dim=head_dim, intermediate=int(cfg["intermediate_size"]),
        vocab=int(cfg["vocab_size"]), rms_eps=float(cfg.get("rms_norm_eps", 1e-6)),
        rope_theta=theta, rope_scaling=rs or None,
        tie_embeddings=bool(cfg.get("tie_word_embeddings", False)),
        max_position=int(cfg.get("max_position_embeddings", 8192)))


def resolve_arch(model: str, **overrides) -> ModelArch:
    """Preset name, HF alias or directory with ``config.json`` → ModelArch."""
    key = ALIASES.get(model, model)
    if key in PRESETS:
        arch = PRESETS[key]
    elif os.path.isdir(model) and os.path.isfile(os.path.join(model, "config.json")):
        with open(os.path.join(model, "config.json")) as f:
            arch = arch_from_hf_config(json.load(f), name=os.path.basename(model))
    else:
        raise ValueError(f"unknown model {model!r}; presets: {sorted(PRESETS)}")
    return replace(arch, **overrides) if overrides else arch
