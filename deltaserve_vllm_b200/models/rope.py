"""RoPE frequencies (NeoX rotate-half), with the scaling variants the served
model and the backward must agree on: default, linear and llama3
(same variant set as the reference, ``bwd_services/common/ops.py:23-58``)."""

from __future__ import annotations

import math

import torch

SUPPORTED_ROPE_TYPES = ("default", "linear", "llama3")


def rope_inv_freq(head_dim: int, theta: float, rope_scaling: dict | None = None,
                  device=None) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device)
                           / head_dim))
    rtype = (rope_scaling or {}).get("rope_type", "default")
    if rtype in (None, "default"):
        return inv
    if rtype == "linear":
        return inv / float(rope_scaling["factor"])
    if rtype == "llama3":
        factor = float(rope_scaling["factor"])
        lo = float(rope_scaling["low_freq_factor"])
        hi = float(rope_scaling["high_freq_factor"])
        orig = float(rope_scaling["original_max_position_embeddings"])
        wavelen = 2 * math.pi / inv
        lo_wl, hi_wl = orig / lo, orig / hi
        smooth = (orig / wavelen - lo) / (hi - lo) if hi != lo else torch.zeros_like(inv)
        mid = (1 - smooth) * inv / factor + smooth * inv
        return torch.where(wavelen < hi_wl, inv, torch.where(wavelen > lo_wl, inv / factor, mid))
    raise NotImplementedError(f"RoPE type {rtype!r} (supported: {SUPPORTED_ROPE_TYPES})")


def cos_sin(positions: torch.Tensor, head_dim: int, theta: float, rope_scaling=None):
    inv = rope_inv_freq(head_dim, theta, rope_scaling, device=positions.device)
    f = torch.outer(positions.float(), inv)
    return f.cos(), f.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [n, H, hd]; cos/sin [n, hd/2]."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c, s = cos[:, None, :].to(x.dtype), sin[:, None, :].to(x.dtype)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def rope_backward(g: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Transpose of ``apply_rope`` (rotation by -angle)."""
    h = g.shape[-1] // 2
    g1, g2 = g[..., :h], g[..., h:]
    c, s = cos[:, None, :].to(g.dtype), sin[:, None, :].to(g.dtype)
    return torch.cat([g1 * c + g2 * s, g2 * c - g1 * s], dim=-1)
