"""Rotary position embedding (NeoX layout: the first and second halves of a
head are the real and imaginary parts of ``head_dim / 2`` complex numbers).

The served forward and the trainer's backward take their cos/sin from
:func:`cos_sin` alone, so the two can never disagree on a position. Scaling
variants: none, ``linear`` (every frequency divided by ``factor``) and
``llama3`` (Llama-3.1's wavelength-dependent rule, the published formula:
frequencies whose wavelength is short against the original context keep
their value, long ones are divided by ``factor``, and the band between the
two blends linearly in ``original_max_position_embeddings / wavelength``).
Other variants are refused rather than trained with different positions; the
reference supports the same set (``bwd_services/common/ops.py:23-58``).
"""

from __future__ import annotations

import math

import torch

SUPPORTED_ROPE_TYPES = ("default", "linear", "llama3")


def _llama3_keep_fraction(inv: torch.Tensor, cfg: dict) -> torch.Tensor:
    """Per frequency, how much of the unscaled value survives: 1 for short
    wavelengths, 0 for long ones (fully divided by ``factor``), linear in
    ``orig / wavelength`` between ``low_freq_factor`` and ``high_freq_factor``."""
    lo, hi = float(cfg["low_freq_factor"]), float(cfg["high_freq_factor"])
    cycles = float(cfg["original_max_position_embeddings"]) * inv / (2 * math.pi)   # = orig / wavelength
    if hi == lo:
        return (cycles > hi).to(inv.dtype)
    return ((cycles - lo) / (hi - lo)).clamp(0.0, 1.0)


def rope_inv_freq(head_dim: int, theta: float, rope_scaling: dict | None = None,
                  device=None) -> torch.Tensor:
    """The ``head_dim / 2`` angular frequencies (fp32) after scaling."""
    exponent = torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim
    inv = 1.0 / (theta ** exponent)
    kind = (rope_scaling or {}).get("rope_type") or "default"
    if kind not in SUPPORTED_ROPE_TYPES:
        raise NotImplementedError(f"RoPE type {kind!r} (supported: {SUPPORTED_ROPE_TYPES})")
    if kind == "default":
        return inv
    factor = float(rope_scaling["factor"])
    if kind == "linear":
        return inv / factor
    keep = _llama3_keep_fraction(inv, rope_scaling)
    return inv * (keep + (1.0 - keep) / factor)


def cos_sin(positions: torch.Tensor, head_dim: int, theta: float, rope_scaling=None):
    """cos and sin of every (position, frequency) angle: two fp32 ``[n, head_dim / 2]``."""
    angles = positions.float()[:, None] * rope_inv_freq(head_dim, theta, rope_scaling, device=positions.device)
    return angles.cos(), angles.sin()


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, direction: float) -> torch.Tensor:
    """Multiply each complex pair of ``x`` [n, H, hd] by exp(direction * i * angle)."""
    re, im = x.split(x.shape[-1] // 2, dim=-1)
    c = cos.unsqueeze(-2).to(x.dtype)
    s = (sin * direction).unsqueeze(-2).to(x.dtype)
    return torch.cat((re * c - im * s, im * c + re * s), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate ``x`` [n, H, hd] by its positions' angles (cos/sin [n, hd/2])."""
    return _rotate(x, cos, sin, 1.0)


def rope_backward(g: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Gradient through :func:`apply_rope`: a rotation is orthogonal, so its
    transpose is the rotation by the opposite angle."""
    return _rotate(g, cos, sin, -1.0)
