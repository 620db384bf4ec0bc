"""Logit adjustments of the OpenAI / vLLM sampling options, applied to a
step's fp32 logits (one row per sampled request) before the sampler kernel.

* ``presence_penalty`` / ``frequency_penalty`` (OpenAI): subtract
  ``presence * [count > 0] + frequency * count`` over the request's generated
  tokens;
* ``repetition_penalty`` (vLLM / CTRL): a token seen in the prompt or the
  output has its logit divided by the penalty when positive, multiplied when
  negative;
* ``logit_bias``: added per token id;
* ``min_tokens``: end-of-sequence and ``stop_token_ids`` are masked until the
  request has that many output tokens.

Only rows of requests that set one of them are touched (a few small tensor
ops per such row), and steps that carry them run eagerly (outside the decode
CUDA graphs), like the top-k / top-p sampler path.
"""

from __future__ import annotations

import torch


def apply_penalties(logits: torch.Tensor, reqs, eos_ids=()) -> int:
    """Adjust ``logits`` [R, V] in place for ``reqs`` (row i = reqs[i]).
    Returns the bytes copied host -> device for the adjustments."""
    dev = logits.device
    V = logits.shape[1]
    h2d = 0
    for i, r in enumerate(reqs):
        p = r.params
        if not p.has_penalties:
            continue
        row = logits[i]
        out = r.output_ids
        if (p.presence_penalty or p.frequency_penalty) and out:
            ids = torch.tensor(out, dtype=torch.int64).to(dev, non_blocking=True)
            h2d += 8 * len(out)
            counts = torch.bincount(ids, minlength=V)[:V].to(row.dtype)
            row -= p.frequency_penalty * counts + p.presence_penalty * (counts > 0).to(row.dtype)
        if p.repetition_penalty != 1.0:
            seen = sorted({int(t) for t in r.prompt_ids} | {int(t) for t in out})
            seen = [t for t in seen if 0 <= t < V]
            if seen:
                idx = torch.tensor(seen, dtype=torch.int64).to(dev, non_blocking=True)
                h2d += 8 * len(seen)
                vals = row.index_select(0, idx)
                row.index_copy_(0, idx, torch.where(vals > 0, vals / p.repetition_penalty,
                                                    vals * p.repetition_penalty))
        if p.logit_bias:
            pairs = [(int(t), float(b)) for t, b in p.logit_bias if 0 <= int(t) < V]
            if pairs:
                idx = torch.tensor([t for t, _ in pairs], dtype=torch.int64).to(dev, non_blocking=True)
                b = torch.tensor([v for _, v in pairs], dtype=row.dtype).to(dev, non_blocking=True)
                h2d += 12 * len(pairs)
                row.index_add_(0, idx, b)
        if len(out) < p.min_tokens:
            ban = set(int(t) for t in p.stop_token_ids)
            if not p.ignore_eos:
                ban |= set(int(t) for t in eos_ids)
            ban = sorted(t for t in ban if 0 <= t < V)
            if ban:
                idx = torch.tensor(ban, dtype=torch.int64).to(dev, non_blocking=True)
                h2d += 8 * len(ban)
                row.index_fill_(0, idx, float("-inf"))
    return h2d
