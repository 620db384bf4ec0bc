"""Launch-time profiling shapes that seed the step-time estimator.

Each shape is driven through real engine steps (synthetic token ids, no
outputs kept) so the estimator sees every regime before serving starts:
prefill sweeps (token count and request count), decode grids (batch and
context), co-served prefill+FT, mixed decode+prefill, FT on decode-only steps
and FT-only steps (the same shape families as the reference's generator,
``deltaserve-plugin/deltaserve/profiling_batch_generator.py:38-259``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field


@dataclass
class ProfileShape:
    kind: str                                   # prefill | decode | coserve | mixed | ft_only
    inf_lens: list[int] = field(default_factory=list)
    ft_lens: list[int] = field(default_factory=list)
    mix_lens: list[int] = field(default_factory=list)
    n_decode: int = 0


class ProfilingShapeGenerator:
    def __init__(self, batch_max_tokens: int, max_saved_finetuning_tokens: int, max_req_len: int,
                 max_ft_sample: int | None = None):
        self.T = int(batch_max_tokens)
        self.ft_cap = max(1, int(max_saved_finetuning_tokens))
        self.max_req = max(16, int(max_req_len) - 16)
        self.inf_cap = max(64, min(self.T, 4096))
        self.ft_sample = max(8, min(max_ft_sample or self.ft_cap, self.ft_cap))

    def _split(self, total: int, n: int) -> list[int]:
        n = max(1, min(n, total))
        n = max(n, math.ceil(total / self.max_req))
        b, r = divmod(total, n)
        return [b + 1] * r + [b] * (n - r)

    def _ft(self, total: int) -> list[int]:
        total = min(total, self.ft_cap)
        return self._split(total, max(1, math.ceil(total / self.ft_sample)))

    def prefill(self) -> list[ProfileShape]:
        out = []
        tgts = sorted({t for t in (64, 128, 256, 512, 1024, 2048, 4096) if t <= self.inf_cap}
                      | {max(64, int(self.inf_cap * f)) for f in (0.5, 0.75, 1.0)})
        for t in tgts:
            out.append(ProfileShape("prefill", inf_lens=self._split(t, max(1, min(8, t // 128)))))
        for t in (min(512, self.inf_cap), min(2048, self.inf_cap)):
            if t >= 256:
                for n in (1, 4, max(4, t // 64)):
                    out.append(ProfileShape("prefill", inf_lens=self._split(t, n)))
        return out

    def decode(self) -> list[ProfileShape]:
        out = []
        for b in (1, 4, 16, 32, 64):
            out.append(ProfileShape("decode", inf_lens=[128] * b, n_decode=4))
        for ctx in (512, 1024, 2048):
            if ctx <= self.max_req:
                out.append(ProfileShape("decode", inf_lens=[ctx] * 8, n_decode=4))
        return out

    def coserve(self) -> list[ProfileShape]:
        out = []
        for inf in (128, 512, 1024):
            for ft in (self.ft_sample, 2 * self.ft_sample, self.ft_cap):
                if inf + min(ft, self.ft_cap) <= self.T:
                    out.append(ProfileShape("coserve", inf_lens=self._split(inf, 2), ft_lens=self._ft(ft)))
        return out

    def mixed(self) -> list[ProfileShape]:
        return [ProfileShape("mixed", inf_lens=[128] * b, mix_lens=self._split(p, 2), n_decode=1)
                for b in (4, 16) for p in (256, 1024) if b * 128 + p <= self.T]

    def ft_on_decode(self) -> list[ProfileShape]:
        return [ProfileShape("decode", inf_lens=[128] * b, ft_lens=self._ft(ft), n_decode=1)
                for b in (4, 16) for ft in (self.ft_sample, self.ft_cap) if b + ft <= self.T]

    def ft_only(self) -> list[ProfileShape]:
        sizes = sorted({self.ft_sample, min(self.ft_cap, 2 * self.ft_sample), self.ft_cap})
        return [ProfileShape("ft_only", ft_lens=self._ft(s)) for s in sizes if s <= self.T]

    def prepare(self, with_ft: bool = True) -> tuple[list[ProfileShape], list[ProfileShape]]:
        rec = self.prefill() + self.decode() + self.mixed()
        if with_ft:
            rec += self.coserve() + self.ft_on_decode() + self.ft_only()
        warm = [ProfileShape("prefill", inf_lens=[256, 256]),
                ProfileShape("decode", inf_lens=[128, 128], n_decode=1)]
        if with_ft:
            warm.append(ProfileShape("coserve", inf_lens=[128], ft_lens=self._ft(min(64, self.ft_cap))))
        return warm, rec
