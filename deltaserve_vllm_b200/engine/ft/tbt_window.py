"""Recent time-between-tokens of the served requests, for the ``avg_tbt_slo``
admission check (the quantity the reference computes in
``deltaserve-plugin/deltaserve/tbt_window.py:26-83``: over the decode steps of
the last ``window_s`` seconds, the token-weighted mean gap
``sum(tokens * gap) / sum(tokens)``).

Design: a fixed-size ring of step records held in numpy arrays (end time,
decode tokens, tokens x gap). Queries mask the ring by age and sum it, so
nothing has to be trimmed or kept consistent between calls; the ring holds
far more steps than any window sees (one step per few milliseconds), and when
it wraps the oldest records are simply overwritten.

The gap a decode token waited is measured from the previous step's end. Two
cases change that:

* a step without decode tokens while requests are still running (an FT-only
  step, a prefill of new arrivals only) delays the next token as well: its
  time is owed by the next decode step's tokens;
* a gap longer than ``idle_gap_s`` means the engine was idle, not that a
  token was late: it starts a fresh measurement.
"""

from __future__ import annotations

import numpy as np


class DecodeGapWindow:
    def __init__(self, window_s: float, idle_gap_s: float = 1.0, capacity: int = 8192):
        self.window_s = float(window_s)
        self.idle_gap_s = float(idle_gap_s)
        self._t_end = np.full(capacity, -np.inf)      # step end time (perf_counter s)
        self._tokens = np.zeros(capacity)             # decode tokens of the step
        self._weighted = np.zeros(capacity)           # tokens * gap they waited
        self._next = 0                                # slot the next record goes to
        self._last_end: float | None = None
        self._owed = 0.0                              # delay the next decode tokens inherit

    def note_step(self, t_end: float, decode_tokens: int, inference_active: bool) -> None:
        """One engine step ended at ``t_end`` with ``decode_tokens`` decode rows."""
        prev, self._last_end = self._last_end, t_end
        if prev is None or t_end - prev > self.idle_gap_s:
            self._owed = 0.0
            return
        waited = (t_end - prev) + self._owed
        if decode_tokens <= 0:
            # Nobody got a token: the running requests' next tokens wait this
            # step too (or, with nothing running, there is nothing to owe).
            self._owed = waited if inference_active else 0.0
            return
        i = self._next
        self._t_end[i] = t_end
        self._tokens[i] = decode_tokens
        self._weighted[i] = decode_tokens * waited
        self._next = (i + 1) % self._t_end.size
        self._owed = 0.0

    def _sums(self, now: float) -> tuple[float, float]:
        live = self._t_end >= now - self.window_s
        return float(self._tokens[live].sum()), float(self._weighted[live].sum())

    def mean(self, now: float) -> float | None:
        """Token-weighted mean gap over the window (None without decode steps)."""
        tok, wsum = self._sums(now)
        return wsum / tok if tok > 0 else None

    def mean_with(self, now: float, decode_tokens: int, step_s: float) -> float:
        """The mean if a step of ``step_s`` seconds with ``decode_tokens``
        decode rows ran next (0 when there would be no decode token at all)."""
        tok, wsum = self._sums(now)
        tok += decode_tokens
        if tok <= 0:
            return 0.0
        return (wsum + decode_tokens * (step_s + self._owed)) / tok
