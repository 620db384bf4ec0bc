"""Sliding-window average time-between-tokens (``sum(b * gap) / sum(b)`` over
the decode tokens of the last ``window_s`` seconds), used to enforce
``avg_tbt_slo`` at admission (reference: ``deltaserve-plugin/deltaserve/tbt_window.py:26-83``).
Steps that gave no decode token while inference was running carry their gap
into the next decode step; gaps above ``max_gap_s`` (idle engine) are not
token gaps."""

from __future__ import annotations

from collections import deque


class TbtWindow:
    def __init__(self, window_s: float, max_gap_s: float = 1.0):
        self.window_s = float(window_s)
        self.max_gap_s = float(max_gap_s)
        self._steps: deque = deque()
        self._sum_b = 0.0
        self._sum_bt = 0.0
        self._prev: float | None = None
        self._carry = 0.0

    def step_done(self, now: float, decode_requests: int, inference_running: bool) -> None:
        gap = None if self._prev is None else now - self._prev
        self._prev = now
        if gap is None or gap > self.max_gap_s:
            self._carry = 0.0
            return
        if decode_requests > 0:
            bt = decode_requests * (gap + self._carry)
            self._steps.append((now, decode_requests, bt))
            self._sum_b += decode_requests
            self._sum_bt += bt
            self._carry = 0.0
        elif inference_running:
            self._carry += gap
        else:
            self._carry = 0.0

    def _trim(self, now: float) -> None:
        cutoff = now - self.window_s
        while self._steps and self._steps[0][0] < cutoff:
            _, b, bt = self._steps.popleft()
            self._sum_b -= b
            self._sum_bt -= bt
        if not self._steps:
            self._sum_b = self._sum_bt = 0.0

    def average(self, now: float) -> float | None:
        self._trim(now)
        return self._sum_bt / self._sum_b if self._sum_b > 0 else None

    def average_with(self, now: float, decode_requests: int, step_s: float) -> float:
        self._trim(now)
        b = self._sum_b + decode_requests
        if b <= 0:
            return 0.0
        return (self._sum_bt + decode_requests * (step_s + self._carry)) / b
