"""SLO-aware finetuning admission for one step.

Given the inference part of the next step (already scheduled, so its
composition is exact), decide how many FT samples ride along. The algorithm
is the reference's iterative admission (``deltaserve-plugin/deltaserve/ft_scheduler.py:562-844``):

0. preconditions (finetuning started, no backward pending, buffer space, corpus);
1. phase gate (``prefill``: no FT on decode-only steps);
2. baseline prediction without FT and headroom checks: max TBT (x the
   decode-only safety margin in ``both`` phase), windowed average TBT, and the
   TTFT deadline ``earliest_arrival + 0.9 * ttft_slo``;
3. shapers: the leaky prefill-credit bucket (``match_prefill_workload_factor``)
   and the proportional cap (``ft_tokens_admission_constrain_factor``);
4. greedy smallest-first loop: each candidate is predicted with the regime of
   the hypothetical step and accepted only if every SLO check still holds.

Every decision leaves an admission code (A/S/F/C/B/T/X/E/D/K).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

from .estimator import (REGIME_DECODE_ONLY, REGIME_DECODE_BWD, REGIME_INF_PREFILL,
                        MergedExecutionEstimator, StepFeatures)

ADMIT_CODES = {
    "A": "admitted",
    "S": "SLO: no headroom / cut short",
    "F": "buffer: admitted what fit / full",
    "C": "step budget: admitted what fit / none left",
    "B": "backward running",
    "T": "admission closed (throttle / epoch flush)",
    "X": "finetuning not started / disabled",
    "E": "corpus finished",
    "D": "decode-only step (admission phase prefill)",
    "K": "waiting for prefill credit (match_prefill_workload_factor)",
    "": "no admission attempted",
}


@dataclass
class AdmissionResult:
    samples: list = field(default_factory=list)
    tokens: int = 0
    code: str = ""
    baseline: float | None = None
    predicted: float | None = None


class FinetuneAdmission:
    def __init__(self, cfg, estimator: MergedExecutionEstimator, coord, store,
                 max_num_batched_tokens: int, tbt_window=None):
        self.cfg = cfg
        self.est = estimator
        self.coord = coord
        self.store = store
        self.max_tokens = int(max_num_batched_tokens)
        self.tbt_window = tbt_window
        self.unspent_prefill = 0
        self.last = AdmissionResult()

    def features(self, out, bwd_in_flight: bool = False) -> StepFeatures:
        lens = [s.num_new for s in out.prefill]
        return StepFeatures(t_in=float(sum(lens)), p=len(lens), t_ft=0.0, b_d=out.b_d,
                            k=float(out.k_decode), prefill_lens=lens or None, bwd=bwd_in_flight)

    def admit(self, out, earliest_arrival: float | None, now: float | None = None,
              bwd_in_flight: bool = False, extra_s: float = 0.0) -> AdmissionResult:
        cfg, coord, store, est = self.cfg, self.coord, self.store, self.est
        now = time.perf_counter() if now is None else now
        res = AdmissionResult()
        self.last = res
        if coord.next_ft_budget() <= 0:
            res.code = ("X" if (not coord.ft_started or coord.disabled) else
                        "B" if coord.pending_backward else
                        "T" if not coord.admission_open else "F")
            return res
        if store.finished() or (not store.has_next() and not store.advance_epoch()):
            res.code = "E"
            return res
        feats = self.features(out, bwd_in_flight)
        decode_only = feats.t_in == 0 and feats.b_d > 0
        idle = feats.t_in == 0 and feats.b_d == 0
        has_prefill = feats.t_in > 0
        phase = cfg.coserving_admission_phase
        if phase == "prefill" and decode_only:
            res.code = "D"
            return res
        margin = cfg.decode_only_ft_safety_margin if (phase == "both" and decode_only) else 1.0
        if not est.is_ready or idle:
            base = 0.0
        elif decode_only:
            base = est.predict(feats, regime=REGIME_DECODE_BWD if bwd_in_flight else REGIME_DECODE_ONLY)
        else:
            base = est.predict(feats, regime=REGIME_INF_PREFILL)
        base += extra_s
        res.baseline = base
        ttft_deadline = (earliest_arrival + 0.9 * cfg.ttft_slo
                         if has_prefill and earliest_arrival is not None else None)
        tbt = cfg.max_tbt_slo * margin
        use_avg = self.tbt_window is not None and cfg.avg_tbt_window_s > 0
        if est.is_ready:
            if feats.b_d > 0:
                if base >= tbt:
                    res.code = "S"
                    return res
                if use_avg and self.tbt_window.mean_with(now, feats.b_d, base) >= cfg.avg_tbt_slo:
                    res.code = "S"
                    return res
            if ttft_deadline is not None and ttft_deadline - now - base <= 0:
                res.code = "S"
                return res
        # ---- shapers
        max_iter = None
        mf, pf = cfg.match_prefill_workload_factor, cfg.ft_tokens_admission_constrain_factor
        if mf > 0 and has_prefill:
            peek = store.pop_next()
            if peek is None:
                res.code = "E"
                return res
            if (self.unspent_prefill + feats.t_in) * mf >= peek.input_len:
                max_iter = 1
            else:
                self.unspent_prefill += int(feats.t_in)
                res.code = "K"
                return res
        buffer_cap = coord.space_remaining()
        token_cap = buffer_cap
        if pf != -1 and has_prefill:
            token_cap = min(buffer_cap, int(feats.t_in * pf))
        budget_left = int(self.max_tokens - feats.t_in - feats.b_d)
        token_cap = min(token_cap, budget_left, coord.next_ft_budget())
        if token_cap <= 0:
            res.code = "C" if budget_left <= 0 else "F"
            return res
        cap_code = "C" if budget_left < buffer_cap else "F"
        # ---- greedy smallest-first
        admitted: list = []
        t_in, t_ft, p = feats.t_in, 0.0, feats.p
        lens = list(feats.prefill_lens or [])
        stop = "A"
        pred_ok = None
        while True:
            if max_iter is not None and len(admitted) >= max_iter:
                break
            if t_ft >= token_cap:
                stop = cap_code
                break
            if not store.has_next() and not store.advance_epoch():
                break
            cand = store.pop_next(exclude=admitted)
            if cand is None:
                break
            if t_ft + cand.input_len > token_cap:
                stop = cap_code
                break
            hyp = StepFeatures(t_in=t_in + cand.input_len, p=p + 1, t_ft=t_ft + cand.input_len,
                               b_d=feats.b_d, k=feats.k, prefill_lens=lens + [cand.input_len],
                               bwd=bwd_in_flight)
            if est.is_ready:
                t_with = est.predict(hyp, regime=est.regime_of(hyp)) + extra_s
                if feats.b_d > 0:
                    if t_with > tbt:
                        stop = "S"
                        break
                    if use_avg and self.tbt_window.mean_with(now, feats.b_d, t_with) > cfg.avg_tbt_slo:
                        stop = "S"
                        break
                if ttft_deadline is not None and ttft_deadline - now - t_with <= 0:
                    stop = "S"
                    break
                pred_ok = t_with
            admitted.append(cand)
            t_in += cand.input_len
            t_ft += cand.input_len
            p += 1
            lens.append(cand.input_len)
        if not admitted:
            res.code = stop if stop != "A" else "E"
            return res
        store.claim(admitted)
        self.unspent_prefill = 0
        res.samples, res.tokens, res.code, res.predicted = admitted, int(t_ft), stop, pred_ok
        return res
