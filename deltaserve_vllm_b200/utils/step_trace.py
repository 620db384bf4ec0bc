"""Per-step predicted-vs-actual trace for estimator validation
(``telemetry.step_trace_path``): one CSV row per timed step written by a
daemon thread, so the engine thread only formats a few floats per step
(reference columns: ``deltaserve-plugin/deltaserve/step_trace.py:48-114``)."""

from __future__ import annotations

import os
import queue
import threading
import time

COLUMNS = ("seq", "kind", "t_done", "regime", "regime_used", "t_in", "p", "t_ft", "b_d", "k", "s",
           "pred_raw", "pred", "actual", "admit_code", "t_baseline", "t_admit", "bwd_in_flight")


def _f(v) -> str:
    """One CSV cell: empty for a missing value, 0/1 for flags, six
    significant digits for floats (six decimals for wall-clock stamps, whose
    integer part alone has ten digits)."""
    if v is None:
        return ""
    if isinstance(v, float):
        return format(v, ".6f" if abs(v) >= 1e6 else ".6g")
    return str(int(v)) if isinstance(v, bool) else str(v)


class StepTraceWriter:
    def __init__(self, path: str, flush_every_s: float = 1.0):
        self.path = path
        if os.path.dirname(path):
            os.makedirs(os.path.dirname(path), exist_ok=True)
        self.q: queue.Queue = queue.Queue()
        self.flush_every_s = flush_every_s
        self.seq = 0
        self.t = threading.Thread(target=self._run, daemon=True, name="dsv-step-trace")
        self.t.start()

    def put_row(self, **kw) -> None:
        self.seq += 1
        kw.setdefault("seq", self.seq)
        self.q.put(",".join(_f(kw.get(c)) for c in COLUMNS))

    def _run(self) -> None:
        with open(self.path, "w") as f:
            f.write(",".join(COLUMNS) + "\n")
            last = time.time()
            while True:
                line = self.q.get()
                if line is None:
                    f.flush()
                    return
                f.write(line + "\n")
                if time.time() - last > self.flush_every_s:
                    f.flush()
                    last = time.time()

    def close(self) -> None:
        self.q.put(None)
        self.t.join(timeout=5)


def attach_step_trace(engine, path: str) -> StepTraceWriter:
    """Stream every timed step of ``engine`` into ``path``."""
    w = StepTraceWriter(path)
    est = engine.estimator

    def on_step(rec, dur):
        f = rec.features
        adm = engine.last_admit
        w.put_row(kind=rec.kind, t_done=time.time(), regime=est.regime_of(f),
                  regime_used=est.select_regime(f), t_in=f.t_in, p=f.p, t_ft=f.t_ft, b_d=f.b_d, k=f.k,
                  s=f.s, pred_raw=est.predict(f, apply_margin=False) if est.is_ready else None,
                  pred=rec.predicted, actual=dur, admit_code=adm.code if adm else None,
                  t_baseline=adm.baseline if adm else None, t_admit=adm.predicted if adm else None,
                  bwd_in_flight=f.bwd)
    engine.step_listeners.append(on_step)
    return w
