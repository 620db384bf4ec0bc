"""Run telemetry: per-request and per-backward CSVs, windowed summaries, GPU
time by step kind, memory snapshots, a rolling per-step log and the live feed
behind ``GET /system_metrics`` / ``/telemetry/data``.

Same outputs as the reference recorder (``deltaserve-plugin/deltaserve/metrics.py:1-48``):

* ``requests.csv``  — one row per finished inference request (TTFT, TBT
  mean/max, latency, tokens);
* ``backward.csv``  — one row per backward cycle (GPU ms, wall ms, tokens,
  loss, memory);
* ``summary.jsonl`` — every ``metrics_interval_s``: TTFT/TBT percentiles and
  SLO attainment of the window, inference and FT token throughput, forward GPU
  seconds by step kind (inference / mixed / FT-only; mixed steps split by
  tokens), backward GPU seconds, run totals;
* ``memory_rank<r>.json`` — weights, KV cache, capture buffers, other;
* ``steps.<n>.jsonl.gz`` — rolling per-step log (decode-only runs folded),
  capped at ``steps_log_max_mb``.

All file writes happen on one daemon thread; the engine thread only appends to
in-memory structures (a few dict operations per step).
"""

from __future__ import annotations

import csv
import gzip
import json
import os
import queue
import threading
import time
from collections import deque

import numpy as np

REQ_FIELDS = ("finish_time", "request_id", "adapter", "prompt_tokens", "output_tokens", "ttft_s",
              "tbt_mean_s", "tbt_max_s", "e2e_s")
BWD_FIELDS = ("time", "cycle", "tokens", "loss", "gpu_ms", "wall_ms", "mem_gb")


def _pct(x, q):
    return float(np.percentile(np.asarray(x), q)) if len(x) else None


class _Writer:
    """Daemon thread owning every telemetry file handle."""

    def __init__(self):
        self.q: queue.Queue = queue.Queue()
        self.t = threading.Thread(target=self._run, daemon=True, name="dsv-metrics")
        self.t.start()

    def put(self, fn) -> None:
        self.q.put(fn)

    def _run(self):
        while True:
            fn = self.q.get()
            if fn is None:
                return
            try:
                fn()
            except Exception:
                pass

    def close(self):
        self.q.put(None)
        self.t.join(timeout=5)


class RollingGz:
    """Append-only gzip JSON-lines segments, oldest deleted past ``max_mb``."""

    def __init__(self, directory: str, prefix: str = "steps", max_mb: float = 256.0,
                 segment_mb: float = 16.0):
        self.dir, self.prefix = directory, prefix
        self.max_bytes = int(max_mb * (1 << 20))
        self.seg_bytes = int(segment_mb * (1 << 20))
        self.n = 0
        self.cur = None
        self.cur_bytes = 0

    def _open(self):
        if self.cur is not None:
            self.cur.close()
        self.n += 1
        self.cur = gzip.open(os.path.join(self.dir, f"{self.prefix}.{self.n}.jsonl.gz"), "at")
        self.cur_bytes = 0
        self._prune()

    def _prune(self):
        segs = sorted((int(f.split(".")[1]), f) for f in os.listdir(self.dir)
                      if f.startswith(self.prefix + ".") and f.endswith(".jsonl.gz"))
        total = sum(os.path.getsize(os.path.join(self.dir, f)) for _, f in segs)
        while segs and total > self.max_bytes and len(segs) > 1:
            _, f = segs.pop(0)
            total -= os.path.getsize(os.path.join(self.dir, f))
            os.remove(os.path.join(self.dir, f))

    def write(self, rec: dict) -> None:
        if self.max_bytes <= 0:
            return
        if self.cur is None or self.cur_bytes > self.seg_bytes:
            self._open()
        line = json.dumps(rec, separators=(",", ":")) + "\n"
        self.cur.write(line)
        self.cur_bytes += len(line)

    def close(self):
        if self.cur is not None:
            self.cur.close()
            self.cur = None


class MetricsRecorder:
    def __init__(self, engine, directory: str | None, interval_s: float = 10.0,
                 steps_log_max_mb: float = 256.0, rank: int = 0):
        self.eng = engine
        self.dir = directory
        self.interval_s = float(interval_s)
        self.rank = rank
        self.ttft_slo = engine.ftcfg.ttft_slo
        self.tbt_slo = engine.ftcfg.avg_tbt_slo
        self.t0 = time.time()
        self.window_start = time.time()
        self._win = self._new_window()
        self.totals = {"requests": 0, "inf_tokens": 0, "ft_tokens": 0, "bwd_cycles": 0,
                       "bwd_gpu_s": 0.0,
                       "fwd_gpu_s": {"inference": 0.0, "mixed": 0.0, "mixed_ft_share": 0.0, "ft_only": 0.0}}
        self.series: deque = deque(maxlen=3600)   # per-second (inf tok, ft tok)
        self.steps: deque = deque(maxlen=4096)    # live step stream (decode runs folded)
        self.step_seq = 0
        self.last_summary: dict | None = None
        self._writer = _Writer() if directory else None
        self._gz = None
        if directory:
            os.makedirs(directory, exist_ok=True)
            self._gz = RollingGz(directory, max_mb=steps_log_max_mb)
            self._csv_header("requests.csv", REQ_FIELDS)
            self._csv_header("backward.csv", BWD_FIELDS)
        engine.step_listeners.append(self.on_step)
        engine.request_listeners.append(self.on_request)
        engine.backward_listeners.append(self.on_backward)
        self.active = True

    @staticmethod
    def _new_window():
        return {"ttft": [], "tbt": [], "req_ok": 0, "req_n": 0, "inf_tokens": 0, "ft_tokens": 0,
                "fwd": {"inference": 0.0, "mixed": 0.0, "mixed_ft_share": 0.0, "ft_only": 0.0}, "bwd_s": 0.0, "steps": 0}

    def _csv_header(self, name, fields):
        path = os.path.join(self.dir, name)
        if not os.path.exists(path):
            with open(path, "w", newline="") as f:
                csv.writer(f).writerow(fields)

    def _append_csv(self, name, row):
        if self._writer is None:
            return
        path = os.path.join(self.dir, name)

        def w():
            with open(path, "a", newline="") as f:
                csv.writer(f).writerow(row)
        self._writer.put(w)

    # ------------------------------------------------------------ hooks
    def on_step(self, rec, dur_s: float) -> None:
        if not self.active:
            return
        f = rec.features
        inf_tokens = int(f.t_in - f.t_ft + f.b_d)
        kind = "ft_only" if (f.t_ft > 0 and inf_tokens == 0) else ("mixed" if f.t_ft > 0 else "inference")
        w = self._win
        if kind == "mixed":  # also split the step's time between the two by tokens
            ft_share = dur_s * f.t_ft / max(1.0, f.t_in + f.b_d)
            w["fwd"]["mixed"] += dur_s
            w["fwd"]["mixed_ft_share"] += ft_share
            self.totals["fwd_gpu_s"]["mixed"] += dur_s
            self.totals["fwd_gpu_s"]["mixed_ft_share"] += ft_share
        else:
            w["fwd"][kind] += dur_s
            self.totals["fwd_gpu_s"][kind] += dur_s
        w["inf_tokens"] += inf_tokens
        w["ft_tokens"] += int(f.t_ft)
        w["steps"] += 1
        self.totals["inf_tokens"] += inf_tokens
        self.totals["ft_tokens"] += int(f.t_ft)
        self.step_seq += 1
        s = {"seq": self.step_seq, "t": time.time(), "kind": kind, "t_in": f.t_in, "t_ft": f.t_ft,
             "b_d": f.b_d, "k": f.k, "gpu_ms": round(dur_s * 1e3, 3),
             "pred_ms": None if rec.predicted is None else round(rec.predicted * 1e3, 3),
             "bwd": bool(f.bwd)}
        last = self.steps[-1] if self.steps else None
        if (last is not None and kind == "inference" and f.t_in == 0 and last.get("t_in") == 0
                and last["kind"] == "inference" and last["b_d"] == f.b_d):
            last["n"] = last.get("n", 1) + 1      # fold a decode-only run
            last["gpu_ms"] = round(last["gpu_ms"] + s["gpu_ms"], 3)
        else:
            self.steps.append(s)
        if self._gz is not None:
            gz = self._gz
            self._writer.put(lambda: gz.write(s))
        self._maybe_summary()

    def on_request(self, kind: str, req) -> None:
        if not self.active or kind != "finish" or req.is_ft:
            return
        ttft = req.ttft()
        gaps = req.tbts()
        w = self._win
        if ttft is not None:
            w["ttft"].append(ttft)
        w["tbt"].extend(gaps)
        w["req_n"] += 1
        ok = ttft is not None and ttft <= self.ttft_slo and (not gaps or np.mean(gaps) <= self.tbt_slo)
        w["req_ok"] += int(ok)
        self.totals["requests"] += 1
        e2e = (req.finish_time - req.arrival_time) if req.finish_time else None
        self._append_csv("requests.csv", [time.time(), req.request_id, req.adapter or "", req.num_prompt,
                                          len(req.output_ids), ttft, float(np.mean(gaps)) if gaps else None,
                                          max(gaps) if gaps else None, e2e])

    def on_backward(self, res) -> None:
        if not self.active:
            return
        self._win["bwd_s"] += res.gpu_ms / 1e3
        self.totals["bwd_cycles"] += 1
        self.totals["bwd_gpu_s"] += res.gpu_ms / 1e3
        mem = None
        try:
            import torch
            if torch.cuda.is_available():
                mem = torch.cuda.memory_allocated() / 1e9
        except Exception:
            pass
        self._append_csv("backward.csv", [time.time(), self.totals["bwd_cycles"], res.n_tokens, res.loss,
                                          res.gpu_ms, res.wall_ms, mem])

    # ------------------------------------------------------------ summaries
    def window_summary(self) -> dict:
        w = self._win
        dt = max(1e-6, time.time() - self.window_start)
        return {"time": time.time(), "window_s": dt,
                "ttft_p50_s": _pct(w["ttft"], 50), "ttft_p99_s": _pct(w["ttft"], 99),
                "tbt_p50_s": _pct(w["tbt"], 50), "tbt_p99_s": _pct(w["tbt"], 99),
                "slo_attainment": (w["req_ok"] / w["req_n"]) if w["req_n"] else None,
                "requests": w["req_n"], "inf_tok_s": w["inf_tokens"] / dt, "ft_tok_s": w["ft_tokens"] / dt,
                "fwd_gpu_s": dict(w["fwd"]), "bwd_gpu_s": w["bwd_s"], "steps": w["steps"],
                "totals": json.loads(json.dumps(self.totals))}

    def _maybe_summary(self) -> None:
        if time.time() - self.window_start < self.interval_s:
            return
        s = self.window_summary()
        self.last_summary = s
        self.series.append((s["time"], s["inf_tok_s"], s["ft_tok_s"]))
        if self.dir:
            path = os.path.join(self.dir, "summary.jsonl")

            def w():
                with open(path, "a") as f:
                    f.write(json.dumps(s) + "\n")
            self._writer.put(w)
        self._win = self._new_window()
        self.window_start = time.time()

    def snapshot(self) -> dict:
        return {"current": self.window_summary(), "last": self.last_summary,
                "totals": json.loads(json.dumps(self.totals)), "uptime_s": time.time() - self.t0}

    def data(self, steps_since: int = 0) -> dict:
        return {"steps": [s for s in self.steps if s["seq"] > steps_since],
                "series": list(self.series)[-600:], "summary": self.window_summary()}

    def memory_snapshot(self, root: str | None = None) -> dict:
        e = self.eng
        def nbytes(ts):
            return sum(t.numel() * t.element_size() for t in ts)
        w = e.weights
        weights = nbytes([w.embed, w.final_norm] + ([w.lm_head] if w.lm_head is not w.embed else [])
                         + ([w.lm_head_full] if w.lm_head_full is not None else [])
                         + [getattr(L, f) for L in w.layers for f in
                            ("qkv", "o", "gate_up", "down", "in_ln", "post_ln")])
        snap = {"rank": self.rank, "weights_gb": weights / 1e9, "kv_cache_gb": e.kv.nbytes() / 1e9,
                "ft_buffers_gb": (e.capture.nbytes() / 1e9) if e.capture is not None else 0.0}
        try:
            import torch
            if torch.cuda.is_available():
                snap["allocated_gb"] = torch.cuda.memory_allocated() / 1e9
                snap["reserved_gb"] = torch.cuda.memory_reserved() / 1e9
                snap["other_gb"] = snap["reserved_gb"] - snap["weights_gb"] - snap["kv_cache_gb"] - snap["ft_buffers_gb"]
        except Exception:
            pass
        root = root or self.dir
        if root:
            os.makedirs(root, exist_ok=True)
            with open(os.path.join(root, f"memory_rank{self.rank}.json"), "w") as f:
                json.dump(snap, f, indent=2)
        return snap

    def close(self) -> None:
        self.active = False
        if self._writer is not None:
            if self._gz is not None:
                gz = self._gz
                self._writer.put(gz.close)
            self._writer.close()
