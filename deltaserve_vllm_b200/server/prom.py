"""Prometheus text exposition for ``GET /metrics``.

``ServingStats`` listens to the engine's request events (on the engine
thread) and keeps counters and fixed-bucket histograms of the served
requests; :func:`render` turns them, plus gauges read from the engine
(queues, KV-cache use, finetuning progress), into the Prometheus text format
(version 0.0.4). It plays the role of the ``/metrics`` route of the vLLM
OpenAI server the reference runs under (its ``vllm:*`` families); names here
carry a ``dserve:`` prefix and the finetuning gauges have no vLLM
counterpart.
"""

from __future__ import annotations

import math
import threading

TTFT_BUCKETS = (0.01, 0.025, 0.05, 0.075, 0.1, 0.15, 0.2, 0.3, 0.4, 0.5, 0.75, 1.0, 2.5, 5.0, 10.0)
TBT_BUCKETS = (0.005, 0.01, 0.02, 0.03, 0.04, 0.05, 0.06, 0.08, 0.1, 0.15, 0.25, 0.5, 1.0)
E2E_BUCKETS = (0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0, 20.0, 40.0, 60.0, 120.0)


class _Histogram:
    def __init__(self, buckets):
        self.buckets = tuple(buckets)
        self.counts = [0] * len(self.buckets)
        self.sum = 0.0
        self.n = 0

    def observe(self, v: float) -> None:
        for i, b in enumerate(self.buckets):
            if v <= b:
                self.counts[i] += 1
                break
        self.sum += v
        self.n += 1

    def lines(self, name: str) -> list[str]:
        out, acc = [], 0
        for b, c in zip(self.buckets, self.counts):
            acc += c
            out.append(f'{name}_bucket{{le="{_num(b)}"}} {acc}')
        out.append(f'{name}_bucket{{le="+Inf"}} {self.n}')
        out.append(f"{name}_sum {_num(self.sum)}")
        out.append(f"{name}_count {self.n}")
        return out


def _num(v) -> str:
    if isinstance(v, bool):
        return "1" if v else "0"
    if isinstance(v, int):
        return str(v)
    v = float(v)
    if math.isnan(v):
        return "NaN"
    if math.isinf(v):
        return "+Inf" if v > 0 else "-Inf"
    return repr(v)


class ServingStats:
    """Counters and histograms of the inference requests that finished."""

    def __init__(self):
        self.lock = threading.Lock()
        self.prompt_tokens = 0
        self.generation_tokens = 0
        self.cached_prompt_tokens = 0
        self.finished: dict[str, int] = {}
        self.ttft = _Histogram(TTFT_BUCKETS)
        self.tbt = _Histogram(TBT_BUCKETS)
        self.e2e = _Histogram(E2E_BUCKETS)

    def on_request(self, kind: str, req) -> None:
        if kind not in ("finish", "abort") or getattr(req, "is_ft", False):
            return
        from .api import _finish_reason
        reason = "abort" if kind == "abort" else _finish_reason(req)
        ttft = req.ttft()
        tbts = req.tbts()
        with self.lock:
            self.prompt_tokens += req.num_prompt
            self.generation_tokens += len(req.output_ids)
            self.cached_prompt_tokens += getattr(req, "num_cached_tokens", 0)
            self.finished[reason] = self.finished.get(reason, 0) + 1
            if ttft is not None:
                self.ttft.observe(ttft)
            for t in tbts:
                self.tbt.observe(t)
            if req.finish_time is not None:
                self.e2e.observe(req.finish_time - req.arrival_time)


def _family(out: list[str], name: str, kind: str, help_: str, samples) -> None:
    out.append(f"# HELP {name} {help_}")
    out.append(f"# TYPE {name} {kind}")
    if isinstance(samples, list):
        out.extend(samples)
    else:
        out.append(f"{name} {_num(samples)}")


def render(stats: ServingStats, engine, model_name: str) -> str:
    """The exposition text. Engine gauges are read without stopping the
    engine thread (single Python attribute reads)."""
    out: list[str] = []
    lab = f'model_name="{model_name}"'
    sched = engine.scheduler
    with stats.lock:
        _family(out, "dserve:prompt_tokens_total", "counter", "Prompt tokens of finished requests.",
                [f"dserve:prompt_tokens_total{{{lab}}} {stats.prompt_tokens}"])
        _family(out, "dserve:generation_tokens_total", "counter", "Generated tokens of finished requests.",
                [f"dserve:generation_tokens_total{{{lab}}} {stats.generation_tokens}"])
        _family(out, "dserve:prefix_cache_hit_tokens_total", "counter",
                "Prompt tokens served from the prefix cache.",
                [f"dserve:prefix_cache_hit_tokens_total{{{lab}}} {stats.cached_prompt_tokens}"])
        _family(out, "dserve:request_success_total", "counter", "Finished requests by finish reason.",
                [f'dserve:request_success_total{{{lab},finished_reason="{k}"}} {v}'
                 for k, v in sorted(stats.finished.items())])
        for name, h, help_ in (("dserve:time_to_first_token_seconds", stats.ttft, "Time to first token."),
                               ("dserve:time_per_output_token_seconds", stats.tbt,
                                "Time between consecutive output tokens."),
                               ("dserve:e2e_request_latency_seconds", stats.e2e, "Arrival to finish.")):
            _family(out, name, "histogram", help_, h.lines(name))
    running = sum(1 for r in list(sched.running) if not r.is_ft)
    waiting = sum(1 for r in list(sched.waiting) if not r.is_ft)
    _family(out, "dserve:num_requests_running", "gauge", "Inference requests in the running batch.",
            [f"dserve:num_requests_running{{{lab}}} {running}"])
    _family(out, "dserve:num_requests_waiting", "gauge", "Inference requests waiting to be scheduled.",
            [f"dserve:num_requests_waiting{{{lab}}} {waiting}"])
    _family(out, "dserve:kv_cache_usage_perc", "gauge", "Fraction of KV-cache pages in use (0..1).",
            [f"dserve:kv_cache_usage_perc{{{lab}}} {_num(engine.kv.allocator.usage())}"])
    _family(out, "dserve:engine_steps_total", "counter", "Engine steps run.",
            [f"dserve:engine_steps_total{{{lab}}} {engine.stats.get('steps', 0)}"])
    # finetuning progress (no vLLM counterpart)
    st = engine.coord.status()
    ft = [("dserve:ft_enabled", "gauge", "Finetuning enabled and not disabled by a failure.",
           bool(engine.ft_enabled and not st["disabled"])),
          ("dserve:ft_started", "gauge", "Finetuning started.", bool(st["ft_started"])),
          ("dserve:ft_tokens_forwarded_total", "counter", "FT tokens run through the co-served forward.",
           engine.stats.get("ft_tokens_forwarded", 0)),
          ("dserve:ft_tokens_trained_total", "counter", "FT tokens whose backward finished.",
           engine.stats.get("ft_tokens_trained", 0)),
          ("dserve:ft_backward_cycles_total", "counter", "Backward cycles finished.", st["completed_cycles"]),
          ("dserve:ft_buffer_fill", "gauge", "Captured FT tokens waiting for the next backward.", st["fill"]),
          ("dserve:ft_buffer_capacity", "gauge", "Capacity of the activation-capture buffer (tokens).",
           st["capacity"]),
          ("dserve:ft_aborts_total", "counter", "FT-only forwards pre-empted between layers.",
           engine.stats.get("ft_aborts", 0)),
          ("dserve:ft_epoch", "gauge", "Current finetuning epoch.", st["epoch"])]
    if st["last_loss"] is not None:
        ft.append(("dserve:ft_last_loss", "gauge", "Loss of the last finished backward cycle.", st["last_loss"]))
    for name, kind, help_, v in ft:
        _family(out, name, kind, help_, [f"{name}{{{lab}}} {_num(v)}"])
    return "\n".join(out) + "\n"
