"""Synthetic inference traces (JSONL, one request per line) and trace edits.

    python -m deltaserve_vllm_b200.eval.trace --rate 8 --duration 120 \\
        --prompt-median 512 --prompt-min 32 --prompt-max 4096 --out-min 32 --out-max 256 > trace.jsonl
    # rate schedule (alternating every --period seconds), log-uniform prompts:
    python -m deltaserve_vllm_b200.eval.trace --rates 1.5,3 --period 15 --prompt-dist loguniform \\
        --prompt-min 16 --prompt-max 160 --out-min 64 --out-max 256 > margin_stress.jsonl
    python -m deltaserve_vllm_b200.eval.trace scale --input trace.jsonl --factor 0.5 > half.jsonl
    python -m deltaserve_vllm_b200.eval.trace slice --input trace.jsonl --start 600 --end 800 > cut.jsonl
    python -m deltaserve_vllm_b200.eval.trace from-csv --input timeline.csv --vocab 151936 > trace.jsonl

Generation: Poisson arrivals at ``rate`` req/s, or at a schedule of rates
taken in turn for ``period`` seconds each (peaks and valleys; a rate of 0 is
an idle stretch); prompt lengths lognormal (median, sigma) or log-uniform,
clipped to [min, max]; output lengths uniform; token ids uniform over the
vocabulary. ``--adapters`` spreads requests over named adapters (or ``auto``
for routing).

Edits: ``scale`` changes the request rate and keeps the arrival pattern
(a factor below 1 keeps a seeded random subset at their original times; above
1 it adds copies of requests, each shifted by less than the mean gap);
``slice`` keeps the requests of [start, end) with times rebased to 0;
``from-csv`` reads a timeline CSV with ``timestamp_s``, ``prompt_length`` and
``max_new_tokens`` columns (the reference's timeline files) and draws each
prompt's token ids.
"""

from __future__ import annotations

import argparse
import csv
import json
import sys

import numpy as np


def make_trace(rate: float, duration_s: float, vocab: int, seed: int = 0, prompt_median: int = 512,
               prompt_sigma: float = 0.8, prompt_min: int = 32, prompt_max: int = 4096, out_min: int = 32,
               out_max: int = 256, adapters: list[str] | None = None, rates: list[float] | None = None,
               period_s: float = 15.0, prompt_dist: str = "lognormal", start_s: float = 0.0) -> list[dict]:
    """Requests in arrival order. ``rates`` (if given) replaces ``rate`` with a
    schedule: ``rates[i % len(rates)]`` during [start + i*period, start + (i+1)*period)."""
    rng = np.random.default_rng(seed)
    sched = list(rates) if rates else [rate]
    if not any(r > 0 for r in sched):
        return []
    out: list[dict] = []
    t = start_s
    end = start_s + duration_s
    while t < end:
        i = int((t - start_s) // period_s) if len(sched) > 1 else 0
        r = sched[i % len(sched)]
        seg_end = min(end, start_s + (i + 1) * period_s) if len(sched) > 1 else end
        if r <= 0:                          # an idle stretch: jump to its end
            t = seg_end
            continue
        t_next = t + rng.exponential(1.0 / r)
        if t_next >= seg_end:               # memoryless: restart the draw at the rate change
            t = seg_end
            continue
        t = t_next
        if prompt_dist == "loguniform":
            n = int(round(np.exp(rng.uniform(np.log(prompt_min), np.log(prompt_max)))))
        else:
            n = int(np.clip(rng.lognormal(np.log(prompt_median), prompt_sigma), prompt_min, prompt_max))
        rec = {"t": round(t, 6), "prompt": rng.integers(3, vocab, size=n).tolist(),
               "max_tokens": int(rng.integers(out_min, out_max + 1))}
        if adapters:
            rec["model"] = adapters[int(rng.integers(0, len(adapters)))]
        out.append(rec)
    return out


def scale_trace(trace: list[dict], factor: float, seed: int = 0) -> list[dict]:
    """The same arrival pattern at ``factor`` times the request rate."""
    if factor <= 0:
        raise ValueError("factor must be > 0")
    rng = np.random.default_rng(seed)
    if factor < 1.0:
        keep = int(round(len(trace) * factor))
        idx = np.sort(rng.choice(len(trace), size=keep, replace=False)) if keep else np.array([], int)
        return [dict(trace[i]) for i in idx]
    if len(trace) < 2:
        return [dict(r) for r in trace]
    mean_gap = (trace[-1]["t"] - trace[0]["t"]) / (len(trace) - 1)
    out = [dict(r) for r in trace]
    extra = int(round(len(trace) * (factor - 1.0)))
    for i in rng.integers(0, len(trace), size=extra):
        r = dict(trace[int(i)])
        r["t"] = round(max(0.0, r["t"] + float(rng.uniform(-0.5, 0.5)) * mean_gap), 6)
        out.append(r)
    out.sort(key=lambda r: r["t"])
    return out


def slice_trace(trace: list[dict], start_s: float, end_s: float) -> list[dict]:
    """Requests with ``start <= t < end``, times rebased so ``start`` is 0."""
    out = []
    for r in trace:
        if start_s <= r["t"] < end_s:
            q = dict(r)
            q["t"] = round(r["t"] - start_s, 6)
            out.append(q)
    return out


def from_timeline_csv(path: str, vocab: int, seed: int = 0) -> list[dict]:
    """A timeline CSV (``timestamp_s``, ``prompt_length``, ``max_new_tokens``)
    as a trace with random token ids."""
    rng = np.random.default_rng(seed)
    out = []
    with open(path) as f:
        for row in csv.DictReader(f):
            n = max(1, int(float(row["prompt_length"])))
            out.append({"t": round(float(row["timestamp_s"]), 6), "prompt": rng.integers(3, vocab, size=n).tolist(),
                        "max_tokens": max(1, int(float(row["max_new_tokens"])))})
    out.sort(key=lambda r: r["t"])
    return out


def _read(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(ln) for ln in f if ln.strip()]


def _write(trace: list[dict]) -> None:
    for r in trace:
        sys.stdout.write(json.dumps(r) + "\n")


def main(argv=None) -> None:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] in ("scale", "slice", "from-csv"):
        cmd = argv.pop(0)
        ap = argparse.ArgumentParser(prog=f"trace {cmd}")
        ap.add_argument("--input", required=True)
        ap.add_argument("--seed", type=int, default=0)
        if cmd == "scale":
            ap.add_argument("--factor", type=float, required=True)
            a = ap.parse_args(argv)
            _write(scale_trace(_read(a.input), a.factor, a.seed))
        elif cmd == "slice":
            ap.add_argument("--start", type=float, required=True)
            ap.add_argument("--end", type=float, required=True)
            a = ap.parse_args(argv)
            _write(slice_trace(_read(a.input), a.start, a.end))
        else:
            ap.add_argument("--vocab", type=int, default=128256)
            a = ap.parse_args(argv)
            _write(from_timeline_csv(a.input, a.vocab, a.seed))
        return
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--rates", default=None, help="comma-separated schedule of rates, each for --period s")
    ap.add_argument("--period", type=float, default=15.0)
    ap.add_argument("--start", type=float, default=0.0, help="time of the schedule's start (s)")
    ap.add_argument("--duration", type=float, default=120.0)
    ap.add_argument("--vocab", type=int, default=128256)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--prompt-dist", default="lognormal", choices=["lognormal", "loguniform"])
    ap.add_argument("--prompt-median", type=int, default=512)
    ap.add_argument("--prompt-sigma", type=float, default=0.8)
    ap.add_argument("--prompt-min", type=int, default=32)
    ap.add_argument("--prompt-max", type=int, default=4096)
    ap.add_argument("--out-min", type=int, default=32)
    ap.add_argument("--out-max", type=int, default=256)
    ap.add_argument("--adapters", default=None, help="comma-separated model names to spread over")
    a = ap.parse_args(argv)
    rates = [float(x) for x in a.rates.split(",")] if a.rates else None
    _write(make_trace(a.rate, a.duration, a.vocab, a.seed, a.prompt_median, a.prompt_sigma, a.prompt_min,
                      a.prompt_max, a.out_min, a.out_max, a.adapters.split(",") if a.adapters else None,
                      rates, a.period, a.prompt_dist, a.start))


if __name__ == "__main__":
    main()
