"""Summaries of replay results and telemetry directories, and A/B comparison.

    python -m deltaserve_vllm_b200.eval.report results.jsonl [--ttft-slo 0.5 --tbt-slo 0.06]
    python -m deltaserve_vllm_b200.eval.report --metrics-dir logs/metrics
    python -m deltaserve_vllm_b200.eval.report --compare a.jsonl b.jsonl
"""

from __future__ import annotations

import argparse
import csv
import json
import os

import numpy as np


def _pct(x, q):
    return round(float(np.percentile(np.asarray(x), q)), 6) if len(x) else None


def summarize(results: list[dict], ttft_slo: float = 0.5, tbt_slo: float = 0.06) -> dict:
    ok = [r for r in results if "error" not in r and r.get("ttft_s") is not None]
    ttft = [r["ttft_s"] for r in ok]
    tbt = [r["tbt_mean_s"] for r in ok if r.get("tbt_mean_s") is not None]
    met = [r for r in ok if r["ttft_s"] <= ttft_slo and (r.get("tbt_mean_s") is None or r["tbt_mean_s"] <= tbt_slo)]
    routed = [r for r in ok if (r.get("headers") or {}).get("x-deltaserve-routing") == "routed"]
    return {"requests": len(results), "completed": len(ok), "errors": len(results) - len(ok),
            "slo_attainment": round(len(met) / len(results), 4) if results else None,
            "ttft_p50_s": _pct(ttft, 50), "ttft_p99_s": _pct(ttft, 99),
            "tbt_p50_s": _pct(tbt, 50), "tbt_p99_s": _pct(tbt, 99),
            "output_tokens": sum(r.get("output_tokens", 0) for r in ok),
            "routed": len(routed)}


def metrics_dir_report(d: str, ttft_slo: float, tbt_slo: float) -> dict:
    out = {}
    p = os.path.join(d, "requests.csv")
    if os.path.exists(p):
        with open(p) as f:
            rows = list(csv.DictReader(f))
        res = [{"ttft_s": float(r["ttft_s"]) if r["ttft_s"] else None,
                "tbt_mean_s": float(r["tbt_mean_s"]) if r["tbt_mean_s"] else None,
                "output_tokens": int(r["output_tokens"])} for r in rows]
        out["requests"] = summarize(res, ttft_slo, tbt_slo)
    p = os.path.join(d, "backward.csv")
    if os.path.exists(p):
        with open(p) as f:
            rows = list(csv.DictReader(f))
        if rows:
            t = [float(r["time"]) for r in rows]
            tok = sum(int(r["tokens"]) for r in rows)
            out["backward"] = {"cycles": len(rows), "tokens": tok,
                               "gpu_ms_mean": round(float(np.mean([float(r["gpu_ms"]) for r in rows])), 3),
                               "ft_tok_s": round(tok / max(1e-9, t[-1] - t[0]), 1) if len(t) > 1 else None,
                               "last_loss": float(rows[-1]["loss"]) if rows[-1]["loss"] else None}
    p = os.path.join(d, "summary.jsonl")
    if os.path.exists(p):
        with open(p) as f:
            lines = [json.loads(ln) for ln in f if ln.strip()]
        if lines:
            out["windows"] = len(lines)
            out["last_window"] = lines[-1]
    return out


def compare(a: dict, b: dict) -> dict:
    keys = [k for k in a if isinstance(a.get(k), (int, float)) and isinstance(b.get(k), (int, float))]
    return {k: {"a": a[k], "b": b[k], "delta": round(b[k] - a[k], 6)} for k in keys}


def _load(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(ln) for ln in f if ln.strip()]


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("results", nargs="?")
    ap.add_argument("--metrics-dir")
    ap.add_argument("--compare", nargs=2)
    ap.add_argument("--ttft-slo", type=float, default=0.5)
    ap.add_argument("--tbt-slo", type=float, default=0.06)
    a = ap.parse_args(argv)
    if a.compare:
        sa, sb = (summarize(_load(p), a.ttft_slo, a.tbt_slo) for p in a.compare)
        print(json.dumps(compare(sa, sb), indent=1))
    elif a.metrics_dir:
        print(json.dumps(metrics_dir_report(a.metrics_dir, a.ttft_slo, a.tbt_slo), indent=1))
    elif a.results:
        print(json.dumps(summarize(_load(a.results), a.ttft_slo, a.tbt_slo), indent=1))
    else:
        ap.error("give a results file, --metrics-dir or --compare")


if __name__ == "__main__":
    main()
