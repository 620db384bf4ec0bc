"""Where the step-time estimator's prediction misses the measured step time.

    python -m deltaserve_vllm_b200.eval.estimator_report step_trace.csv \\
        [--results results.jsonl --ttft-slo 0.5] [--max-tbt-slo 0.06] [--top 10] [--json]
    python -m deltaserve_vllm_b200.eval.estimator_report --compare legacy.csv relative_1.5.csv

``--compare`` prints one line per trace with the admission margin's scores,
for an A/B of ``slo.admission_margin`` (one run per arm, each with its own
``telemetry.step_trace_path``; the reference's ``eval-tp/margin_ab.py``).

Reads the per-step trace the engine writes with ``telemetry.step_trace_path``
(``utils/step_trace.py``: one row per timed step with the raw model
prediction ``pred_raw``, the margined prediction ``pred`` the admission used,
the measured GPU time ``actual`` and the step's features) and reports:

1. accuracy of the raw model per regime: RMSE, bias, percentiles of
   ``actual / pred_raw`` and the share of steps above 1.5x and 2x of it;
2. the same split by backward in flight, step kind and the previous step's
   regime (interference from the co-running backward and regime transitions);
3. margin coverage: the share of steps whose measured time stayed within the
   margined prediction, which is what protects the SLOs;
4. admission fidelity: for steps where finetuning rows were admitted, the time
   the admission loop predicted for the composition it reasoned on
   (``t_admit``) against the step's own prediction and the measured time;
5. over the TBT limit: FT-carrying steps next to running decodes that took
   longer than ``--max-tbt-slo`` (what the margin is there to prevent), with
   inference-only steps as the control;
6. the worst misses with their neighbouring steps;
7. with ``--results`` (``eval.replay`` output, which records each request's
   send wall time): every request over the TTFT SLO with the steps that
   finished while it waited for its first token.

The reference has the same tool for its own trace format
(``eval-tp/analyze_step_trace.py``); this one reads this engine's columns.
"""

from __future__ import annotations

import argparse
import csv
import json
import math

import numpy as np

_NUM = ("t_done", "t_in", "p", "t_ft", "b_d", "k", "s", "pred_raw", "pred", "actual", "t_baseline", "t_admit")


def load_trace(path: str) -> list[dict]:
    """Rows of a step-trace CSV with numeric columns parsed (empty -> None)."""
    rows = []
    with open(path) as f:
        for r in csv.DictReader(f):
            for c in _NUM:
                v = r.get(c)
                r[c] = float(v) if v not in (None, "") else None
            r["seq"] = int(r["seq"]) if r.get("seq") else len(rows) + 1
            r["bwd_in_flight"] = r.get("bwd_in_flight") in ("1", "True", "true")
            rows.append(r)
    return rows


def _stats(pairs: list[tuple[float, float]]) -> dict:
    """pairs: (predicted, actual) seconds with predicted > 0."""
    if not pairs:
        return {"n": 0}
    p = np.array([a for a, _ in pairs])
    y = np.array([b for _, b in pairs])
    ratio = y / p
    return {"n": len(pairs),
            "actual_ms_mean": round(1e3 * float(y.mean()), 3),
            "rmse_ms": round(1e3 * float(np.sqrt(np.mean((p - y) ** 2))), 3),
            "bias_ms": round(1e3 * float(np.mean(p - y)), 3),          # > 0: over-predicts
            "ratio_p50": round(float(np.percentile(ratio, 50)), 3),
            "ratio_p90": round(float(np.percentile(ratio, 90)), 3),
            "ratio_p99": round(float(np.percentile(ratio, 99)), 3),
            "over_1_5x": round(float(np.mean(ratio > 1.5)), 4),
            "over_2x": round(float(np.mean(ratio > 2.0)), 4)}


def _raw_pairs(rows) -> list[tuple[float, float]]:
    return [(r["pred_raw"], r["actual"]) for r in rows
            if r["pred_raw"] is not None and r["pred_raw"] > 0 and r["actual"] is not None]


def _group(rows, key) -> dict:
    out: dict = {}
    for r in rows:
        out.setdefault(str(key(r)), []).append(r)
    return {k: _stats(_raw_pairs(v)) for k, v in sorted(out.items())}


def accuracy(rows: list[dict]) -> dict:
    """Sections 1-3: raw-model accuracy overall, per regime and per split;
    margin coverage per regime."""
    prev = {}
    last = None
    for r in rows:
        prev[r["seq"]] = last
        last = r.get("regime_used") or r.get("regime")
    cover: dict = {}
    for r in rows:
        if r["pred"] is None or r["actual"] is None:
            continue
        c = cover.setdefault(r.get("regime_used") or "", [0, 0])
        c[0] += 1
        c[1] += int(r["actual"] <= r["pred"])
    return {"overall": _stats(_raw_pairs(rows)),
            "by_regime": _group(rows, lambda r: r.get("regime_used") or r.get("regime")),
            "by_backward_in_flight": _group(rows, lambda r: r["bwd_in_flight"]),
            "by_kind": _group(rows, lambda r: r.get("kind")),
            "by_transition": _group(rows, lambda r: f"{prev.get(r['seq'])}->{r.get('regime_used') or r.get('regime')}"),
            "margin_coverage": {k: round(v[1] / v[0], 4) for k, v in sorted(cover.items()) if v[0]}}


def admission_fidelity(rows: list[dict]) -> dict:
    """Section 4: steps that carried admitted finetuning rows."""
    adm = [r for r in rows if r["t_admit"] is not None and r["t_ft"] and r["actual"] is not None]
    if not adm:
        return {"n": 0}
    t_admit = np.array([r["t_admit"] for r in adm])
    y = np.array([r["actual"] for r in adm])
    own = np.array([r["pred"] if r["pred"] is not None else math.nan for r in adm])
    ok = ~np.isnan(own)
    codes: dict = {}
    for r in rows:
        c = r.get("admit_code") or ""
        if c:
            codes[c] = codes.get(c, 0) + 1
    return {"n": len(adm),
            "admit_vs_actual_ms_mean": round(1e3 * float(np.mean(t_admit - y)), 3),
            "actual_over_admit": round(float(np.mean(y > t_admit)), 4),
            "admit_vs_step_prediction_ms_mean": round(1e3 * float(np.mean(t_admit[ok] - own[ok])), 3) if ok.any() else None,
            "admit_codes": dict(sorted(codes.items()))}


def over_limit(rows: list[dict], max_tbt_slo: float) -> dict:
    """What the admission margin is for: steps that carried finetuning rows
    next to running decodes and still took longer than ``max_tbt_slo`` (the
    admission promised the limit and missed), with the same share for
    inference-only steps with decodes as the control, and the ratio of the
    measured time to the admission's prediction on the FT-carrying steps."""
    ft = [r for r in rows if r["t_ft"] and r["b_d"] and r["actual"] is not None]
    ctl = [r for r in rows if not r["t_ft"] and r["b_d"] and r["actual"] is not None]
    ratio = [r["actual"] / r["t_admit"] for r in ft if r["t_admit"]]
    return {"max_tbt_slo_s": max_tbt_slo,
            "ft_steps_with_decodes": len(ft),
            "ft_over_limit": round(sum(r["actual"] > max_tbt_slo for r in ft) / len(ft), 4) if ft else None,
            "inference_steps_with_decodes": len(ctl),
            "inference_over_limit": round(sum(r["actual"] > max_tbt_slo for r in ctl) / len(ctl), 4) if ctl else None,
            "ft_actual_over_admit_p50": round(float(np.percentile(ratio, 50)), 3) if ratio else None,
            "ft_actual_over_admit_p95": round(float(np.percentile(ratio, 95)), 3) if ratio else None}


def worst_misses(rows: list[dict], top: int = 10) -> list[dict]:
    """Section 6: the steps with the largest actual / raw prediction, each with
    the step before and after it."""
    idx = [i for i, r in enumerate(rows) if r["pred_raw"] and r["actual"] is not None]
    idx.sort(key=lambda i: rows[i]["actual"] / rows[i]["pred_raw"], reverse=True)

    def brief(r):
        return {"seq": r["seq"], "kind": r.get("kind"), "regime": r.get("regime_used"),
                "t_in": r["t_in"], "t_ft": r["t_ft"], "b_d": r["b_d"], "bwd": r["bwd_in_flight"],
                "pred_raw_ms": None if r["pred_raw"] is None else round(1e3 * r["pred_raw"], 3),
                "actual_ms": None if r["actual"] is None else round(1e3 * r["actual"], 3)}

    out = []
    for i in idx[:top]:
        out.append({"step": brief(rows[i]), "ratio": round(rows[i]["actual"] / rows[i]["pred_raw"], 3),
                    "before": brief(rows[i - 1]) if i > 0 else None,
                    "after": brief(rows[i + 1]) if i + 1 < len(rows) else None})
    return out


def ttft_violations(rows: list[dict], results: list[dict], ttft_slo: float) -> list[dict]:
    """Section 7: requests over the TTFT SLO (with a send wall time) and the
    steps that finished while they waited for the first token."""
    done = sorted((r["t_done"], i) for i, r in enumerate(rows) if r["t_done"] is not None)
    times = [t for t, _ in done]
    out = []
    for q in results:
        tt, sent = q.get("ttft_s"), q.get("sent_unix")
        if tt is None or sent is None or tt <= ttft_slo:
            continue
        lo = int(np.searchsorted(times, sent))
        hi = int(np.searchsorted(times, sent + tt, side="right"))
        steps = [rows[done[j][1]] for j in range(lo, hi)]
        kinds: dict = {}
        for s in steps:
            kinds[s.get("kind")] = kinds.get(s.get("kind"), 0) + 1
        out.append({"t": q.get("t"), "ttft_s": round(tt, 4), "steps_while_waiting": len(steps),
                    "gpu_s_while_waiting": round(sum(s["actual"] or 0.0 for s in steps), 4),
                    "steps_by_kind": kinds,
                    "ft_tokens_while_waiting": int(sum(s["t_ft"] or 0 for s in steps))})
    return out


def report(rows: list[dict], results: list[dict] | None = None, ttft_slo: float = 0.5, top: int = 10,
           max_tbt_slo: float = 0.06) -> dict:
    rep = {"steps": len(rows), "accuracy": accuracy(rows), "admission": admission_fidelity(rows),
           "over_limit": over_limit(rows, max_tbt_slo), "worst_misses": worst_misses(rows, top)}
    if results is not None:
        rep["ttft_violations"] = ttft_violations(rows, results, ttft_slo)
    return rep


def compare_row(name: str, rows: list[dict], max_tbt_slo: float) -> dict:
    """One A/B arm: the margin's scores of one run's step trace."""
    acc = accuracy(rows)
    cov = [r for r in rows if r["pred"] is not None and r["actual"] is not None]
    return {"trace": name, "steps": len(rows), **over_limit(rows, max_tbt_slo),
            "margin_coverage": round(sum(r["actual"] <= r["pred"] for r in cov) / len(cov), 4) if cov else None,
            "raw_ratio_p50": acc["overall"].get("ratio_p50"), "raw_ratio_p90": acc["overall"].get("ratio_p90"),
            "ft_tokens": int(sum(r["t_ft"] or 0 for r in rows))}


def _print_text(rep: dict) -> None:
    print(f"steps: {rep['steps']}")
    acc = rep["accuracy"]
    hdr = f"{'group':<34}{'n':>7}{'mean ms':>10}{'rmse ms':>10}{'bias ms':>10}{'p50':>7}{'p90':>7}{'p99':>7}{'>1.5x':>8}{'>2x':>8}"
    for title in ("by_regime", "by_backward_in_flight", "by_kind", "by_transition"):
        print(f"\n{title} (raw model: ratio = actual / predicted)")
        print(hdr)
        for k, s in acc[title].items():
            if not s.get("n"):
                continue
            print(f"{k:<34}{s['n']:>7}{s['actual_ms_mean']:>10}{s['rmse_ms']:>10}{s['bias_ms']:>10}"
                  f"{s['ratio_p50']:>7}{s['ratio_p90']:>7}{s['ratio_p99']:>7}{s['over_1_5x']:>8}{s['over_2x']:>8}")
    print(f"\nmargin coverage (actual <= margined prediction): {acc['margin_coverage']}")
    print(f"admission fidelity: {json.dumps(rep['admission'])}")
    print(f"over the TBT limit: {json.dumps(rep['over_limit'])}")
    print("\nworst misses:")
    for m in rep["worst_misses"]:
        print(f"  x{m['ratio']}: {json.dumps(m['step'])}")
    if "ttft_violations" in rep:
        print(f"\nTTFT violations: {len(rep['ttft_violations'])}")
        for v in rep["ttft_violations"]:
            print(f"  {json.dumps(v)}")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("trace", nargs="+", help="one step trace, or several (arms of an A/B) with --compare")
    ap.add_argument("--results", default=None, help="eval.replay results (jsonl)")
    ap.add_argument("--ttft-slo", type=float, default=0.5)
    ap.add_argument("--max-tbt-slo", type=float, default=0.06)
    ap.add_argument("--compare", action="store_true",
                    help="one line per trace with the margin's scores (e.g. runs with different admission margins)")
    ap.add_argument("--top", type=int, default=10)
    ap.add_argument("--json", action="store_true", help="print the report as one JSON object")
    a = ap.parse_args(argv)
    if a.compare:
        for path in a.trace:
            print(json.dumps(compare_row(path, load_trace(path), a.max_tbt_slo)))
        return
    if len(a.trace) != 1:
        ap.error("several traces need --compare")
    rows = load_trace(a.trace[0])
    results = None
    if a.results:
        with open(a.results) as f:
            results = [json.loads(line) for line in f if line.strip()]
    rep = report(rows, results, a.ttft_slo, a.top, a.max_tbt_slo)
    if a.json:
        print(json.dumps(rep))
    else:
        _print_text(rep)


if __name__ == "__main__":
    main()
