"""Prefill time on an otherwise idle server: TTFT against prompt length.

    python -m deltaserve_vllm_b200.eval.prefill_probe --server http://127.0.0.1:8000 \\
        [--lengths 2048,4096,8192] [--reps 4] [--conc 4 --conc-len 8192] [--vocab 128256] [--out probe.jsonl]

Phase 1 sends ``--reps`` streaming requests per length one after another
(``--gap`` idle seconds between them); with nothing else running, the time to
the first token is the prefill time, reported per length as the median TTFT
and milliseconds per prompt token. Phase 2 (``--conc`` > 0) sends that many
requests of ``--conc-len`` tokens at once and reports each TTFT and the
aggregate prefill rate. Every prompt is a distinct random token sequence, so
prefix caching never hits. The reference's probe does the same with real
articles (``eval-arxiv/prefill_bench.py``); token ids need no tokenizer here.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import random
import statistics
import time

import aiohttp

from .replay import _one


def _prompt(rng: random.Random, n: int, vocab: int, serial: int) -> list[int]:
    ids = [rng.randrange(vocab) for _ in range(n)]
    ids[0] = serial % vocab               # distinct first token per request: no shared prefix page
    return ids


async def probe(server: str, lengths: list[int], reps: int = 4, gap: float = 0.0, conc: int = 0,
                conc_len: int = 8192, vocab: int = 32000, max_tokens: int = 4, seed: int = 0,
                model: str | None = None) -> dict:
    rng = random.Random(seed)
    serial = 0
    rows: list[dict] = []
    timeout = aiohttp.ClientTimeout(total=None)
    async with aiohttp.ClientSession(timeout=timeout) as s:
        for n in lengths:
            for r in range(reps):
                serial += 1
                rec = {"t": 0.0, "prompt": _prompt(rng, n, vocab, serial), "max_tokens": max_tokens}
                res = await _one(s, server, rec, model, time.perf_counter(), 1.0)
                rows.append({"phase": "sequential", "len": n, "rep": r, "ttft_s": res.get("ttft_s"),
                             "error": res.get("error")})
                if gap > 0:
                    await asyncio.sleep(gap)
        if conc > 0:
            recs = []
            for _ in range(conc):
                serial += 1
                recs.append({"t": 0.0, "prompt": _prompt(rng, conc_len, vocab, serial), "max_tokens": max_tokens})
            t0 = time.perf_counter()
            res = await asyncio.gather(*[_one(s, server, rec, model, t0, 1.0) for rec in recs])
            for i, q in enumerate(res):
                rows.append({"phase": "concurrent", "len": conc_len, "rep": i, "ttft_s": q.get("ttft_s"),
                             "error": q.get("error")})
    summary: dict = {"sequential": {}, "concurrent": None}
    for n in lengths:
        tt = [r["ttft_s"] for r in rows if r["phase"] == "sequential" and r["len"] == n and r["ttft_s"] is not None]
        if tt:
            med = statistics.median(tt)
            summary["sequential"][str(n)] = {"n": len(tt), "ttft_p50_s": round(med, 4),
                                             "ttft_min_s": round(min(tt), 4),
                                             "ms_per_token": round(1e3 * med / n, 4),
                                             "prefill_tok_s": round(n / med, 1)}
    ct = [r["ttft_s"] for r in rows if r["phase"] == "concurrent" and r["ttft_s"] is not None]
    if ct:
        summary["concurrent"] = {"n": len(ct), "len": conc_len, "ttft_max_s": round(max(ct), 4),
                                 "ttft_p50_s": round(statistics.median(ct), 4),
                                 "aggregate_prefill_tok_s": round(len(ct) * conc_len / max(ct), 1)}
    summary["errors"] = sum(1 for r in rows if r["error"])
    return {"summary": summary, "rows": rows}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--server", default="http://127.0.0.1:8000")
    ap.add_argument("--lengths", default="2048,4096,8192")
    ap.add_argument("--reps", type=int, default=4)
    ap.add_argument("--gap", type=float, default=0.0)
    ap.add_argument("--conc", type=int, default=4)
    ap.add_argument("--conc-len", type=int, default=8192)
    ap.add_argument("--vocab", type=int, default=32000, help="token ids are drawn below this")
    ap.add_argument("--max-tokens", type=int, default=4)
    ap.add_argument("--model", default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--out", default=None, help="per-request rows (jsonl)")
    a = ap.parse_args(argv)
    lengths = [int(x) for x in a.lengths.split(",") if x]
    out = asyncio.run(probe(a.server.rstrip("/"), lengths, a.reps, a.gap, a.conc, a.conc_len, a.vocab,
                            a.max_tokens, a.seed, a.model))
    if a.out:
        with open(a.out, "w") as f:
            for r in out["rows"]:
                f.write(json.dumps(r) + "\n")
    print(json.dumps(out["summary"]))


if __name__ == "__main__":
    main()
