"""Replay a trace against a running server and measure every request.

    python -m deltaserve_vllm_b200.eval.replay --server http://127.0.0.1:8000 \\
        --trace trace.jsonl --out results.jsonl [--model llama3-8b] [--speed 1.0]

Each request is sent at its trace time (scaled by ``--speed``) as a streaming
``POST /v1/completions`` (token-id prompt, ``ignore_eos``); the client records
TTFT (first streamed chunk) and the gaps between chunks (TBT), plus the
routing headers when present. One JSON line per request goes to ``--out``;
a summary (percentiles, SLO attainment, finetuning progress read from
``/finetuning_status`` before and after) is printed at the end.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import time

import aiohttp

from .report import summarize


async def _one(session, url: str, rec: dict, model: str | None, t0: float, speed: float) -> dict:
    await asyncio.sleep(max(0.0, t0 + rec["t"] / speed - time.perf_counter()))
    body = {"prompt": rec["prompt"], "max_tokens": rec["max_tokens"], "stream": True, "ignore_eos": True,
            "temperature": 0.0}
    if rec.get("model") or model:
        body["model"] = rec.get("model") or model
    sent = time.perf_counter()
    sent_unix = time.time()        # joins the engine's step trace (wall clock)
    first, last, gaps, n = None, None, [], 0
    headers = {}
    status = 0
    try:
        async with session.post(url + "/v1/completions", json=body) as r:
            status = r.status
            headers = {k: v for k, v in r.headers.items() if k.lower().startswith("x-deltaserve")}
            async for raw in r.content:
                line = raw.decode().strip()
                if not line.startswith("data: ") or line == "data: [DONE]":
                    continue
                chunk = json.loads(line[6:])
                toks = chunk["choices"][0].get("token_ids") or []
                if not toks:
                    continue
                now = time.perf_counter()
                if first is None:
                    first = now
                else:
                    gaps.append((now - last) / len(toks))
                last = now
                n += len(toks)
    except Exception as e:  # recorded, not raised: one failure must not stop the replay
        return {"t": rec["t"], "error": repr(e), "status": status}
    return {"t": rec["t"], "status": status, "prompt_tokens": len(rec["prompt"]), "output_tokens": n,
            "ttft_s": None if first is None else first - sent,
            "tbt_mean_s": sum(gaps) / len(gaps) if gaps else None, "tbt_max_s": max(gaps) if gaps else None,
            "headers": headers, "sent_unix": sent_unix}


async def replay(server: str, trace: list[dict], model: str | None = None, speed: float = 1.0) -> list[dict]:
    timeout = aiohttp.ClientTimeout(total=None)
    async with aiohttp.ClientSession(timeout=timeout) as s:
        t0 = time.perf_counter()
        return await asyncio.gather(*[_one(s, server, r, model, t0, speed) for r in trace])


def _status(server: str) -> dict:
    import urllib.request
    try:
        with urllib.request.urlopen(server + "/finetuning_status", timeout=10) as r:
            return json.loads(r.read().decode())
    except Exception:
        return {}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--server", default="http://127.0.0.1:8000")
    ap.add_argument("--trace", required=True)
    ap.add_argument("--out", default=None)
    ap.add_argument("--model", default=None)
    ap.add_argument("--speed", type=float, default=1.0)
    ap.add_argument("--ttft-slo", type=float, default=0.5)
    ap.add_argument("--tbt-slo", type=float, default=0.06)
    a = ap.parse_args(argv)
    with open(a.trace) as f:
        trace = [json.loads(ln) for ln in f if ln.strip()]
    before = _status(a.server)
    t0 = time.time()
    res = asyncio.run(replay(a.server.rstrip("/"), trace, a.model, a.speed))
    wall = time.time() - t0
    after = _status(a.server)
    if a.out:
        with open(a.out, "w") as f:
            for r in res:
                f.write(json.dumps(r) + "\n")
    s = summarize(res, a.ttft_slo, a.tbt_slo)
    s["wall_s"] = round(wall, 3)
    ft0 = (before.get("total_trained_tokens") or 0)
    ft1 = (after.get("total_trained_tokens") or 0)
    s["ft_tokens_trained"] = ft1 - ft0
    s["ft_tok_s"] = round((ft1 - ft0) / wall, 1) if wall > 0 else None
    print(json.dumps(s))


if __name__ == "__main__":
    main()
