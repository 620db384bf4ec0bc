"""Synthetic inference traces (JSONL, one request per line).

    python -m deltaserve_vllm_b200.eval.trace --rate 8 --duration 120 \\
        --prompt-median 512 --prompt-min 32 --prompt-max 4096 --out-min 32 --out-max 256 > trace.jsonl

Poisson arrivals at ``rate`` req/s; prompt lengths lognormal (median, sigma)
clipped to [min, max]; output lengths uniform; token ids uniform over the
vocabulary (the headline benchmark's shapes). ``--adapters`` spreads requests
over named adapters (or ``auto`` for routing).
"""

from __future__ import annotations

import argparse
import json
import sys

import numpy as np


def make_trace(rate: float, duration_s: float, vocab: int, seed: int = 0, prompt_median: int = 512,
               prompt_sigma: float = 0.8, prompt_min: int = 32, prompt_max: int = 4096, out_min: int = 32,
               out_max: int = 256, adapters: list[str] | None = None) -> list[dict]:
    rng = np.random.default_rng(seed)
    t, out = 0.0, []
    while True:
        t += rng.exponential(1.0 / rate)
        if t > duration_s:
            break
        n = int(np.clip(rng.lognormal(np.log(prompt_median), prompt_sigma), prompt_min, prompt_max))
        rec = {"t": round(t, 6), "prompt": rng.integers(3, vocab, size=n).tolist(),
               "max_tokens": int(rng.integers(out_min, out_max + 1))}
        if adapters:
            rec["model"] = adapters[int(rng.integers(0, len(adapters)))]
        out.append(rec)
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--duration", type=float, default=120.0)
    ap.add_argument("--vocab", type=int, default=128256)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--prompt-median", type=int, default=512)
    ap.add_argument("--prompt-sigma", type=float, default=0.8)
    ap.add_argument("--prompt-min", type=int, default=32)
    ap.add_argument("--prompt-max", type=int, default=4096)
    ap.add_argument("--out-min", type=int, default=32)
    ap.add_argument("--out-max", type=int, default=256)
    ap.add_argument("--adapters", default=None, help="comma-separated model names to spread over")
    a = ap.parse_args(argv)
    tr = make_trace(a.rate, a.duration, a.vocab, a.seed, a.prompt_median, a.prompt_sigma, a.prompt_min,
                    a.prompt_max, a.out_min, a.out_max, a.adapters.split(",") if a.adapters else None)
    for r in tr:
        sys.stdout.write(json.dumps(r) + "\n")


if __name__ == "__main__":
    main()
