"""Finetuning-only throughput: the engine with no inference load.

    python -m deltaserve_vllm_b200.eval.pure_ft --model llama3-8b --seq 512 --batch 8 --cycles 20

Every step is an FT-only forward (the samples' activations captured) and
every full buffer a backward cycle; the number reported is trained tokens per
second over the timed cycles (after ``--warmup`` cycles), with the split of
wall time between forward steps and backward cycles. This is the ceiling the
co-served FT throughput is measured against (the reference's
``eval/pure_ft_bench.py``).
"""

from __future__ import annotations

import argparse
import json
import time


def run(model: str, seq: int, batch: int, cycles: int, warmup: int = 2, device: str | None = None,
        rank: int = 16, graphs: bool = True, seed: int = 0) -> dict:
    import torch

    from ..config import EngineConfig, FinetuneConfig
    from ..engine.ft.store import FinetuningStore
    from ..engine.llm_engine import CoServingEngine
    from ..models.configs import resolve_arch

    arch = resolve_arch(model)
    cap = seq * batch
    n_samples = batch * (cycles + warmup + 1)
    ecfg = EngineConfig(model=model, device=device, max_model_len=max(2 * seq, 1024), block_size=64,
                        max_num_batched_tokens=max(cap, 2048), max_loras=2, max_lora_rank=rank, seed=seed)
    fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=cap, learning_rate=1e-4,
                          backward_cuda_graph=graphs, profile_on_launch=False)
    store = FinetuningStore.synthetic(arch.vocab, n_samples, seq, seq, seed=seed, max_saved_finetuning_tokens=cap)
    eng = CoServingEngine(ecfg, fcfg, ft_store=store)
    cuda = eng.cuda

    def sync():
        if cuda:
            torch.cuda.synchronize(eng.device)

    def cycles_done():
        return eng.coord.completed_cycles

    fwd_s = [0.0]

    def step():
        t0 = time.perf_counter()
        eng.step()
        fwd_s[0] += time.perf_counter() - t0

    while cycles_done() < warmup:
        step()
    sync()
    tok0, c0 = eng.stats["ft_tokens_trained"], cycles_done()
    fwd_s[0] = 0.0
    t0 = time.perf_counter()
    while cycles_done() < c0 + cycles:
        step()
    eng._drain_backward()
    sync()
    wall = time.perf_counter() - t0
    toks = eng.stats["ft_tokens_trained"] - tok0
    eng.close()
    return {"metric": "pure FT tokens/s", "model": model, "seq": seq, "batch": batch,
            "cycles": cycles_done() - c0, "ft_tokens": int(toks), "wall_s": round(wall, 4),
            "ft_tok_s": round(toks / wall, 2) if wall > 0 else None,
            "step_loop_s": round(fwd_s[0], 4), "device": str(eng.device)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--cycles", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--rank", type=int, default=16)
    ap.add_argument("--device", default=None)
    ap.add_argument("--no-graphs", action="store_true")
    a = ap.parse_args(argv)
    print(json.dumps(run(a.model, a.seq, a.batch, a.cycles, a.warmup, a.device, a.rank, not a.no_graphs)))


if __name__ == "__main__":
    main()
