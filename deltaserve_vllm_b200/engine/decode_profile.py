"""Decode-step cost of the serving engine alone (no finetuning), at TP = N.

    python -m deltaserve_vllm_b200.engine.decode_profile [--model llama3-8b] [--batch 16] [--prompt 512]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port 29620 -m deltaserve_vllm_b200.engine.decode_profile --batch 64

Builds the engine as ``bench.py`` does (random-init weights, one served LoRA
adapter on every request), prefills ``--batch`` prompts of ``--prompt``
tokens, then runs ``--steps`` decode-only engine iterations (CUDA graphs) and
reports, from the engine's per-iteration CUDA events (max over ranks for TP):

* ``decode_ms``: mean device time of a decode iteration;
* ``bytes_per_step``: weights read per step on this rank (every layer's
  projections, the LM head slice and the adapter factors) plus the KV cache
  read by the attention; ``frac_hbm`` = those bytes / time / the measured
  copy bandwidth (``MEASURED_PEAKS.json``, else the fallback 6.65 TB/s).

``--profile-step`` brackets one extra decode iteration with
``cudaProfilerStart/Stop``, so ``ncu --profile-from-start off`` lists exactly
that iteration's kernels.
"""

from __future__ import annotations

import argparse
import json
import os

import torch


def _peak_hbm_gbs() -> float:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--lora-rank", type=int, default=16)
    ap.add_argument("--no-lora", action="store_true", help="serve the base model only")
    ap.add_argument("--profile-step", action="store_true")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)

    from .. import dprint, ops
    from ..config import EngineConfig, FinetuneConfig
    from ..models.configs import resolve_arch
    from ..parallel.comm import init_tp
    from .llm_engine import CoServingEngine
    from .request import SamplingParams

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    comm = init_tp(timeout_s=300) if ws > 1 else None
    rank = comm.rank if comm is not None else 0
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    arch = resolve_arch(a.model)
    max_len = a.prompt + a.warmup + a.steps + 64
    ecfg = EngineConfig(model=a.model, device="cuda" if cuda else "cpu", tensor_parallel_size=ws,
                        max_model_len=max_len, block_size=64, max_num_seqs=max(256, a.batch), max_num_batched_tokens=8192, max_loras=2,
                        max_lora_rank=a.lora_rank, gpu_memory_utilization=0.85, seed=0)
    eng = CoServingEngine(ecfg, FinetuneConfig(enable_finetuning=False), comm=comm, arch=arch)
    adapter = None
    if rank == 0 and not a.no_lora:
        eng.load_inference_adapter("inf", rank=a.lora_rank, alpha=2 * a.lora_rank, seed=11)
        adapter = "inf"
    if rank != 0:
        eng.follow()
        eng.close()
        if comm is not None:
            torch.distributed.destroy_process_group()
        return
    g = torch.Generator().manual_seed(1)
    for i in range(a.batch):
        ids = torch.randint(0, arch.vocab, (a.prompt,), generator=g).tolist()
        eng.add_request(f"d{i}", ids, SamplingParams(max_tokens=max_len - a.prompt, ignore_eos=True), adapter=adapter)
    durs: list[float] = []

    def on_step(rec, dur):
        f = rec.features
        if f.t_in == 0 and f.t_ft == 0 and f.b_d == a.batch:
            durs.append(dur)

    eng.step_listeners.append(on_step)
    while any(r.first_token_time is None for r in eng.requests.values()):
        eng.step()
    for _ in range(a.warmup):
        eng.step()
    eng.synchronize()
    durs.clear()
    for _ in range(a.steps):
        eng.step()
    eng.synchronize()
    n = len(durs)
    ms = 1e3 * sum(durs) / max(1, n)
    if a.profile_step and cuda:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        eng.step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    # Bytes a decode step must read on this rank.
    tp = max(1, ws)
    per_layer = (arch.hidden * (arch.num_heads + 2 * arch.num_kv_heads) * arch.head_dim      # qkv
                 + arch.num_heads * arch.head_dim * arch.hidden                               # o
                 + arch.hidden * 2 * arch.intermediate                                        # gate_up
                 + arch.intermediate * arch.hidden) // tp                                     # down
    weights = 2 * (arch.num_layers * per_layer + arch.vocab * arch.hidden // tp)
    ctx = a.prompt + a.warmup + a.steps // 2
    kv = 2 * 2 * arch.num_layers * (arch.num_kv_heads // tp) * arch.head_dim * ctx * a.batch
    byts = weights + kv
    out = {"model": a.model, "tp": tp, "batch": a.batch, "prompt": a.prompt, "lora": not a.no_lora,
           "decode_steps_timed": n, "decode_ms": round(ms, 3), "bytes_per_step": int(byts),
           "achieved_gbs": round(byts / (ms / 1e3) / 1e9, 1) if ms > 0 else None,
           "frac_hbm": round(byts / (ms / 1e3) / 1e9 / _peak_hbm_gbs(), 3) if ms > 0 else None,
           "device_error": ops.check_device_error()}
    dprint(json.dumps(out))
    print(json.dumps(out), flush=True)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(out, f, indent=1)
    eng.close()
    if comm is not None:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
