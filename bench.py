#!/usr/bin/env python
"""Headline benchmark: co-served finetuning tokens/s at >= 99 % SLO attainment,
with p99 TTFT / TBT, Llama-3-8B architecture (random init, bf16) at TP=N.

Trace (the Llama-3-8B co-serving configuration): Poisson arrivals at 8 req/s
per GPU; prompt lengths lognormal (median 512, clipped to 32..4096); output
lengths uniform 32..256; uniform-random token ids; every inference request
uses an r=16 inference LoRA. Finetuning stream: uniform-random 512-token
sequences, 8 per backward cycle, AdamW, trainable r=16 / alpha=32 LoRA on all
seven projections. SLOs: TTFT 500 ms, TBT 60 ms.

A bench *step* is one second of serving (``--step-s``): every engine
iteration that runs while one second of the arrival trace is served. The
metric is a rate over a trace, so the window has to hold many requests and
many backward cycles to mean anything (at 8 req/s per GPU a 20-step window
holds about 160 x N requests).

Timing: W warm-up steps, then EXACTLY K steps bracketed by a device-wide
synchronize + stamp on every rank (the stamps travel in the rank-0 step plan,
so every rank stamps at the same point); device time of the region is the
max over ranks. ``value`` = FT tokens forwarded-and-captured for training in
the region / region seconds (each captured token is trained in the next
backward cycle; the tokens whose backward finished inside the region are
reported next to it as ``ft_tokens_trained``). ``valid_slo`` is true only
when attainment is >= 99 % over at least 100 requests and at least 3
backward cycles completed inside the region. The e2e number is the same
count over the wall clock of the region measured around the public
``CoServingEngine.step()`` calls, which copy every step's inputs
host->device (pinned) and read sampled tokens back.

``--impl reference`` runs the reference plugin (vLLM + DeltaServe) when it can
run here, else prints an ``unavailable`` line.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W]; for N > 1 launch
under torchrun (one rank per GPU).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_VALUE = None  # the reference publishes no number for this metric on this config
METRIC = "co-served FT tokens/s at ≥99% SLO attainment; p99 TTFT & TBT (Llama-3-8B TP8)"


# Workload presets (``--config``): model, trace, finetuning stream, SLOs, LoRA
# rank. ``llama3-8b`` is the headline configuration; the others run the same
# harness on the other model families of the benchmark plan.
CONFIGS = {
    "llama3-8b": dict(model="llama3-8b", rate_per_gpu=8.0, prompt_median=512, prompt_min=32,
                      prompt_max=4096, out_min=32, out_max=256, ft_min=512, ft_max=512, ft_batch=8,
                      ttft_slo=0.5, tbt_slo=0.06, lora_rank=16, max_model_len=4096 + 512),
    # Qwen3-0.6B on one GPU: 20 req/s, prompts median 256 (16..2048), outputs
    # 16..256, FT sequences of 128..512 tokens, SLOs 200 ms / 50 ms.
    "qwen3-0.6b": dict(model="qwen3-0.6b", rate_per_gpu=20.0, prompt_median=256, prompt_min=16,
                       prompt_max=2048, out_min=16, out_max=256, ft_min=128, ft_max=512, ft_batch=8,
                       ttft_slo=0.2, tbt_slo=0.05, lora_rank=16, max_model_len=2048 + 256),
    # Qwen3-14B at TP=2/4/8, LoRA r=32, the Llama-3-8B trace shapes.
    "qwen3-14b": dict(model="qwen3-14b", rate_per_gpu=8.0, prompt_median=512, prompt_min=32,
                      prompt_max=4096, out_min=32, out_max=256, ft_min=512, ft_max=512, ft_batch=8,
                      ttft_slo=0.5, tbt_slo=0.06, lora_rank=32, max_model_len=4096 + 512),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--config", default="llama3-8b", choices=sorted(CONFIGS),
                   help="workload preset (model, trace, FT stream, SLOs, LoRA rank)")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--step-s", type=float, default=1.0, help="seconds of serving per bench step")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--rate-per-gpu", type=float, default=None, help="override the preset's arrival rate")
    p.add_argument("--max-batched-tokens", type=int, default=8192)
    p.add_argument("--profile-repeats", type=int, default=1)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--tp-comm", default="fused", choices=["nccl", "fused"],
                   help="row-parallel all-reduce: fused GEMM+all-reduce kernel over NVLink peer memory "
                        "(falls back to NCCL if its start-up self-test fails) or plain NCCL")
    p.add_argument("--run-ahead", type=int, default=6, help="backward layers queued ahead of the GPU")
    p.add_argument("--bwd-sm-pct", type=int, default=0,
                   help="backward_mps_percentage: cap the backward GEMMs at this share of the SMs (0 = no cap)")
    p.add_argument("--fwd-small-gemm-ctas", type=int, default=0,
                   help="grid cap of the forward GEMMs of batches <= 128 rows (decode): they are "
                        "HBM-bound, fewer SMs keep the pace and leave the rest to the backward (0 = all)")
    p.add_argument("--pause", default="arrival", choices=["arrival", "off"],
                   help="pause_on_arrival: stop feeding the backward while an inference prefill is pending")
    p.add_argument("--phase", default="both", choices=["prefill", "both"],
                   help="coserving_admission_phase (both: FT may ride decode-only steps too)")
    a = p.parse_args()
    for k, v in CONFIGS[a.config].items():
        if getattr(a, k, None) is None:
            setattr(a, k, v)
    a.ft_seq = a.ft_max
    return a


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: str):
        self.rows: list[list[str]] = []
        self._stop = threading.Event()
        self._gpus = gpus
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                      "-i", self._gpus], capture_output=True, text=True, timeout=5).stdout
                for line in out.strip().splitlines():
                    self.rows.append([c.strip() for c in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=6)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def make_trace(rate: float, duration_s: float, vocab: int, seed: int, args):
    """Poisson arrivals; lognormal prompt lengths (sigma 0.8) clipped to the
    preset's range; uniform output lengths; uniform-random token ids."""
    rng = np.random.default_rng(seed)
    t, out = 0.0, []
    while t < duration_s:
        t += rng.exponential(1.0 / rate)
        plen = int(np.clip(np.round(rng.lognormal(np.log(args.prompt_median), 0.8)), args.prompt_min,
                           args.prompt_max))
        olen = int(rng.integers(args.out_min, args.out_max + 1))
        out.append((t, rng.integers(0, vocab, size=plen).tolist(), olen))
    return out


def percentile(x, q):
    return float(np.percentile(np.asarray(x), q)) if len(x) else None


def reference_arm(args) -> None:
    line = {"impl": "reference", "metric": METRIC, "n_gpus": args.gpus}
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    try:
        sys.path.insert(0, ref_dir)
        import deltaserve  # noqa: F401
        import vllm
        ver = vllm.__version__
    except Exception as e:
        print(json.dumps({"impl": "reference", "unavailable": f"reference plugin not importable: {e!r}"}))
        return
    if not ver.startswith("0.33"):
        print(json.dumps({"impl": "reference", "unavailable":
                          f"reference targets vLLM 0.33.0; only vLLM {ver} is installed here and no "
                          f"0.33 wheel exists offline (plugin installed with --no-deps)"}))
        return
    print(json.dumps(line))


def _exit_watchdog(seconds: float = 90.0) -> None:
    """The result line is out: if tearing down (graphs, peer mappings, process
    group) takes longer than ``seconds``, dump every thread's stack and exit
    with status 3, so a teardown hang shows up as a failed run."""
    import faulthandler
    import threading

    def fire():
        sys.stderr.write(f"bench: teardown still running after {seconds:.0f} s; exiting with status 3\n")
        faulthandler.dump_traceback(all_threads=True)
        sys.stderr.flush()
        os._exit(3)
    t = threading.Timer(seconds, fire)
    t.daemon = True
    t.start()


def main():
    args = parse()
    if args.fwd_small_gemm_ctas:
        os.environ["DSV_FWD_SMALL_GEMM_CTAS"] = str(args.fwd_small_gemm_ctas)   # read at package import
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            reference_arm(args)
        return
    import torch
    from deltaserve_vllm_b200 import dprint, ops
    from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
    from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
    from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
    from deltaserve_vllm_b200.engine.request import SamplingParams
    from deltaserve_vllm_b200.models.configs import resolve_arch
    from deltaserve_vllm_b200.parallel.comm import init_tp

    dump_s = float(os.environ.get("DSV_BENCH_STACKDUMP_S", "0"))
    if dump_s > 0:  # diagnostics: dump every thread's stack if still running then
        import faulthandler
        faulthandler.dump_traceback_later(dump_s, repeat=False)
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ws}; launch N>1 under torchrun")
    comm = init_tp(timeout_s=300) if ws > 1 else None
    rank = comm.rank if comm is not None else 0
    if not torch.cuda.is_available() or not ops.native_available():
        raise SystemExit("bench needs a B200 and the built extension")
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    arch = resolve_arch(args.model)
    cap = args.ft_seq * args.ft_batch
    ecfg = EngineConfig(model=args.model, tensor_parallel_size=args.gpus, max_model_len=args.max_model_len,
                        block_size=64, max_num_seqs=256, max_num_batched_tokens=args.max_batched_tokens,
                        max_loras=2, max_lora_rank=args.lora_rank, gpu_memory_utilization=0.85, seed=args.seed,
                        tp_comm=args.tp_comm)
    fcfg = FinetuneConfig(enable_finetuning=True, backward_cuda_graph=True, max_saved_finetuning_tokens=cap, learning_rate=1e-4,
                          num_epochs=1000, ttft_slo=args.ttft_slo, max_tbt_slo=args.tbt_slo,
                          avg_tbt_slo=args.tbt_slo, admission_margin="relative", admission_margin_k=1.5,
                          pause_on_arrival=args.pause == "arrival", backward_mps_percentage=args.bwd_sm_pct,
                          backward_run_ahead_boundaries=args.run_ahead,
                          coserving_admission_phase=args.phase,
                          profile_num_repeats=args.profile_repeats)
    store = FinetuningStore.synthetic(arch.vocab, 512, args.ft_min, args.ft_max, seed=args.seed + 7,
                                      max_saved_finetuning_tokens=cap, total_epochs=1000)
    t0 = time.perf_counter()
    eng = CoServingEngine(ecfg, fcfg, comm=comm, arch=arch, ft_store=store)
    if rank == 0:   # replayed on the other ranks
        eng.load_inference_adapter("inf", rank=args.lora_rank, alpha=2 * args.lora_rank, seed=11)
    if rank != 0:
        eng.follow()
        _exit_watchdog()
        eng.close()
        if comm is not None:
            torch.distributed.destroy_process_group()
        return
    dprint(f"engine up in {time.perf_counter() - t0:.1f}s; KV blocks {eng.kv.num_blocks}")
    eng.profile_execution_model(repeats=args.profile_repeats)
    dprint(f"profiling done at {time.perf_counter() - t0:.1f}s; estimator ready={eng.estimator.is_ready}")
    rate = args.rate_per_gpu * args.gpus
    trace = make_trace(rate, 3600.0, arch.vocab, args.seed, args)
    ti = 0
    clock0 = time.perf_counter()

    def ingest():
        nonlocal ti
        now = time.perf_counter() - clock0
        while ti < len(trace) and trace[ti][0] <= now:
            t_arr, ids, olen = trace[ti]
            eng.add_request(f"q{ti}", ids, SamplingParams(max_tokens=olen), adapter="inf",
                            arrival_time=clock0 + t_arr)
            ti += 1

    verbose = os.environ.get("DSV_BENCH_VERBOSE") == "1"

    def bench_step() -> int:
        """Serve ``--step-s`` seconds of the trace; returns engine iterations."""
        t_end = time.perf_counter() + args.step_s
        k = 0
        while time.perf_counter() < t_end:
            ingest()
            eng.step()
            k += 1
        return k

    for i in range(args.warmup):
        k = bench_step()
        if verbose:
            dprint(f"warmup step {i}: {k} iterations, {eng.coord.status()['cycle']} cycles, "
                   f"bwd_active={eng.bwd_active}")
    eng.synchronize()
    stats0 = dict(eng.stats)
    host0 = dict(eng.host_s)
    l0 = ops.LAUNCHES[0]
    cyc0 = len(eng.coord.history)
    trk0 = eng.tracker.appended
    iters = 0
    gpu_idx = os.environ.get("CUDA_VISIBLE_DEVICES", ",".join(str(i) for i in range(args.gpus)))
    with ClockSampler(gpu_idx) as clocks:
        eng.mark("t0")
        w0 = time.perf_counter()
        for _ in range(args.steps):
            iters += bench_step()
        w1 = time.perf_counter()
        eng.mark("t1")
    regions = eng.gather_region("t0", "t1")
    launches = ops.LAUNCHES[0] - l0
    dev_ms = max(r[0] for r in regions)
    wall_ms = (w1 - w0) * 1e3
    st = {k: eng.stats.get(k, 0) - stats0.get(k, 0) for k in eng.stats}
    # requests that arrived inside the timed region
    t_lo, t_hi = w0, w1
    reqs = [r for r in list(eng.finished) + list(eng.requests.values())
            if t_lo <= r.arrival_time <= t_hi and not r.request_id.startswith("__")]
    ttfts = [r.ttft() for r in reqs if r.ttft() is not None]
    tbts = [g for r in reqs for g in r.tbts()]
    ok = 0
    counted = 0
    for r in reqs:
        tt = r.ttft()
        if tt is None:
            if t_hi - r.arrival_time > args.ttft_slo:
                counted += 1  # waited past the SLO without a token: violation
            continue
        counted += 1
        g = r.tbts()
        if tt <= args.ttft_slo and (not g or float(np.mean(g)) <= args.tbt_slo):
            ok += 1
    attain = ok / counted if counted else None
    value = st["ft_tokens_forwarded"] / (dev_ms / 1e3)
    e2e = st["ft_tokens_forwarded"] / (wall_ms / 1e3)
    cs = clocks.summary()
    # Decode-only steps: host time to enqueue the forward vs its GPU time
    # (launch-bound when the first is larger).
    eng._drain_timing(block=True)
    n_new = min(eng.tracker.appended - trk0, eng.tracker.size())
    feats = eng.tracker.features[-n_new:] if n_new else []
    durs = eng.tracker.durations[-n_new:].tolist() if n_new else []
    dec_gpu = [d for f, d in zip(feats, durs) if f.t_in == 0 and f.t_ft == 0 and f.b_d > 0]
    n_dec = st.get("decode_steps", 0)
    dec_info = {"host_enqueue_ms": round(1e3 * st.get("decode_enqueue_s", 0.0) / max(1, n_dec), 3),
                "gpu_ms": round(1e3 * float(np.mean(dec_gpu)), 3) if dec_gpu else None,
                "steps": n_dec}
    # Engine iterations of the region by kind: count and mean GPU time.
    kinds: dict = {}
    for f, d in zip(feats, durs):
        k = ("ft_only" if f.t_ft > 0 and f.t_in == 0 and f.b_d == 0 else
             "mixed_ft" if f.t_ft > 0 else "prefill" if f.t_in > 0 else "decode")
        kinds.setdefault(k, []).append(d)
    step_kinds = {k: {"n": len(v), "gpu_ms_mean": round(1e3 * float(np.mean(v)), 3),
                      "gpu_ms_sum": round(1e3 * float(np.sum(v)), 1)} for k, v in kinds.items()}
    # Backward cycles completed in the region: fill (admission reopened ->
    # buffer full) and backward (trigger -> trained and published) wall time.
    hist = eng.coord.history[cyc0:]
    cyc = {"completed": len(hist),
           "bwd_gpu_ms_mean": round(float(np.mean([h["gpu_ms"] for h in hist])), 2) if hist else None,
           "bwd_wall_ms_mean": round(float(np.mean([h["wall_ms"] for h in hist])), 2) if hist else None,
           "fill_wall_ms_mean": (round(float(np.mean([h["fill_ms"] for h in hist if h.get("fill_ms")])), 2)
                                 if any(h.get("fill_ms") for h in hist) else None)}
    enough = len(reqs) >= 100 and len(hist) >= 3
    line = {
        "metric": (METRIC if args.config == "llama3-8b" else
                   f"co-served FT tokens/s at ≥99% SLO attainment; p99 TTFT & TBT ({args.model})"),
        "value": round(value, 2), "unit": "FT tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (round(value / BASELINE_VALUE, 3) if BASELINE_VALUE else None),
        "dtype": "bf16", "data": "synthetic (random-init weights, uniform-random token ids)",
        "config": {"model": args.model, "global_batch": args.ft_batch, "seq_len": args.ft_seq,
                   "parallelism": f"tp{args.gpus}", "rate_req_s": rate, "preset": args.config,
                   "step": f"{args.step_s:g} s of serving (all engine iterations in it)",
                   "prompts": f"lognormal(median {args.prompt_median}, sigma 0.8) clip "
                              f"{args.prompt_min}..{args.prompt_max}",
                   "outputs": f"uniform {args.out_min}..{args.out_max}",
                   "ft_seq": f"uniform {args.ft_min}..{args.ft_max}", "lora_rank": args.lora_rank,
                   "slo": {"ttft_s": args.ttft_slo, "tbt_s": args.tbt_slo},
                   "l2": "inputs larger than L2 (16 GB of weights stream every step)",
                   "tp_comm": args.tp_comm, "admission_phase": args.phase, "pause": args.pause,
                   "bwd_sm_pct": args.bwd_sm_pct, "fwd_small_gemm_ctas": args.fwd_small_gemm_ctas,
                   "run_ahead_layers": args.run_ahead},
        "fused_ar_active": eng.peer_ws is not None,
        "slo_attainment": attain, "p99_ttft_ms": (percentile(ttfts, 99) or 0) * 1e3 if ttfts else None,
        "p99_tbt_ms": (percentile(tbts, 99) or 0) * 1e3 if tbts else None,
        "p50_ttft_ms": (percentile(ttfts, 50) or 0) * 1e3 if ttfts else None,
        "requests_in_region": len(reqs), "ft_tokens": st["ft_tokens_forwarded"],
        "ft_tokens_trained": st["ft_tokens_trained"],
        "ft_tokens_trained_per_s": round(st["ft_tokens_trained"] / (dev_ms / 1e3), 2),
        "backward_cycles_total": eng.coord.completed_cycles, "backward_cycles": cyc,
        "engine_iterations": iters, "iteration_kinds": step_kinds,
        "host_ms_per_iteration": {k: round(1e3 * (v - host0.get(k, 0.0)) / max(1, iters), 3)
                                  for k, v in sorted(eng.host_s.items())},
        # followers (ranks 1..N-1), whole run: seconds waiting for / replaying step plans
        "follower_host_s_max": ({k: round(max(f.get(k, 0.0) for f in eng.follower_host_s), 2)
                                 for k in ("follower_wait_plan", "follower_replay")}
                                if getattr(eng, "follower_host_s", None) else None),
        "last_loss": eng.coord.last_loss,
        "valid_slo": bool(attain is not None and attain >= 0.99 and enough),
        "e2e": {"value": round(e2e, 2), "unit": "FT tokens/s (wall clock, public step() API)",
                "h2d_bytes_per_step": int(st["h2d_bytes"] / max(1, args.steps)),
                "d2h_bytes_per_step": int(st["d2h_bytes"] / max(1, args.steps))},
        "gpu_launches": int(launches), "clocks": cs, "device_ms_per_rank": [round(r[0], 2) for r in regions],
        "decode_steps": dec_info,
    }
    eng.shutdown()
    print(json.dumps(line), flush=True)
    _exit_watchdog()
    eng.close()
    if comm is not None:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
