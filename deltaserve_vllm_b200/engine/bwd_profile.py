"""Where a backward cycle's time goes, per phase and per collective, at TP = N.

    python -m deltaserve_vllm_b200.engine.bwd_profile [--model llama3-8b] [--seqs 8] [--seq-len 512]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port 29610 -m deltaserve_vllm_b200.engine.bwd_profile --out bwd_tpN.json

Builds the trainer exactly as the engine does (random-init base weights at this
TP degree, the served LoRA slot of the trained adapter, the backward's own
communicator) over a capture buffer filled with synthetic activations of the
FT batch shape, then measures, every number the max over ranks:

* ``graph_cycle_ms``: a whole cycle on the production path (per-layer CUDA
  graphs), CUDA events on the launching stream, mean of ``--cycles``;
* ``phases``: the same cycle run eagerly with a CUDA event at every phase
  boundary of the head and of each layer (summed over layers). A spin kernel
  (``torch.cuda._sleep``) is queued first so the host has enqueued the whole
  cycle before the GPU reaches it: the phase times are device time, not host
  launch gaps;
* ``collectives``: each collective of the cycle timed on its own at the
  cycle's sizes (the two per-layer residual-gradient all-reduces and the
  bucketed factor-gradient all-reduce), plus the same all-reduce in bf16.

Rank 0 prints one JSON object; ``--out`` also writes it to a file.
"""

from __future__ import annotations

import argparse
import json
import os
import time
from collections import defaultdict

import torch


class PhaseTimer:
    """CUDA events at phase boundaries on the current stream; a phase's time
    is the gap between its closing event and the previous one."""

    def __init__(self):
        self.marks: list[tuple[str, torch.cuda.Event]] = []
        self.comms: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    def start(self) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.marks.append(("<start>", ev))

    def mark(self, name: str) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.marks.append((name, ev))

    def comm(self, name: str, ev0, ev1) -> None:
        self.comms.append((name, ev0, ev1))

    def totals(self) -> tuple[dict, dict]:
        torch.cuda.synchronize()
        ph: dict = defaultdict(float)
        for (_, e0), (name, e1) in zip(self.marks, self.marks[1:]):
            ph[name] += e0.elapsed_time(e1)
        cm: dict = defaultdict(lambda: [0, 0.0])
        for name, e0, e1 in self.comms:
            cm[name][0] += 1
            cm[name][1] += e0.elapsed_time(e1)
        return dict(ph), {k: {"calls": v[0], "ms": v[1]} for k, v in cm.items()}


def _fill_capture(cap, n: int, vocab: int, seed: int) -> None:
    g = torch.Generator(device=cap.layer_in.device).manual_seed(seed)
    for t in (cap.layer_in, cap.qkv, cap.ctx, cap.resid_mid, cap.gate_up, cap.act):
        if t is not None:
            t[:, :n].copy_(torch.randn(t[:, :n].shape, generator=g, device=t.device).to(t.dtype))
    cap.final_in[:n].copy_(torch.randn(cap.final_in[:n].shape, generator=g, device=cap.final_in.device))
    cap.ids[:n].copy_(torch.randint(0, vocab, (n,), generator=g, device=cap.ids.device))


def _max_over_ranks(comm, d):
    if comm is None or comm.size == 1:
        return d
    allv = comm.all_gather_object(d)

    def merge(vals):
        if isinstance(vals[0], dict):
            keys = set().union(*[v.keys() for v in vals])
            return {k: merge([v.get(k, 0.0) for v in vals]) for k in keys}
        if isinstance(vals[0], (int, float)):
            return max(vals)
        return vals[0]
    return merge(allv)


def _time_collective(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--seq-len", type=int, default=512)
    ap.add_argument("--rank", type=int, default=16, help="LoRA rank of the trained adapter")
    ap.add_argument("--cycles", type=int, default=3)
    ap.add_argument("--tp-comm", default="fused", choices=["fused", "nccl"],
                    help="residual-gradient reductions over peer memory (fused) or NCCL all-reduces")
    ap.add_argument("--out", default="")
    ap.add_argument("--profile-cycle", action="store_true",
                    help="bracket one extra graph cycle with cudaProfilerStart/Stop (for "
                         "`ncu --profile-from-start off` launch lists); skips the eager phase runs; one GPU only")
    args = ap.parse_args()
    if args.profile_cycle and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--profile-cycle profiles one GPU; run it without torchrun")

    import torch.distributed as dist

    from .. import dprint, ops
    from ..models.configs import resolve_arch
    from ..models.decoder import CaptureBuffers
    from ..models.lora import LoraServeBuffers
    from ..ops.reference import rope_cos_sin_table
    from ..models.weights import TPInfo, init_weights
    from ..parallel.comm import init_tp, new_backward_group
    from .trainer import BUCKET_LAYERS, LoraTrainer

    if not torch.cuda.is_available() or not ops.native_available():
        raise SystemExit("bwd_profile needs a GPU and the built extension")
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    comm = init_tp(timeout_s=300) if ws > 1 else None
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dev = torch.device("cuda", torch.cuda.current_device())
    tp = TPInfo(comm.rank, comm.size) if comm is not None else TPInfo()
    bwd_comm = new_backward_group(comm) if comm is not None else None
    arch = resolve_arch(args.model)
    t0 = time.perf_counter()
    w = init_weights(arch, tp, seed=0, device=dev, dtype=torch.bfloat16, keep_full_head=True)
    served = LoraServeBuffers(arch, tp, 2, args.rank, dev, torch.bfloat16)
    n = args.seqs * args.seq_len
    cap = CaptureBuffers.allocate(w, n + 8, dev, torch.bfloat16)
    _fill_capture(cap, n, arch.vocab, seed=5)
    cap.positions[:n].copy_(torch.arange(args.seq_len, device=dev).repeat(args.seqs))
    trainer = LoraTrainer(w, served, 1, args.rank, 2.0 * args.rank, comm=bwd_comm,
                          cos_sin_table=rope_cos_sin_table(max(arch.max_position, 8192), arch.head_dim,
                                                                    arch.rope_theta, arch.rope_scaling, device=dev))
    trainer.init_random(1)
    trainer.publish()
    tpws = None
    if comm is not None and args.tp_comm == "fused":
        from ..parallel.peer import BwdPeerWorkspace
        tpws = BwdPeerWorkspace(comm, n + 8, arch.hidden)
        trainer.bwd.tpws = tpws
    lens = [args.seq_len] * args.seqs
    starts = [i * args.seq_len for i in range(args.seqs)]
    rank0 = tp.rank == 0
    if rank0:
        dprint(f"[bwd_profile] tp={tp.size} model={args.model} rows={n}; set up in "
               f"{time.perf_counter() - t0:.1f}s")
    trainer.warmup(cap, n, starts, lens)
    # ---- production path: graph replays
    gms = []
    for i in range(args.cycles + 1):
        if comm is not None:
            comm.barrier()
        torch.cuda.synchronize()
        ms = trainer.run_cycle(cap, n, starts, lens).gpu_ms
        if i > 0:                      # the first replays upload the graphs
            gms.append(ms)
    if args.profile_cycle:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        trainer.run_cycle(cap, n, starts, lens)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        trainer.release_graphs()
        print(json.dumps({"graph_cycle_ms": sum(gms) / len(gms), "profiled": True}), flush=True)
        return
    # ---- eager path with phase events (the graphs are dropped: a cached
    # graph set would otherwise be replayed)
    trainer.release_graphs()
    trainer.use_graphs = False
    phase_runs, comm_runs, eager_ms = [], [], []
    for _ in range(max(1, args.cycles - 1)):
        if comm is not None:
            comm.barrier()
        torch.cuda.synchronize()
        timer = PhaseTimer()
        trainer.bwd.timer = timer
        torch.cuda._sleep(int(1.5e9))      # ~0.8 s at 1.9 GHz: the host runs ahead of the GPU
        timer.start()
        res = trainer.run_cycle(cap, n, starts, lens)
        trainer.bwd.timer = None
        ph, cm = timer.totals()
        phase_runs.append(ph)
        comm_runs.append(cm)
        eager_ms.append(res.gpu_ms)
    trainer.use_graphs = True

    def mean_dicts(ds):
        keys = set().union(*[d.keys() for d in ds])
        out = {}
        for k in keys:
            vals = [d[k] for d in ds if k in d]
            if isinstance(vals[0], dict):
                out[k] = {kk: sum(v[kk] for v in vals) / len(vals) for kk in vals[0]}
            else:
                out[k] = sum(vals) / len(vals)
        return out
    phases = mean_dicts(phase_runs)
    comms = mean_dicts(comm_runs)
    # ---- collectives alone, at the cycle's sizes
    coll = {}
    if bwd_comm is not None:
        D = arch.hidden
        f32 = torch.zeros(n, D, dtype=torch.float32, device=dev)
        b16 = torch.zeros(n, D, dtype=torch.bfloat16, device=dev)
        m = trainer.masters
        bucket = m.rep_block(m.grads, 0, min(arch.num_layers, BUCKET_LAYERS))
        coll["allreduce_resid_fp32_ms"] = _time_collective(lambda: bwd_comm.all_reduce(f32), 10)
        coll["allreduce_resid_bf16_ms"] = _time_collective(lambda: bwd_comm.all_reduce(b16), 10)
        coll["allreduce_bucket_ms"] = _time_collective(lambda: bwd_comm.all_reduce(bucket), 10)
        coll["bucket_bytes"] = bucket.numel() * 4
        coll["resid_bytes_fp32"] = f32.numel() * 4
        from ..parallel.comm import BWD_NCCL_MAX_CTAS
        coll["bwd_nccl_max_ctas"] = BWD_NCCL_MAX_CTAS
    rec = {"tp": tp.size, "tp_comm": args.tp_comm if comm is not None else None, "model": args.model,
           "rows": n, "seqs": args.seqs, "seq_len": args.seq_len,
           "lora_rank": args.rank,
           "graph_cycle_ms": sum(gms) / len(gms), "graph_cycle_ms_runs": gms,
           "eager_cycle_ms": sum(eager_ms) / len(eager_ms),
           "phases_ms": {k: round(v, 3) for k, v in sorted(phases.items(), key=lambda kv: -kv[1])},
           "phase_sum_ms": round(sum(phases.values()), 3),
           "side_stream_collectives": comms, "collectives": coll,
           "device_error": ops.check_device_error()}
    rec = _max_over_ranks(comm, rec)
    if rank0:
        print(json.dumps(rec), flush=True)
        if args.out:
            os.makedirs(os.path.dirname(os.path.abspath(args.out)), exist_ok=True)
            with open(args.out, "w") as f:
                json.dump(rec, f, indent=1)
    trainer.release_graphs()
    if tpws is not None:
        trainer.bwd.tpws = None
        tpws.close()
    if comm is not None:
        comm.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
