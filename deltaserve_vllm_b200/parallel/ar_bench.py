"""Fused GEMM + all-reduce vs GEMM then NCCL all-reduce, on N GPUs.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29600 -m deltaserve_vllm_b200.parallel.ar_bench [--iters 20]

Shapes are Llama-3-8B's row-parallel projections at this TP degree
(o: K = 4096/tp, down: K = 14336/tp, N = 4096) for a decode step (M = 64) up
to prefill steps (M = 4096, 8192), then the backward's residual-gradient
reductions (see ``_backward_cases``) and the all-gather -> column-parallel
GEMMs (see ``_all_gather_cases``). Each variant is timed with CUDA events over
``iters`` launches after warm-up; the max over ranks is reported. The
roofline of the fused path is the slower of its FLOPs at the measured bf16
peak and the bytes each rank must send over NVLink at 770 GB/s per direction
(one-shot push of the partial, (tp-1)/tp of it, plus the reduced result to
tp-1 peers, (tp-1)/tp of it).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from .. import ops
from ..ops.kernel_bench import _peaks
from .comm import init_tp
from .peer import PeerWorkspace

NVLINK_GBS = 770.0


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", choices=["all_reduce", "backward", "all_gather"], default=None,
                    help="run one group of cases")
    args = ap.parse_args(argv)
    comm = init_tp()
    tp, rank = comm.size, comm.rank
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    ws = PeerWorkspace(comm, 8192, 4096)
    peak = _peaks()
    g = torch.Generator(device="cuda").manual_seed(rank)
    ar_cases = [] if args.only not in (None, "all_reduce") else [
                       ("o_decode", 64, 4096 // tp), ("down_decode", 64, 14336 // tp),
                       ("o_m256", 256, 4096 // tp), ("o_m1024", 1024, 4096 // tp),
                       ("down_m1024", 1024, 14336 // tp), ("o_m2048", 2048, 4096 // tp),
                       ("o_prefill", 4096, 4096 // tp), ("down_prefill", 4096, 14336 // tp),
                       ("o_m8192", 8192, 4096 // tp), ("down_m8192", 8192, 14336 // tp)]
    for name, M, K in ar_cases:
        N = 4096
        a = torch.randn(M, K, generator=g, device="cuda").bfloat16()
        b = (torch.randn(N, K, generator=g, device="cuda") * 0.02).bfloat16()
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")

        def base():
            ops.gemm(a, b, out)
            dist.all_reduce(out)

        def gemm_only():
            ops.gemm(a, b, out)

        def fused():
            ops.gemm_ar(a, b, ws)

        def fused_r0():      # GEMM CTAs reduce after their tiles
            ops.gemm_ar(a, b, ws, force_reducers=0)

        def fused_r16():     # 16 dedicated reducer CTAs overlap the exchange
            ops.gemm_ar(a, b, ws, force_reducers=16)

        t_base, t_gemm, t_fused = _time(base, args.iters), _time(gemm_only, args.iters), _time(fused, args.iters)
        t_r0, t_r16 = _time(fused_r0, args.iters), _time(fused_r16, args.iters)
        ref = a.float() @ b.float().t()
        dist.all_reduce(ref)
        err = float((ops.gemm_ar(a, b, ws).float() - ref).abs().max() / ref.abs().max())
        flops = 2 * M * N * K
        nvl_bytes = 2 * (tp - 1) / tp * M * N * 2
        bound_ms = max(flops / (peak["bf16_tflops"] * 1e9), nvl_bytes / (NVLINK_GBS * 1e6))
        if rank == 0:
            print(json.dumps({"case": name, "tp": tp, "M": M, "N": N, "K": K, "gemm_ms": round(t_gemm, 4),
                              "gemm_nccl_ms": round(t_base, 4), "fused_ms": round(t_fused, 4),
                              "fused_r0_ms": round(t_r0, 4), "fused_r16_ms": round(t_r16, 4),
                              "speedup_vs_nccl": round(t_base / t_fused, 3),
                              "roofline_ms": round(bound_ms, 4), "frac_roofline": round(bound_ms / t_fused, 3),
                              "max_rel_err": round(err, 5), "peaks": peak["src"]}), flush=True)
    if args.only in (None, "backward"):
        _backward_cases(comm, args.iters, peak, g)
    if args.only in (None, "all_gather"):
        _all_gather_cases(comm, args.iters, peak, g)
    assert ops.check_device_error() == 0
    ws.close()
    dist.destroy_process_group()


def _backward_cases(comm, iters: int, peak: dict, g) -> None:
    """The backward's residual-gradient reduction at Llama-3-8B shapes (4096
    FT rows): dX GEMM (MN-major) + row push + owner reduce + RMSNorm backward
    + all-gather over peer memory, against GEMM (fp32 out) + NCCL fp32
    all-reduce + RMSNorm backward, and against GEMM + NCCL bf16 all-reduce.
    Roofline: the slower of the GEMM at peak and the push + gather bytes
    ((tp-1)/tp of the bf16 rows each way) at 770 GB/s."""
    from .peer import BwdPeerWorkspace
    tp, rank = comm.size, comm.rank
    M, D = 4096, 4096
    bws = BwdPeerWorkspace(comm, M, D)
    x = torch.randn(M, D, generator=g, device="cuda").bfloat16()
    wn = (torch.randn(D, generator=g, device="cuda") * 0.1 + 1).bfloat16()
    add = torch.randn(M, D, generator=g, device="cuda")
    out32 = torch.empty(M, D, device="cuda")
    for name, K in [("bwd_gate_up_dx", 2 * 14336 // tp), ("bwd_qkv_dx", 6144 // tp)]:
        a = torch.randn(M, K, generator=g, device="cuda").bfloat16()
        b = (torch.randn(K, D, generator=g, device="cuda") * 0.02).bfloat16()
        y32 = torch.empty(M, D, device="cuda")
        y16 = torch.empty(M, D, dtype=torch.bfloat16, device="cuda")

        def fused():
            ops.gemm_push(a, b, bws)
            ops.tp_reduce_rows(bws, M, 0, out32, x=x, w=wn, eps=1e-5, add=add)

        def nccl_f32():
            ops.gemm(a, b, y32, b_mn=True, epi=ops.EPI_F32)
            dist.all_reduce(y32)
            ops.rms_norm_bwd(x, y32, wn, 1e-5, add=add, out=out32)

        def nccl_bf16():
            ops.gemm(a, b, y16, b_mn=True, epi=ops.EPI_BF16)
            dist.all_reduce(y16)

        t_f, t_n32, t_n16 = _time(fused, iters), _time(nccl_f32, iters), _time(nccl_bf16, iters)
        flops = 2 * M * D * K
        nvl = 2 * (tp - 1) / tp * M * D * 2
        bound = max(flops / (peak["bf16_tflops"] * 1e9), nvl / (NVLINK_GBS * 1e6))
        if rank == 0:
            print(json.dumps({"case": name, "tp": tp, "M": M, "N": D, "K": K, "fused_ms": round(t_f, 4),
                              "gemm_nccl_f32_norm_ms": round(t_n32, 4), "gemm_nccl_bf16_ms": round(t_n16, 4),
                              "speedup_vs_nccl_f32": round(t_n32 / t_f, 3), "roofline_ms": round(bound, 4),
                              "frac_roofline": round(bound / t_f, 3), "peaks": peak["src"]}), flush=True)
    bws.close()


def _all_gather_cases(comm, iters: int, peak: dict, g) -> None:
    """All-gather -> column-parallel GEMM (qkv, gate_up + SwiGLU) at Llama-3-8B
    shapes: the GEMM copying each remote row block once from its owner's
    memory (``ops.gemm_ag``; ``tile_reads_from_owner_ms``: every tile read
    from the owner by TMA instead) against NCCL all-gather into a local
    tensor + GEMM.
    Roofline: the slower of the GEMM at peak and the (tp-1)/tp of the rows
    that cross NVLink at 770 GB/s."""
    from .peer import AGPeerWorkspace
    tp, rank = comm.size, comm.rank
    D = 4096
    ws = AGPeerWorkspace(comm, 8192 // tp, D)
    for M in (1024, 4096, 8192):
        rows = M // tp
        if rows % 128:
            continue
        x = torch.randn(rows, D, generator=g, device="cuda").bfloat16()
        ws.local[:rows].copy_(x)
        full = torch.empty(M, D, dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        comm.barrier()
        for name, N, epi in [("qkv", 6144 // tp, ops.EPI_BF16), ("gate_up_swiglu", 2 * 14336 // tp, ops.EPI_SWIGLU)]:
            w = (torch.randn(N, D, generator=g, device="cuda") * 0.02).bfloat16()
            out = torch.empty(M, N // 2 if epi == ops.EPI_SWIGLU else N, dtype=torch.bfloat16, device="cuda")

            def fused():
                ops.gemm_ag(ws, rows, w, out, epi=epi)

            def direct():
                ops.gemm_ag(ws, rows, w, out, epi=epi, copy_once=False)

            def nccl():
                dist.all_gather_into_tensor(full, x)
                ops.gemm(full, w, out, epi=epi)

            def gemm_only():
                ops.gemm(full, w, out, epi=epi)

            t_f, t_n, t_g, t_d = _time(fused, iters), _time(nccl, iters), _time(gemm_only, iters), _time(direct, iters)
            flops = 2 * M * N * D
            nvl = (tp - 1) / tp * M * D * 2
            bound = max(flops / (peak["bf16_tflops"] * 1e9), nvl / (NVLINK_GBS * 1e6))
            if rank == 0:
                print(json.dumps({"case": f"ag_{name}_m{M}", "tp": tp, "M": M, "N": N, "K": D,
                                  "gemm_ms": round(t_g, 4), "ag_nccl_gemm_ms": round(t_n, 4),
                                  "fused_ms": round(t_f, 4), "tile_reads_from_owner_ms": round(t_d, 4),
                                  "speedup_vs_nccl": round(t_n / t_f, 3),
                                  "roofline_ms": round(bound, 4), "frac_roofline": round(bound / t_f, 3),
                                  "peaks": peak["src"]}), flush=True)
    ws.close()


if __name__ == "__main__":
    main()
