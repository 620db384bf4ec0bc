"""Per-kernel timing against the measured roofline.

    python -m deltaserve_vllm_b200.ops.kernel_bench                 # every case
    python -m deltaserve_vllm_b200.ops.kernel_bench --case gemm_prefill_o --iters 1 --warmup 3

Each case builds Llama-3-8B-shaped inputs (TP=1) on the GPU, runs ``warmup``
untimed launches, then times ``iters`` launches with CUDA events on the
launching stream; an L2 flush (a 256 MiB write, more than the 126 MB L2)
separates timed launches and is excluded from the time. It prints one JSON
line per case: duration, the algorithmic bytes / FLOPs of one launch, and the
achieved fraction of the measured copy bandwidth / bf16 GEMM throughput read
from ``MEASURED_PEAKS.json`` at the repository root (fallback 6.65 TB/s and
1.59 PFLOP/s when the file is absent). With ``--iters 1 --warmup 3`` it is a
small, self-terminating target for an ``ncu`` capture of one kernel.
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch

from .. import ops

DEV = "cuda"


def _peaks() -> dict:
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]), "src": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def rnd(*shape, scale=1.0, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(dtype)


# ------------------------------------------------------------------ cases
# Each returns (launch fn, algorithmic bytes, algorithmic flops).

def _gemm(M, N, K, epi=ops.EPI_BF16, max_ctas=0):
    """``max_ctas``: grid cap (a share of the SMs; 0 = all)."""
    a, b = rnd(M, K, seed=1), rnd(N, K, scale=0.02, seed=2)
    out = torch.empty(M, N // 2 if epi == ops.EPI_SWIGLU else N, dtype=torch.bfloat16, device=DEV)
    return (lambda: ops.gemm(a, b, out, epi=epi, max_ctas=max_ctas),
            2 * (M * K + N * K + out.numel()), 2 * M * N * K)


def _gemm_ar(M, N, K):
    from ..parallel.peer import PeerWorkspace
    ws = PeerWorkspace(None, M, N)
    a, b = rnd(M, K, seed=1), rnd(N, K, scale=0.02, seed=2)
    return (lambda: ops.gemm_ar(a, b, ws), 2 * (M * K + N * K + 2 * M * N), 2 * M * N * K)


def _paged(lens, qlens, Hq=32, Hkv=8, bs=64, seed=0):
    nb = sum(-(-l // bs) for l in lens) + 4
    kc = rnd(nb, Hkv, bs, 128, seed=seed)
    vc = rnd(nb, Hkv, bs, 128, seed=seed + 1)
    maxb = max(-(-l // bs) for l in lens)
    bt = torch.zeros(len(lens), maxb, dtype=torch.int32)
    k = 0
    perm = torch.randperm(nb).tolist()
    for i, l in enumerate(lens):
        n = -(-l // bs)
        bt[i, :n] = torch.tensor(perm[k:k + n])
        k += n
    cu = [0]
    for q in qlens:
        cu.append(cu[-1] + q)
    q = rnd(cu[-1], Hq * 128, seed=seed + 2)
    return kc, vc, bt.to(DEV), cu, torch.tensor(lens, dtype=torch.int32, device=DEV), q


def _prefill(n_seq, L, Hq=32, Hkv=8, warp_kernel=False):
    """Paged causal prefill of n_seq x L new tokens: the tcgen05 kernel, or
    (``warp_kernel``) the warp-level mma.sync kernel on the same tiles."""
    kc, vc, bt, cu, ctx, q = _paged([L] * n_seq, [L] * n_seq, Hq, Hkv)
    tiles = torch.tensor(ops.prefill_tiles(cu), dtype=torch.int32, device=DEV)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=DEV)
    out = torch.empty(q.shape[0], Hq * 128, dtype=torch.bfloat16, device=DEV)
    flops = n_seq * Hq * 128 * 4 * (L * (L + 1) / 2)
    byts = 2 * (2 * q.numel() + 2 * n_seq * L * Hkv * 128)
    if warp_kernel:
        nat = ops._native()
        return (lambda: nat.paged_prefill(q, kc, vc, bt, cu_t, ctx, tiles, out, Hq, 1 / math.sqrt(128),
                                          ops.PREFILL_TILE), byts, flops)
    return (lambda: ops.paged_prefill(q, kc, vc, bt, cu_t, ctx, tiles, out, Hq, 1 / math.sqrt(128)),
            byts, flops)


def _decode(B, L, Hq=32, Hkv=8):
    kc, vc, bt, _, ctx, _ = _paged([L] * B, [1] * B, Hq, Hkv)
    q = rnd(B, Hq * 128, seed=5)
    out = torch.empty(B, Hq * 128, dtype=torch.bfloat16, device=DEV)
    splits, kps = ops.decode_splits(B, Hkv, L)
    po = torch.empty(B * Hq * splits * 128, device=DEV)
    pml = torch.empty(B * Hq * splits * 2, device=DEV)
    byts = 2 * B * L * Hkv * 128 * 2
    return (lambda: ops.paged_decode(q, kc, vc, bt, ctx, out, Hq, 1 / math.sqrt(128), po, pml, splits, kps),
            byts, 4 * B * Hq * 128 * L)


def _rms(T, D):
    x, r = rnd(T, D, seed=1), rnd(T, D, seed=2)
    w = rnd(D, seed=3)
    out = torch.empty_like(x)
    return (lambda: ops.rms_norm(x, w, out, 1e-5, residual=r), 2 * T * D * 4, 0)


def _shrink(T, K, PR, slots=2, seg=64):
    x = rnd(T, K, seed=1)
    A = rnd(slots, PR, K, scale=0.05, seed=2)
    ids = torch.zeros(T, dtype=torch.int32, device=DEV)
    Z = torch.empty(T, slots * seg, dtype=torch.bfloat16, device=DEV)
    return (lambda: ops.lora_shrink(x, A, ids, Z, seg), 2 * (T * K + slots * PR * K + T * slots * seg),
            2 * T * PR * K)


def _rope(T, Hq=32, Hkv=8):
    qkv = rnd(T, (Hq + 2 * Hkv) * 128, seed=1)
    pos = torch.arange(T, dtype=torch.int64, device=DEV)
    cs = ops.ref.rope_cos_sin_table(8192, 128, 5e5, None, device=DEV)
    bs = 64
    nb = -(-T // bs) + 1
    kc = torch.zeros(nb, Hkv, bs, 128, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.arange(T, dtype=torch.int64, device=DEV)
    return (lambda: ops.qk_norm_rope_cache(qkv, pos, cs, None, None, 1e-6, Hq, Hkv, kc, vc, slots),
            2 * (2 * qkv.numel() + 2 * T * Hkv * 128), 0)


def _ce(R, V):
    logits = rnd(R, V, dtype=torch.float32, seed=1)
    tgt = torch.randint(0, V, (R,), device=DEV)
    loss = torch.empty(R, device=DEV)
    grad = torch.empty(R, V, dtype=torch.bfloat16, device=DEV)
    return (lambda: ops.ce_fwd_bwd(logits, tgt, loss, grad, 1.0), R * V * (4 + 2), 0)


def _attn_fwd_dense_tc(n_seq, L, Hq=32, Hkv=8):
    """The trainer's attention recompute on the tcgen05 kernel: O plus the
    row log-sum-exp the backward reuses."""
    from ..models.lora_backward import attention_groups
    n = n_seq * L
    qkv = rnd(n, (Hq + 2 * Hkv) * 128, seed=7)
    q = qkv[:, :Hq * 128].view(n, Hq, 128)
    k = qkv[:, Hq * 128:(Hq + Hkv) * 128].view(n, Hkv, 128)
    v = qkv[:, (Hq + Hkv) * 128:].view(n, Hkv, 128)
    groups = attention_groups([i * L for i in range(n_seq)], [L] * n_seq, DEV)
    out = torch.empty(n, Hq * 128, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(Hq, n, device=DEV)
    flops = n_seq * Hq * 128 * 4 * (L * (L + 1) / 2)
    byts = 2 * qkv.numel() + 2 * out.numel() + 4 * lse.numel()
    return (lambda: ops.attn_fwd_dense(q, k, v, groups.tiles, 1 / math.sqrt(128), out, tiles128=groups.tiles128,
                                       lse=lse), byts, flops)


def _attn_bwd(n_seq, L, Hq=32, Hkv=8, torch_path=False, tc=False):
    """Trainer attention backward over n_seq packed causal samples of L tokens
    (q/k/v strided views of one fused qkv buffer, fp32 dO). FLOPs: the five
    causal 128-deep products of a standard flash backward (QK^T, dP, dV, dQ,
    dK); the fused kernels also recompute QK^T and PV in their q-side pass."""
    from ..models.lora_backward import attn_backward, attention_groups
    n = n_seq * L
    qkv = rnd(n, (Hq + 2 * Hkv) * 128, seed=7)
    q = qkv[:, :Hq * 128].view(n, Hq, 128)
    k = qkv[:, Hq * 128:(Hq + Hkv) * 128].view(n, Hkv, 128)
    v = qkv[:, (Hq + Hkv) * 128:].view(n, Hkv, 128)
    d_o = rnd(n, Hq * 128, dtype=torch.float32, seed=8)
    starts, lens = [i * L for i in range(n_seq)], [L] * n_seq
    groups = attention_groups(starts, lens, DEV)
    flops = 5 * n_seq * Hq * 128 * 2 * (L * (L + 1) / 2)
    byts = 2 * qkv.numel() + 4 * d_o.numel() + 4 * n * (Hq + 2 * Hkv) * 128
    if torch_path:
        fn = lambda: attn_backward(q, k, v, d_o.view(n, Hq, 128), starts, lens, 1 / math.sqrt(128), groups)
    elif tc:
        # The trainer's call: bf16 dO, and O / lse from the recompute forward.
        g = d_o.to(torch.bfloat16)
        o = torch.empty(n, Hq * 128, dtype=torch.bfloat16, device=DEV)
        lse = torch.empty(Hq, n, device=DEV)
        dd = torch.empty_like(lse)
        ops.attn_fwd_dense(q, k, v, groups.tiles, 1 / math.sqrt(128), o, tiles128=groups.tiles128, lse=lse)
        byts = 2 * qkv.numel() + 2 * 2 * d_o.numel() + 4 * n * (Hq + 2 * Hkv) * 128
        fn = lambda: ops.attn_bwd(q, k, v, g, groups.tiles, 1 / math.sqrt(128), o=o, lse=lse,
                                  tiles128=groups.tiles128, dd=dd)
    else:
        fn = lambda: ops.attn_bwd(q, k, v, d_o, groups.tiles, 1 / math.sqrt(128))
    return fn, byts, flops


def _dx_gemm(M, K, N, swiglu: bool):
    """The backward's MN-major dX GEMM (dY [M, K] . W [K, N]); with ``swiglu``
    the epilogue applies the SwiGLU backward over a saved gate/up [M, 2N]."""
    a = rnd(M, K, seed=11)
    b = rnd(K, N, scale=0.02, seed=12)
    flops = 2 * M * N * K
    if swiglu:
        gu = rnd(M, 2 * N, seed=13)
        out = torch.empty(M, 2 * N, dtype=torch.bfloat16, device=DEV)
        byts = 2 * (M * K + K * N) + 2 * 2 * M * 2 * N
        return (lambda: ops.gemm(a, b, out, b_mn=True, epi=ops.EPI_SWIGLU_BWD, aux=gu), byts, flops)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    byts = 2 * (M * K + K * N) + 4 * M * N
    return (lambda: ops.gemm(a, b, out, b_mn=True, epi=ops.EPI_F32), byts, flops)


def _swiglu_bwd(T, I):
    gu = rnd(T, 2 * I, seed=14)
    dact = rnd(T, I, dtype=torch.float32, seed=15)
    dgu = torch.empty(T, 2 * I, dtype=torch.bfloat16, device=DEV)
    return (lambda: ops.swiglu_bwd(gu, dact, dgu), T * I * (2 * 2 + 4 + 2 * 2), 0)


def _rms_bwd(T, D):
    x = rnd(T, D, seed=16)
    w = rnd(D, seed=17)
    dy = rnd(T, D, dtype=torch.float32, seed=18)
    add = rnd(T, D, dtype=torch.float32, seed=19)
    out = torch.empty(T, D, device=DEV)
    obf = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    return (lambda: ops.rms_norm_bwd(x, dy, w, 1e-5, add=add, out=out, out_bf16=obf),
            T * D * (2 + 4 + 4 + 4 + 2), 0)


def _adamw(n):
    p, g = rnd(n, dtype=torch.float32, seed=1), rnd(n, dtype=torch.float32, seed=2)
    m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    return (lambda: ops.adamw(p, g, m, v, seg_len=n, lr=1e-4, step=1), n * 4 * 7, 0)


def _lora_backward(n_seq: int, L: int, graphs: bool):
    """One LoRA backward cycle (head + 2 layers of Llama-3-8B geometry, r=16,
    all projections) over captured activations of n_seq x L tokens, eager or
    as the per-layer CUDA graphs. FLOPs: the frozen dX GEMMs of both layers and
    the LM head (2 x 4 per weight element per token)."""
    from ..engine.trainer import LoraTrainer
    from ..models.configs import resolve_arch
    from ..models.decoder import CaptureBuffers
    from ..models.lora import LoraServeBuffers
    from ..models.weights import TPInfo, init_weights
    arch = resolve_arch("llama3-8b-2l")
    w = init_weights(arch, TPInfo(), seed=0, device=torch.device(DEV), dtype=torch.bfloat16, keep_full_head=True)
    served = LoraServeBuffers(arch, w.tp, 2, 16, torch.device(DEV), torch.bfloat16)
    from .reference import rope_cos_sin_table
    cs = rope_cos_sin_table(8192, arch.head_dim, arch.rope_theta, arch.rope_scaling, device=DEV)
    tr = LoraTrainer(w, served, 1, 16, 32.0, lr=1e-4, cos_sin_table=cs)
    tr.init_random(1)
    tr.use_graphs = graphs
    n = n_seq * L
    cap = CaptureBuffers.allocate(w, n + 8, torch.device(DEV))
    g = torch.Generator(device=DEV).manual_seed(3)
    for t in (cap.layer_in, cap.qkv, cap.ctx, cap.resid_mid, cap.gate_up, cap.act, cap.final_in):
        t.copy_((torch.randn(t.shape, generator=g, device=DEV) * 0.5).to(t.dtype))
    cap.ids.copy_(torch.randint(0, arch.vocab, cap.ids.shape, device=DEV))
    cap.positions.copy_(torch.arange(n + 8, device=DEV) % L)
    starts, lens = [i * L for i in range(n_seq)], [L] * n_seq
    # dX of every frozen projection (2 FLOPs per weight element per token) in
    # both layers, plus the LM head forward and dX.
    per_tok = 2 * (arch.hidden * (arch.q_size + 2 * arch.kv_size) + arch.q_size * arch.hidden
                   + 3 * arch.hidden * arch.intermediate) * arch.num_layers + 4 * arch.hidden * arch.vocab
    flops = n * per_tok
    return (lambda: tr.run_cycle(cap, n, starts, lens), 0, flops)


CASES = {
    # Llama-3-8B projections, 4096-token prefill step (TP=1)
    "gemm_prefill_qkv": lambda: _gemm(4096, 6144, 4096),
    "gemm_prefill_o": lambda: _gemm(4096, 4096, 4096),
    "gemm_prefill_gateup_swiglu": lambda: _gemm(4096, 28672, 4096, ops.EPI_SWIGLU),
    "gemm_prefill_down": lambda: _gemm(4096, 4096, 14336),
    # decode step of 64 sequences (split-K, weight-streaming bound)
    "gemm_decode_qkv": lambda: _gemm(64, 6144, 4096),
    "gemm_decode_qkv_cap74": lambda: _gemm(64, 6144, 4096, max_ctas=74),
    "gemm_decode_qkv_cap96": lambda: _gemm(64, 6144, 4096, max_ctas=96),
    "gemm_decode_gateup_swiglu": lambda: _gemm(64, 28672, 4096, ops.EPI_SWIGLU),
    "gemm_decode_gateup_swiglu_cap74": lambda: _gemm(64, 28672, 4096, ops.EPI_SWIGLU, max_ctas=74),
    "gemm_decode_gateup_swiglu_cap96": lambda: _gemm(64, 28672, 4096, ops.EPI_SWIGLU, max_ctas=96),
    "gemm_decode_down": lambda: _gemm(64, 4096, 14336),
    "gemm_decode_down_cap74": lambda: _gemm(64, 4096, 14336, max_ctas=74),
    "gemm_decode_down_cap96": lambda: _gemm(64, 4096, 14336, max_ctas=96),
    # fused GEMM + all-reduce on one rank (the push / reduce / broadcast phases run locally)
    "gemm_ar_prefill_o": lambda: _gemm_ar(4096, 4096, 4096),
    "gemm_ar_decode_down": lambda: _gemm_ar(64, 4096, 14336),
    "attn_prefill_8x512": lambda: _prefill(8, 512),
    "attn_prefill_2x2048": lambda: _prefill(2, 2048),
    "attn_prefill_warp_8x512": lambda: _prefill(8, 512, warp_kernel=True),
    "attn_prefill_warp_2x2048": lambda: _prefill(2, 2048, warp_kernel=True),
    "attn_fwd_dense_tc_8x512": lambda: _attn_fwd_dense_tc(8, 512),
    "attn_bwd_tc_8x512": lambda: _attn_bwd(8, 512, tc=True),
    # one TP = 8 rank's share of the same attention: 4 query heads, 1 KV head
    "attn_prefill_8x512_tp8": lambda: _prefill(8, 512, Hq=4, Hkv=1),
    "attn_fwd_dense_tc_8x512_tp8": lambda: _attn_fwd_dense_tc(8, 512, Hq=4, Hkv=1),
    "attn_bwd_tc_8x512_tp8": lambda: _attn_bwd(8, 512, Hq=4, Hkv=1, tc=True),
    "attn_bwd_8x512_tp8": lambda: _attn_bwd(8, 512, Hq=4, Hkv=1),
    "attn_bwd_8x512": lambda: _attn_bwd(8, 512),
    "attn_bwd_torch_fp32_8x512": lambda: _attn_bwd(8, 512, torch_path=True),
    "attn_decode_64x1024": lambda: _decode(64, 1024),
    "attn_decode_16x4096": lambda: _decode(16, 4096),
    "rms_norm_add_8192x4096": lambda: _rms(8192, 4096),
    "rms_norm_bwd_4096x4096": lambda: _rms_bwd(4096, 4096),
    "rms_norm_bwd_qknorm_131072x128": lambda: _rms_bwd(131072, 128),
    # backward dX of the down projection (Llama-3-8B, 4096 FT tokens): plain
    # fp32 store, and with the SwiGLU backward fused in the epilogue
    "gemm_dx_down_f32": lambda: _dx_gemm(4096, 4096, 14336, False),
    "gemm_dx_down_swiglu_bwd": lambda: _dx_gemm(4096, 4096, 14336, True),
    "swiglu_bwd_4096x14336": lambda: _swiglu_bwd(4096, 14336),
    "lora_shrink_4096x4096_r16x3": lambda: _shrink(4096, 4096, 48),
    "lora_shrink_decode_16x4096_r16x3": lambda: _shrink(16, 4096, 48),
    "lora_shrink_decode_16x14336_r16": lambda: _shrink(16, 14336, 16),
    "rope_kvwrite_4096": lambda: _rope(4096),
    "ce_fwd_bwd_512x128256": lambda: _ce(512, 128256),
    "adamw_64M": lambda: _adamw(64 << 20),
    "lora_backward_2l_8x512_eager": lambda: _lora_backward(8, 512, False),
    "lora_backward_2l_8x512_graphs": lambda: _lora_backward(8, 512, True),
}


def run_case(name: str, iters: int, warmup: int, flush: torch.Tensor) -> dict:
    fn, byts, flops = CASES[name]()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush.fill_(1.0)           # evict the inputs from L2
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        total += e0.elapsed_time(e1)
    assert ops.check_device_error() == 0, "kernel reported a device error"
    ms = total / iters
    pk = _peaks()
    out = {"case": name, "ms": round(ms, 4), "bytes": int(byts), "flops": int(flops),
           "tb_s": round(byts / ms / 1e9, 3), "tflops": round(flops / ms / 1e9, 1), "peaks": pk["src"]}
    out["frac_hbm"] = round(byts / ms / 1e9 / (pk["hbm_gbs"] / 1e3), 3)
    out["frac_tensor"] = round(flops / ms / 1e9 / pk["bf16_tflops"], 3) if flops else None
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", action="append", help="case name (repeatable); default: all")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=DEV)
    for name in args.case or list(CASES):
        print(json.dumps(run_case(name, args.iters, args.warmup, flush)), flush=True)


if __name__ == "__main__":
    main()
