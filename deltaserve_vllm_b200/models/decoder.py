"""Serving forward of the Llama-3 / Qwen3 decoder over one flattened batch.

A step's batch is laid out as: decode tokens first (one per sequence), then
the prefill chunks of inference requests, then the finetuning (FT) samples,
so the FT rows are one contiguous range ``[ft_lo, ft_hi)`` at the end. The
activations the LoRA backward needs are captured for exactly those rows as a
second store inside the kernels that produce them (the reference registers
per-layer hooks that index_copy them, ``deltaserve-plugin/deltaserve/accumulate.py:345-579``):

* ``layer_in[l]``  residual stream entering layer l   (fused add+RMSNorm)
* ``qkv[l]``       raw q/k/v projection output          (qkv GEMM epilogue)
* ``ctx[l]``       attention output                      (row-range copy)
* ``resid_mid[l]`` residual after attention              (fused add+RMSNorm)
* ``gate_up[l]``   raw gate/up pre-activation            (SwiGLU GEMM epilogue)
* ``final_in``     final residual stream                 (final add+RMSNorm)

Per layer: RMSNorm -> qkv GEMM (+LoRA) -> q/k norm + RoPE + KV write ->
paged attention -> o GEMM (+LoRA) -> TP all-reduce -> add+RMSNorm ->
gate_up GEMM with SwiGLU epilogue (+LoRA) -> down GEMM (+LoRA) -> all-reduce.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from .. import ops
from ..ops import EPI_BF16, EPI_F32, EPI_SWIGLU
from .configs import ModelArch
from .lora import LoraServeBuffers
from .weights import ModelWeights

# Launch each LoRA GEMM to overlap the shrink kernel right before it (its base
# K blocks stream while the shrink runs); DSV_OVERLAP_SHRINK=0 serialises them.
OVERLAP_SHRINK = os.environ.get("DSV_OVERLAP_SHRINK", "1") != "0"
# Grid cap of the forward's GEMMs when the batch has at most 128 rows
# (decode): these stream weights at the HBM bound, so fewer SMs can keep the
# same pace and the rest stay free for a concurrently running backward.
# 0 = every SM.
FWD_SMALL_GEMM_CTAS = int(os.environ.get("DSV_FWD_SMALL_GEMM_CTAS", "0"))


@dataclass
class ForwardBatch:
    input_ids: torch.Tensor          # [T] int64
    positions: torch.Tensor          # [T] int64
    slot_mapping: torch.Tensor       # [T] int64 (-1 = do not cache)
    num_decode: int = 0
    dec_block_tables: torch.Tensor | None = None   # [B_d, maxb] int32
    dec_ctx_lens: torch.Tensor | None = None       # [B_d] int32
    dec_splits: int = 1
    dec_keys_per_split: int = 64
    num_prefill_seqs: int = 0
    pf_cu_q: torch.Tensor | None = None            # [S+1] int32, relative to num_decode
    pf_ctx_lens: torch.Tensor | None = None        # [S] int32
    pf_block_tables: torch.Tensor | None = None    # [S, maxb] int32
    pf_tile_info: torch.Tensor | None = None       # [tiles, 2] int32
    slot_ids: torch.Tensor | None = None           # [T] int32 LoRA slot per token (-1 none)
    tile_slots: torch.Tensor | None = None         # [ceil(T/128)] int32 slot bitmask per M tile
    logits_idx: torch.Tensor | None = None         # [R] int64 rows whose logits are needed
    ft_lo: int = 0
    ft_hi: int = 0
    ft_dst: int = 0

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])


@dataclass
class CaptureBuffers:
    """Activation-capture buffers for up to ``cap`` FT tokens per backward cycle."""
    layer_in: torch.Tensor   # [L, cap, D]
    qkv: torch.Tensor        # [L, cap, qkv_l]
    ctx: torch.Tensor        # [L, cap, q_l]
    resid_mid: torch.Tensor  # [L, cap, D]
    gate_up: torch.Tensor    # [L, cap, 2*I_l]
    act: torch.Tensor        # [L, cap, I_l]  silu(gate) * up (the down projection's input)
    final_in: torch.Tensor   # [cap, D]
    ids: torch.Tensor        # [cap] int64
    positions: torch.Tensor  # [cap] int64

    @staticmethod
    def allocate(w: ModelWeights, cap: int, device, dtype=torch.bfloat16, save_qkv: bool = True,
                 save_ctx: bool = True, save_resid_mid: bool = True) -> "CaptureBuffers":
        """Buffers switched off by ``save_*`` are None: the backward recomputes
        those activations from the layer input instead."""
        a = w.arch
        L, D = a.num_layers, a.hidden
        qkv_l = w.q_local + 2 * w.kv_local
        z = lambda *s: torch.zeros(*s, dtype=dtype, device=device)
        return CaptureBuffers(
            layer_in=z(L, cap, D), qkv=z(L, cap, qkv_l) if save_qkv else None,
            ctx=z(L, cap, w.q_local) if save_ctx else None,
            resid_mid=z(L, cap, D) if save_resid_mid else None,
            gate_up=z(L, cap, 2 * w.i_local), act=z(L, cap, w.i_local),
            final_in=z(cap, D),
            ids=torch.zeros(cap, dtype=torch.long, device=device),
            positions=torch.zeros(cap, dtype=torch.long, device=device))

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.layer_in, self.qkv, self.ctx, self.resid_mid, self.gate_up, self.act,
                    self.final_in) if t is not None)


class FTAborted(Exception):
    """Raised between layers when an FT-only forward is pre-empted (tier C)."""


class Communicator:
    """Tensor-parallel collectives used by the forward. ``size == 1`` is a no-op."""

    size = 1

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        return t

    def all_gather_cols(self, t: torch.Tensor) -> torch.Tensor:
        return t


class DecoderModel:
    def __init__(self, weights: ModelWeights, kv_k: list[torch.Tensor] | None,
                 kv_v: list[torch.Tensor] | None, lora: LoraServeBuffers | None = None,
                 comm: Communicator | None = None):
        self.w = weights
        self.arch: ModelArch = weights.arch
        self.kv_k, self.kv_v = kv_k, kv_v
        self.lora = lora
        self.comm = comm or Communicator()
        dev = weights.embed.device
        self.cos_sin = ops.ref.rope_cos_sin_table(
            max(self.arch.max_position, 8192), self.arch.head_dim, self.arch.rope_theta,
            self.arch.rope_scaling, device=dev)
        self.hq_l = self.arch.num_heads // weights.tp.size
        self.hkv_l = self.arch.num_kv_heads // weights.tp.size
        self.scale = 1.0 / math.sqrt(self.arch.head_dim)
        self._dec_ws: tuple[torch.Tensor, torch.Tensor] | None = None
        # A parallel.peer.PeerTable of the embedding shards (set by the engine
        # under TP with the fused communication path) replaces embedding + all-reduce.
        self.embed_peer = None

    # ------------------------------------------------------------------ helpers
    def _proj(self, x, w, out, layer: int, group: str, b: ForwardBatch, epi=EPI_BF16, save=None,
              save_lo=0, save_hi=0, save_dst=0):
        kw = {}
        if self.lora is not None and b.slot_ids is not None:
            A = self.lora.A[layer][group]
            seg = self.lora.seg[group]
            z = torch.empty(x.shape[0], A.shape[0] * seg, dtype=x.dtype, device=x.device)
            ops.lora_shrink(x, A, b.slot_ids, z, seg)
            kw = dict(z=z, b2=self.lora.B2[layer][group], tile_slots=b.tile_slots, lora_seg=seg,
                      after_shrink=OVERLAP_SHRINK)
        cap = FWD_SMALL_GEMM_CTAS if x.shape[0] <= 128 else 0
        return ops.gemm(x, w, out, epi=epi, save=save, save_lo=save_lo, save_hi=save_hi,
                        save_dst=save_dst, max_ctas=cap, **kw)

    def _proj_reduce(self, x, w, out, layer: int, group: str, b: ForwardBatch):
        """Row-parallel projection followed by the TP all-reduce. With a peer
        workspace on the communicator (``tp_comm: fused``) both happen in one
        kernel over NVLink peer memory; otherwise GEMM then NCCL all-reduce."""
        ws = getattr(self.comm, "peer_ws", None)
        if ws is None or not ws.prefer(x.shape[0], w.shape[0]):
            self._proj(x, w, out, layer, group, b)
            return self.comm.all_reduce(out)
        kw = {}
        if self.lora is not None and b.slot_ids is not None:
            A = self.lora.A[layer][group]
            seg = self.lora.seg[group]
            z = torch.empty(x.shape[0], A.shape[0] * seg, dtype=x.dtype, device=x.device)
            ops.lora_shrink(x, A, b.slot_ids, z, seg)
            kw = dict(z=z, b2=self.lora.B2[layer][group], tile_slots=b.tile_slots, lora_seg=seg)
        return ops.gemm_ar(x, w, ws, **kw)

    def _decode_ws(self, n: int, device):
        need_o = n * 128
        if self._dec_ws is None or self._dec_ws[0].numel() < need_o:
            # Sized once for every decode shape (CUDA graphs keep the address).
            self._dec_ws = (torch.empty(max(need_o, 1 << 22), dtype=torch.float32, device=device),
                            torch.empty(max(n * 2, 1 << 16), dtype=torch.float32, device=device))
        return self._dec_ws

    def attention(self, layer: int, qkv: torch.Tensor, ctx: torch.Tensor, b: ForwardBatch):
        q = qkv[:, : self.w.q_local]
        kc, vc = self.kv_k[layer], self.kv_v[layer]
        nd = b.num_decode
        if nd > 0:
            po, pml = self._decode_ws(nd * self.hq_l * b.dec_splits, qkv.device)
            ops.paged_decode(q[:nd], kc, vc, b.dec_block_tables, b.dec_ctx_lens, ctx[:nd], self.hq_l,
                             self.scale, po, pml, b.dec_splits, b.dec_keys_per_split)
        if b.num_prefill_seqs > 0:
            ops.paged_prefill(q[nd:], kc, vc, b.pf_block_tables, b.pf_cu_q, b.pf_ctx_lens,
                              b.pf_tile_info, ctx[nd:], self.hq_l, self.scale)

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, b: ForwardBatch, cap: CaptureBuffers | None = None, layer_hook=None) -> torch.Tensor:
        """Runs all layers; returns fp32 logits [R, V] for ``b.logits_idx`` rows
        (or the final hidden states [T, D] when ``logits_idx`` is None).
        ``layer_hook(l)`` runs on the host before layer ``l`` is enqueued; a
        True return abandons the forward (:class:`FTAborted`)."""
        a, w = self.arch, self.w
        T, D = b.num_tokens, a.hidden
        dev, dt = w.embed.device, w.embed.dtype
        cap_on = cap is not None and b.ft_hi > b.ft_lo
        lo, hi, dst = (b.ft_lo, b.ft_hi, b.ft_dst) if cap_on else (0, 0, 0)

        residual = torch.empty(T, D, dtype=dt, device=dev)
        if self.embed_peer is not None:
            ops.embedding_peer(b.input_ids, self.embed_peer, residual)     # every shard over peer memory
        else:
            ops.embedding(b.input_ids, w.embed, residual, w.tp.rank * w.v_local)
            self.comm.all_reduce(residual)
        if cap_on:
            cap.ids[dst:dst + hi - lo] = b.input_ids[lo:hi]
            cap.positions[dst:dst + hi - lo] = b.positions[lo:hi]

        x = torch.empty(T, D, dtype=dt, device=dev)
        qkv = torch.empty(T, w.q_local + 2 * w.kv_local, dtype=dt, device=dev)
        ctx = torch.empty(T, w.q_local, dtype=dt, device=dev)
        o = torch.empty(T, D, dtype=dt, device=dev)
        act = torch.empty(T, w.i_local, dtype=dt, device=dev)
        mlp = torch.empty(T, D, dtype=dt, device=dev)
        eps = a.rms_eps
        for l, lw in enumerate(w.layers):
            if layer_hook is not None and layer_hook(l):
                raise FTAborted(l)
            sv = cap.layer_in[l] if cap_on else None
            if l == 0:
                ops.rms_norm(residual, lw.in_ln, x, eps, save=sv, save_lo=lo, save_hi=hi, save_dst=dst)
            else:
                ops.rms_norm(mlp_red, lw.in_ln, x, eps, residual=residual, save=sv, save_lo=lo,
                             save_hi=hi, save_dst=dst)
            self._proj(x, lw.qkv, qkv, l, "qkv", b,
                       save=cap.qkv[l] if cap_on and cap.qkv is not None else None,
                       save_lo=lo, save_hi=hi, save_dst=dst)
            ops.qk_norm_rope_cache(qkv, b.positions, self.cos_sin, lw.q_norm, lw.k_norm, eps,
                                   self.hq_l, self.hkv_l, self.kv_k[l], self.kv_v[l], b.slot_mapping)
            self.attention(l, qkv, ctx, b)
            if cap_on and cap.ctx is not None:
                cap.ctx[l, dst:dst + hi - lo] = ctx[lo:hi]
            o_red = self._proj_reduce(ctx, lw.o, o, l, "o", b)
            ops.rms_norm(o_red, lw.post_ln, x, eps, residual=residual,
                         save=cap.resid_mid[l] if cap_on and cap.resid_mid is not None else None,
                         save_lo=lo, save_hi=hi,
                         save_dst=dst)
            self._proj(x, lw.gate_up, act, l, "gate_up", b, epi=EPI_SWIGLU,
                       save=cap.gate_up[l] if cap_on else None, save_lo=lo, save_hi=hi,
                       save_dst=dst)
            if cap_on:
                cap.act[l, dst:dst + hi - lo] = act[lo:hi]
            mlp_red = self._proj_reduce(act, lw.down, mlp, l, "down", b)
        ops.rms_norm(mlp_red, w.final_norm, x, eps, residual=residual,
                     save=cap.final_in if cap_on else None, save_lo=lo, save_hi=hi, save_dst=dst)
        if b.logits_idx is None:
            return x
        rows = x.index_select(0, b.logits_idx) if b.logits_idx.numel() else x[:0]
        logits = torch.empty(rows.shape[0], w.v_local, dtype=torch.float32, device=dev)
        if rows.shape[0]:
            ops.gemm(rows.contiguous(), w.lm_head, logits, epi=EPI_F32)
        return self.comm.all_gather_cols(logits)
