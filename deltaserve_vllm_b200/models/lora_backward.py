"""Hand-written LoRA backward over the activations captured in the serving forward.

The math follows the reference's manual backward (Llama-3:
``deltaserve-plugin/deltaserve/bwd_services/llama3.py:149-219``; Qwen3 adds the
per-head q/k RMSNorm backward, ``bwd_services/qwen3.py:133-204``), extended to
LoRA on all seven projections and to prompt-masked labels, and laid out for
this engine's fused weights:

* The LoRA factors of one projection *group* (qkv / o / gate_up / down, see
  ``models/lora.py``) are kept as one fp32 master pair ``A [P*R, K]`` and
  ``Bt [R, N]`` (``Bt[j, n] = B_p(n)[n, j]``). Every group backward is five
  GEMMs on the group's input ``X`` and output gradient ``dY``::

      Z   = X A^T                 dZ  = dY Bfull         (Bfull = scatter(Bt) * s)
      dX += dZ A                  dA  = dZ^T X           dBfull^T = s Z^T dY

* The base-weight input gradients ``dX = dY W`` are "MN-major" GEMMs on the
  tcgen05 kernel (no transposed weight copy).
* Attention: on CUDA the fused varlen flash-style backward of
  ``ops/csrc/attn_bwd.cu`` (scores, softmax statistics and the dS terms in
  fp32 registers; the S / P / dS tiles never reach memory); on CPU the fp32
  batched-matmul oracle :func:`attn_backward`.
* Precision: GEMM operands bf16 with fp32 accumulation; residual-stream
  gradient, RMSNorm backward, attention scores/softmax and the LM head / CE in
  fp32 (the reference's precision contract).

Tensor parallelism: the two residual-stream gradients per layer (after the MLP
and after the qkv input gradient) are per-rank partials. On GPUs with the
peer workspace (:attr:`LoraBackward.tpws`) each dX GEMM pushes its bf16 partial
rows to their owner rank, which sums them, applies the RMSNorm backward for
its rows and all-gathers the bf16 result over NVLink (``ops/csrc/tp_bwd.cu``);
otherwise ``comm.all_reduce`` sums them from a side stream. Either way the
factor-gradient GEMMs of the same half-layer run meanwhile. The LM head is
vocabulary-parallel: each rank computes the cross-entropy statistics and
gradient of its vocabulary slice only. Replicated factor gradients
(column-parallel ``A``, row-parallel ``B``) are summed by the trainer in
buckets, overlapped with the next layer's backward.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .. import ops
from ..ops import EPI_BF16, EPI_F32, EPI_F32_ACCUM, EPI_SWIGLU_BWD
from ..ops.reference import interleave64
from .configs import ModelArch
from .lora import GROUP_PROJS, GROUPS, GroupGeom, group_geoms, peft_key, shard_lora_factor
from .rope import rope_backward
from .weights import ModelWeights, TPInfo

REPLICATED = {"qkv": "A", "gate_up": "A", "o": "B", "down": "B"}


class LoraMasters:
    """fp32 masters of one trained adapter for every layer and group, as views
    into flat ``params`` / ``grads`` buffers laid out in two blocks:

    * ``[0, rep_total)``: the factors replicated across TP ranks (column-parallel
      ``A``, row-parallel ``B``), one contiguous segment per layer — a bucket of
      consecutive layers is one contiguous slab for the gradient all-reduce;
    * ``[rep_total, total)``: the per-rank shards, one segment per layer.

    AdamW is then two launches and per-layer clipping two segmented reductions."""

    def __init__(self, arch: ModelArch, tp: TPInfo, rank: int, device):
        self.arch, self.tp, self.R = arch, tp, rank
        self.geom = group_geoms(arch, tp)
        L = arch.num_layers
        rep, shard = [], []
        for g in GROUPS:
            gg = self.geom[g]
            for ab, shape in (("A", (gg.P * rank, gg.K)), ("Bt", (rank, gg.N))):
                is_rep = (REPLICATED[g] == "A") == (ab == "A")
                (rep if is_rep else shard).append((g, ab, shape))
        self.rep_per_layer = sum(s[0] * s[1] for _, _, s in rep)
        self.shard_per_layer = sum(s[0] * s[1] for _, _, s in shard)
        self.rep_total = self.rep_per_layer * L
        total = self.rep_total + self.shard_per_layer * L
        self.layout: list[tuple[str, str, int, int, tuple[int, ...]]] = []  # (g, ab, base, stride, shape)
        off = 0
        for g, ab, shape in rep:
            self.layout.append((g, ab, off, self.rep_per_layer, shape))
            off += shape[0] * shape[1]
        off = self.rep_total
        for g, ab, shape in shard:
            self.layout.append((g, ab, off, self.shard_per_layer, shape))
            off += shape[0] * shape[1]
        self.params = torch.zeros(total, dtype=torch.float32, device=device)
        self.grads = torch.zeros_like(self.params)
        self.exp_avg = torch.zeros_like(self.params)
        self.exp_avg_sq = torch.zeros_like(self.params)
        self._views_p = self._views(self.params)
        self._views_g = self._views(self.grads)

    def _views(self, flat):
        out = []
        for l in range(self.arch.num_layers):
            d = {}
            for g, ab, base, stride, shape in self.layout:
                s = base + l * stride
                d[(g, ab)] = flat[s:s + shape[0] * shape[1]].view(shape)
            out.append(d)
        return out

    def rep_block(self, flat: torch.Tensor, l0: int = 0, l1: int | None = None) -> torch.Tensor:
        l1 = self.arch.num_layers if l1 is None else l1
        return flat[l0 * self.rep_per_layer:l1 * self.rep_per_layer]

    def shard_block(self, flat: torch.Tensor) -> torch.Tensor:
        return flat[self.rep_total:]

    def p(self, layer, group, ab):
        return self._views_p[layer][(group, ab)]

    def g(self, layer, group, ab):
        return self._views_g[layer][(group, ab)]

    @torch.no_grad()
    def load_peft(self, tensors: dict[str, torch.Tensor], rank: int) -> None:
        """Full PEFT factors -> this rank's masters (zero for absent projections)."""
        if rank > self.R:
            raise ValueError(f"adapter rank {rank} > trainer rank {self.R}")
        self.params.zero_()
        for l in range(self.arch.num_layers):
            for g in GROUPS:
                gg = self.geom[g]
                A, Bt = self.p(l, g, "A"), self.p(l, g, "Bt")
                for p, proj in enumerate(GROUP_PROJS[g]):
                    ka, kb = peft_key(l, proj, "A"), peft_key(l, proj, "B")
                    if ka not in tensors:
                        continue
                    a = shard_lora_factor(self.arch, proj, "A", tensors[ka].float(), self.tp)
                    b = shard_lora_factor(self.arch, proj, "B", tensors[kb].float(), self.tp)
                    A[p * self.R:p * self.R + rank] = a.to(A.device)
                    rows = gg.proj_rows(p).to(Bt.device)
                    Bt[:rank, rows] = b.t().to(Bt.device)

    @torch.no_grad()
    def export_peft(self, rank: int, targets=None, grads: bool = False) -> dict[str, torch.Tensor]:
        """This rank's shard of every factor (or of its gradient), PEFT names,
        fp32 on CPU."""
        get = self.g if grads else self.p
        out = {}
        for l in range(self.arch.num_layers):
            for g in GROUPS:
                gg = self.geom[g]
                A, Bt = get(l, g, "A").cpu(), get(l, g, "Bt").cpu()
                for p, proj in enumerate(GROUP_PROJS[g]):
                    if targets is not None and proj not in targets:
                        continue
                    out[peft_key(l, proj, "A")] = A[p * self.R:p * self.R + rank].clone()
                    out[peft_key(l, proj, "B")] = Bt[:rank, gg.proj_rows(p)].t().contiguous()
        return out


@dataclass
class CycleInputs:
    n: int                        # captured tokens
    n_pad: int                    # rows processed (multiple of 8)
    starts: list[int]
    lens: list[int]
    labels: torch.Tensor          # [n_pad] int64, -1 = no loss
    cos: torch.Tensor             # [n_pad, hd/2] fp32
    sin: torch.Tensor
    # Equal-length sample groups for the batched attention backward:
    # (length, row index tensor [B*length]); built once per batch shape so the
    # backward can be captured in a CUDA graph.
    attn_groups: list | None = None


class AttnGroups(list):
    """Samples of equal length as (length, count, row index) groups, for the
    batched fp32 path, plus the tile tables of the fused attention kernels
    (built here, outside any CUDA-graph capture): ``tiles`` (64-row, the
    warp-level kernels) and ``tiles128`` (the tcgen05 kernels)."""
    tiles: torch.Tensor | None = None
    tiles128: torch.Tensor | None = None


def attention_groups(starts, lens, device) -> AttnGroups:
    groups: dict[int, list[int]] = {}
    for st, ln in zip(starts, lens):
        groups.setdefault(int(ln), []).append(int(st))
    out = AttnGroups()
    for ln, sts in groups.items():
        idx = (torch.tensor(sts, device=device)[:, None]
               + torch.arange(ln, device=device)[None, :]).reshape(-1)
        out.append((ln, len(sts), idx))
    out.tiles = ops.dense_attn_tiles(starts, lens, device)
    out.tiles128 = ops.dense_attn_tiles(starts, lens, device, bm=128)
    return out


def make_labels(ids: torch.Tensor, starts, lens, n_pad: int, mask_prefix: int = 0) -> torch.Tensor:
    """Row t of a sample predicts token t+1; the last row of a sample and its
    first ``mask_prefix`` rows carry no loss."""
    lab = torch.full((n_pad,), -1, dtype=torch.long, device=ids.device)
    for st, ln in zip(starts, lens):
        if ln < 2:
            continue
        lab[st:st + ln - 1] = ids[st + 1:st + ln]
        if mask_prefix > 0:
            lab[st:st + min(mask_prefix, ln - 1)] = -1
    return lab


def rmsnorm_fwd(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def rmsnorm_bwd(x, dy, w, eps):
    """Gradient of rmsnorm(x)*w w.r.t. x, fp32."""
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    xhat = xf * inv
    g = dy.float() * w.float()
    dot = (g * xhat).sum(-1, keepdim=True)
    return (g - xhat * dot / xf.shape[-1]) * inv


def attn_backward(qh, kh, vh, d_ctx, starts, lens, scale, groups=None):
    """Causal GQA attention backward, fp32 scores/softmax. Inputs [n, H, hd].

    Samples of equal length are processed as one batch (one set of batched
    matmuls); on CUDA the fp32 matmuls run on TF32 tensor cores, which is exact
    for the bf16-valued q/k/v/dO operands (8 of TF32's 10 mantissa bits)."""
    n, Hq, hd = qh.shape
    Hkv = kh.shape[1]
    G = Hq // Hkv
    dq = torch.zeros(n, Hq, hd, dtype=torch.float32, device=qh.device)
    dk = torch.zeros(n, Hkv, hd, dtype=torch.float32, device=qh.device)
    dv = torch.zeros_like(dk)
    if groups is None:
        groups = attention_groups(starts, lens, qh.device)
    for ln, B, idx in groups:
        def take(t, H):
            return t.index_select(0, idx).view(B, ln, H, hd).transpose(1, 2).float()  # [B, H, l, hd]
        q = take(qh, Hq)
        k = take(kh, Hkv).repeat_interleave(G, 1)
        v = take(vh, Hkv).repeat_interleave(G, 1)
        do = take(d_ctx, Hq)
        s = torch.matmul(q, k.transpose(-1, -2)) * scale
        mask = torch.triu(torch.ones(ln, ln, dtype=torch.bool, device=qh.device), 1)
        p = s.masked_fill_(mask, float("-inf")).softmax(-1)
        dvv = torch.matmul(p.transpose(-1, -2), do)
        dp = torch.matmul(do, v.transpose(-1, -2))
        ds = p * (dp - (dp * p).sum(-1, keepdim=True))
        dqq = torch.matmul(ds, k) * scale
        dkk = torch.matmul(ds.transpose(-1, -2), q) * scale
        put = lambda t, H: t.transpose(1, 2).reshape(B * ln, H, hd)
        dq.index_copy_(0, idx, put(dqq, Hq))
        dk.index_copy_(0, idx, put(dkk.view(B, Hkv, G, ln, hd).sum(2), Hkv))
        dv.index_copy_(0, idx, put(dvv.view(B, Hkv, G, ln, hd).sum(2), Hkv))
    return dq, dk, dv


def attn_forward(qh, kh, vh, starts, lens, scale, groups=None):
    """Causal GQA attention forward (fp32 scores, TF32 on CUDA), same sample
    grouping as :func:`attn_backward`. Inputs [n, H, hd]; returns [n, Hq, hd]
    fp32. Used when the attention context was not captured in the forward."""
    n, Hq, hd = qh.shape
    Hkv = kh.shape[1]
    G = Hq // Hkv
    out = torch.zeros(n, Hq, hd, dtype=torch.float32, device=qh.device)
    if groups is None:
        groups = attention_groups(starts, lens, qh.device)
    for ln, B, idx in groups:
        def take(t, H):
            return t.index_select(0, idx).view(B, ln, H, hd).transpose(1, 2).float()
        q = take(qh, Hq)
        k = take(kh, Hkv).repeat_interleave(G, 1)
        v = take(vh, Hkv).repeat_interleave(G, 1)
        s = torch.matmul(q, k.transpose(-1, -2)) * scale
        mask = torch.triu(torch.ones(ln, ln, dtype=torch.bool, device=qh.device), 1)
        o = torch.matmul(s.masked_fill_(mask, float("-inf")).softmax(-1), v)
        out.index_copy_(0, idx, o.transpose(1, 2).reshape(B * ln, Hq, hd))
    return out


# The SwiGLU backward as the epilogue of the down-projection dX GEMM
# (``EPI_SWIGLU_BWD``) or as a separate bandwidth-bound kernel after an fp32
# d(act) store. Measured on one B200 (Llama-3-8B, 4096 FT rows): fused
# 0.596 ms vs 0.442 + 0.115 ms separate — the epilogue's per-row gate/up
# reads stall the persistent GEMM more than the extra fp32 round trip costs.
FUSE_SWIGLU_BWD = False


def _bf(t, cdt):
    return t if t.dtype == cdt else t.to(cdt)


class LoraBackward:
    """Per-cycle backward state (compute copies of the LoRA factors) and the
    head / layer backward steps. Works on CPU (fp32 oracle ops) and CUDA."""

    def __init__(self, weights: ModelWeights, masters: LoraMasters, scaling: float, comm=None,
                 cdt=torch.bfloat16, served=None, ft_slot: int = -1):
        self.w, self.m, self.s = weights, masters, scaling
        # The served copy of the trained adapter (its slot of the serving LoRA
        # buffers, republished after every optimizer step): A [P*R, K] and the
        # scaled, scattered expand factor in the compute dtype, read in place
        # instead of being rebuilt from the fp32 masters for every group.
        self.served = served if (served is not None and ft_slot >= 0) else None
        self.ft_slot = ft_slot
        self.arch = weights.arch
        self.comm = comm
        self.cdt = cdt if weights.embed.is_cuda else torch.float32
        self.geom = masters.geom
        self.hq = self.arch.num_heads // weights.tp.size
        self.hkv = self.arch.num_kv_heads // weights.tp.size
        self.hd = self.arch.head_dim
        self.scale = 1.0 / math.sqrt(self.hd)
        self._rows: dict[tuple[str, int], torch.Tensor] = {}
        self._ones_slots: dict = {}
        # Backward GEMMs launch one CTA per tile so the inference stream can
        # interleave between tiles (the backward runs at low priority); with
        # an SM share (:meth:`set_sm_share`) they run persistent grids of that
        # many CTAs instead, leaving the rest of the GPU to the forward.
        self.max_ctas = 1 << 30
        self._comm_streams: dict = {}
        # Side-stream collective debugging (read once): DSERVE_BWD_COMM_SYNC=1
        # joins every side-stream all-reduce right after it is issued;
        # DSERVE_BWD_COMM_DELAY=<GPU cycles> spins the side stream before each
        # one, turning a missing reduce_end into a deterministic stale read.
        self.comm_sync = os.environ.get("DSERVE_BWD_COMM_SYNC", "0") == "1"
        self.comm_delay_cycles = int(os.environ.get("DSERVE_BWD_COMM_DELAY", "0") or 0)
        # The head's gradient pass takes the vocabulary slice in chunks of
        # this many columns (a bf16 [n, chunk] gradient block at a time).
        self.vocab_chunk = 16384
        self.scratch_rows = 0          # rows of the cycle scratch (set by prepare)
        self._astats = None            # tcgen05 attention (lse, dd) scratch
        self._head_bufs: dict | None = None
        self._head_out = None
        # Fused TP path (``parallel.peer.BwdPeerWorkspace``, set by the
        # engine): residual-gradient reductions over peer memory instead of
        # NCCL all-reduces. ``resid_bf16`` is then the current residual
        # gradient's bf16 rows (every row, gathered); the fp32 rows live in
        # ``_resid32`` (owned rows only).
        self.tpws = None
        self.resid_bf16 = None
        self._r32: list | None = None
        # Optional per-phase CUDA-event recorder (``engine.bwd_profile``):
        # ``mark(name)`` closes the phase that ends here on the current stream,
        # ``comm(name, ev0, ev1)`` brackets a collective on its side stream.
        self.timer = None

    def set_sm_share(self, percent: float, num_sms: int) -> None:
        """Cap every backward GEMM at ``percent`` of the GPU's SMs (the
        reference's ``backward_mps_percentage``, which gives its backward
        process that share of the GPU through MPS); 0 or >= 100 = no cap."""
        if percent <= 0 or percent >= 100:
            self.max_ctas = 1 << 30
        else:
            self.max_ctas = max(8, int(round(num_sms * percent / 100.0)))

    def _mark(self, name: str) -> None:
        if self.timer is not None:
            self.timer.mark(name)

    # ------------------------------------------------------------ TP sums
    def reduce_begin(self, t: torch.Tensor):
        """Start the sum of ``t`` over the TP ranks. On CUDA the all-reduce is
        issued from a side stream forked off the current one, so the kernels
        enqueued next (work that does not read ``t``) overlap it; inside a
        CUDA-graph capture this is a fork that :meth:`reduce_end` joins. The
        collectives keep one issue order on every rank."""
        if self.comm is None or self.comm.size == 1:
            return None
        if not t.is_cuda:
            self.comm.all_reduce(t)
            return None
        cs = self._comm_streams.get(t.device)
        if cs is None:
            cs = self._comm_streams[t.device] = torch.cuda.Stream(t.device)
        cs.wait_stream(torch.cuda.current_stream(t.device))
        with torch.cuda.stream(cs):
            if self.comm_delay_cycles > 0:
                # Race exposure: the collective starts late, so a consumer that
                # reads ``t`` without reduce_end reads stale data every time.
                torch.cuda._sleep(self.comm_delay_cycles)
            if self.timer is not None:
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record()
                self.comm.all_reduce(t)
                ev1.record()
                self.timer.comm(f"allreduce_{tuple(t.shape)}_{str(t.dtype)[6:]}", ev0, ev1)
            else:
                self.comm.all_reduce(t)
        if self.comm_sync:
            # Debug: join right away (the asynchronous path must match this).
            torch.cuda.current_stream(t.device).wait_stream(cs)
        return cs

    @staticmethod
    def reduce_end(handle, device) -> None:
        """Order the current stream after a :meth:`reduce_begin`."""
        if handle is not None:
            torch.cuda.current_stream(device).wait_stream(handle)

    # ------------------------------------------------------------ GEMM helpers
    def _mm(self, a, b, b_mn, epi=EPI_F32, out=None):
        a = _bf(a, self.cdt)
        b = _bf(b, self.cdt)
        if a.stride(-1) != 1:
            a = a.contiguous()
        if b.stride(-1) != 1:
            b = b.contiguous()
        if out is None:
            n = b.shape[1] if b_mn else b.shape[0]
            out = torch.empty(a.shape[0], n, dtype=torch.float32, device=a.device)
        ops.gemm(a, b, out, b_mn=b_mn, epi=epi, max_ctas=self.max_ctas)
        return out

    def rows(self, g: str, p: int, device) -> torch.Tensor:
        key = (g, p)
        t = self._rows.get(key)
        if t is None or t.device != torch.device(device):
            t = self.geom[g].proj_rows(p).to(device)
            self._rows[key] = t
        return t

    def _bfull(self, layer, g):
        """[N, P*R] scattered, scaled expand factor (compute dtype)."""
        gg = self.geom[g]
        R = self.m.R
        Bt = self.m.p(layer, g, "Bt")
        full = torch.zeros(gg.N, gg.P * R, dtype=torch.float32, device=Bt.device)
        for p in range(gg.P):
            # Strided views of the projection's rows/columns: no index tensors.
            if gg.interleave:
                full.view(gg.N // 128, 2, 64, gg.P * R)[:, p, :, p * R:(p + 1) * R] = \
                    (self._cols3(Bt, gg, p) * self.s).permute(1, 2, 0)
            else:
                b0, b1 = self._bounds(gg, p)
                full[b0:b1, p * R:(p + 1) * R] = Bt[:, b0:b1].t() * self.s
        return _bf(full, self.cdt)

    @staticmethod
    def _bounds(gg: GroupGeom, p: int) -> tuple[int, int]:
        b = [0, gg.b1, gg.b2, gg.N] if gg.P == 3 else [0, gg.N]
        return b[p], b[p + 1]

    @staticmethod
    def _cols3(t: torch.Tensor, gg: GroupGeom, p: int) -> torch.Tensor:
        """Columns of projection ``p`` (64-interleaved layout) of an [R, N]
        tensor as a writable view [R, N/128, 64]."""
        return t.view(t.shape[0], gg.N // 128, 2, 64)[:, :, p]

    def slot_A(self, layer: int, g: str) -> torch.Tensor:
        """The trained A factor [P*R, K] in the compute dtype."""
        if self.served is not None:
            return self.served.A[layer][g][self.ft_slot]
        return _bf(self.m.p(layer, g, "A"), self.cdt)

    def slot_B(self, layer: int, g: str) -> torch.Tensor:
        """The scaled, scattered expand factor [N, P*R] in the compute dtype
        (a strided view of the served slot when there is one)."""
        if self.served is not None:
            sv = self.served
            c0 = self.ft_slot * sv.seg[g]
            return sv.B2[layer][g][:, c0:c0 + self.geom[g].P * self.m.R]
        return self._bfull(layer, g)

    def group_dz(self, layer: int, g: str, dY: torch.Tensor) -> torch.Tensor:
        """dZ = dY . B_full, the adapter's share of the input gradient before
        the A factor, in the compute dtype and zero-padded to a 64-column
        segment: [n, seg] (columns P*R.. are zero) — the extra K-block of the
        fused dX GEMM and the left operand of the A gradient."""
        n = dY.shape[0]
        PR = self.geom[g].P * self.m.R
        seg = -(-PR // 64) * 64
        zp = torch.zeros(n, seg, dtype=self.cdt, device=dY.device)
        self._mm(dY, self.slot_B(layer, g), b_mn=True, epi=EPI_BF16 if self.cdt == torch.bfloat16 else EPI_F32,
                 out=zp[:, :PR])
        return zp

    def dx_gemm(self, layer: int, g: str, dY: torch.Tensor, W: torch.Tensor, dZ: torch.Tensor,
                swiglu_gu: torch.Tensor | None = None, act_out: torch.Tensor | None = None,
                bf16_out: bool = False) -> torch.Tensor:
        """dX = dY . W + dZ . A in ONE GEMM: the rank-R adapter term rides as
        one extra 64-deep K block (dZ and A zero-padded to 64) instead of a
        second pass over the fp32 dX.

        With ``swiglu_gu`` (the saved interleaved gate/up of the MLP) the
        product is d(act) and the epilogue applies the SwiGLU backward
        instead of storing it: the result is d(gate_up) in the compute dtype
        (and the activation into ``act_out`` when given)."""
        n = dY.shape[0]
        zp = dZ                       # [n, seg] from group_dz (zero-padded columns)
        seg = zp.shape[1]
        ap = self.slot_A(layer, g)    # [P*R, K]: rows seg.. of the K-block read as zero
        if not dY.is_cuda:
            out = self._mm(dY, W, b_mn=True)
            out += zp[:, :ap.shape[0]].float() @ ap.float()
            if swiglu_gu is not None:
                d_gu = torch.empty(n, swiglu_gu.shape[1], dtype=self.cdt, device=dY.device)
                ops.swiglu_bwd(swiglu_gu, out, d_gu, act_out)
                return d_gu
            return out
        key = (-(-n // 128), dY.device)
        ts = self._ones_slots.get(key)
        if ts is None:
            ts = torch.ones(key[0], dtype=torch.int32, device=dY.device)
            self._ones_slots[key] = ts
        if swiglu_gu is not None:
            out = torch.empty(n, swiglu_gu.shape[1], dtype=self.cdt, device=dY.device)
            ops.gemm(_bf(dY, self.cdt).contiguous(), _bf(W, self.cdt).contiguous(), out, b_mn=True,
                     epi=EPI_SWIGLU_BWD, z=zp, b2=ap, tile_slots=ts, lora_seg=seg, max_ctas=self.max_ctas,
                     aux=swiglu_gu, aux_out=act_out)
            return out
        out = torch.empty(n, W.shape[1], dtype=torch.bfloat16 if bf16_out else torch.float32, device=dY.device)
        ops.gemm(_bf(dY, self.cdt).contiguous(), _bf(W, self.cdt).contiguous(), out, b_mn=True,
                 epi=EPI_BF16 if bf16_out else EPI_F32, z=zp, b2=ap, tile_slots=ts, lora_seg=seg,
                 max_ctas=self.max_ctas)
        return out

    def prepare(self, n: int, device, max_rows: int = 0) -> None:
        """Allocate the cycle scratch (once, for ``max_rows`` rows: the capture
        buffer's size) before any CUDA-graph capture, so no scratch lives in a
        graph pool and every shape's graphs see the same buffers."""
        self.scratch_rows = max(self.scratch_rows, int(max_rows))
        if self.w.embed.is_cuda:
            self._head_scratch(n, device)
            if ops.ATTN_TC:
                self.attn_stats(n, device)
            if self.tpws is not None:
                self._resid32(n, device)

    def _tile_ones(self, n: int, device) -> torch.Tensor:
        key = (-(-n // 128), device)
        ts = self._ones_slots.get(key)
        if ts is None:
            ts = torch.ones(key[0], dtype=torch.int32, device=device)
            self._ones_slots[key] = ts
        return ts

    def push_dx(self, layer: int, g: str, dY: torch.Tensor, W: torch.Tensor, dZ: torch.Tensor) -> None:
        """The fused TP form of :meth:`dx_gemm`: ``dY . W + dZ . A`` in one
        GEMM whose epilogue pushes each 128-row block's bf16 partial to the
        block's owner rank (completed by ``ops.tp_reduce_rows``)."""
        ap = self.slot_A(layer, g)
        ops.gemm_push(_bf(dY, self.cdt).contiguous(), _bf(W, self.cdt).contiguous(), self.tpws, z=dZ, b2=ap,
                      tile_slots=self._tile_ones(dY.shape[0], dY.device), lora_seg=dZ.shape[1],
                      max_ctas=self.max_ctas)

    def group_grads(self, layer: int, g: str, X: torch.Tensor, dY: torch.Tensor, dZ: torch.Tensor) -> None:
        """Factor gradients of one group into the trainer's grad buffer, three
        GEMMs over the token dimension:

        * ``Z = X A^T`` [n, P*R];
        * ``dA = dZ^T X`` — written transposed by the GEMM (token-major
          operands, no transposed copies);
        * ``dB_p^T = s Z_p^T dY`` for every projection p at once: output
          feature m keeps its own projection's R columns, scaled."""
        gg = self.geom[g]
        R = self.m.R
        PR = gg.P * R
        A = self.slot_A(layer, g)
        n = X.shape[0]
        Z = torch.empty(n, PR, dtype=self.cdt, device=X.device)
        self._mm(X, A, b_mn=False, epi=EPI_BF16 if self.cdt == torch.bfloat16 else EPI_F32, out=Z)
        Xc, dYc = _bf(X, self.cdt), _bf(dY, self.cdt)
        ops.gemm_wgrad(Xc if Xc.stride(-1) == 1 else Xc.contiguous(), dZ, self.m.g(layer, g, "A"),
                       kind="t", n_valid=PR, max_ctas=self.max_ctas)
        b1, b2 = (gg.b1, gg.b2) if gg.P == 3 else (gg.N, gg.N)
        ops.gemm_wgrad(dYc if dYc.stride(-1) == 1 else dYc.contiguous(), Z, self.m.g(layer, g, "Bt"),
                       kind="bt", n_valid=PR, R=R, b1=b1, b2=b2, interleave=gg.interleave, scale=self.s,
                       max_ctas=self.max_ctas)

    def group_backward(self, layer: int, g: str, X: torch.Tensor, dY: torch.Tensor,
                       dX: torch.Tensor) -> None:
        """LoRA part of one group on its own: accumulates dZ . A into ``dX``
        (fp32) and writes the factor gradients (the layer backward uses the
        fused :meth:`dx_gemm` instead)."""
        dZ = self.group_dz(layer, g, dY)
        A = self.slot_A(layer, g)
        self._mm(dZ[:, :A.shape[0]], A, b_mn=True, epi=EPI_F32_ACCUM, out=dX)
        self.group_grads(layer, g, X, dY, dZ)

    # ------------------------------------------------------------ head
    def head_chunks(self) -> list[tuple[int, int]]:
        """Column ranges of this rank's vocabulary slice that the head's
        gradient pass takes one at a time (bounds the bf16 gradient block)."""
        V = self.w.lm_head.shape[0]
        return [(c, min(V, c + self.vocab_chunk)) for c in range(0, V, self.vocab_chunk)]

    def _head_scratch(self, n: int, device) -> dict:
        """The head's scratch for ``n`` rows: views of buffers allocated once
        for :attr:`scratch_rows` rows. Captured CUDA graphs keep the buffers'
        addresses, so they are never reallocated while the trainer lives."""
        if self._head_bufs is None or n > self._head_bufs["rows"]:
            # (the trainer prepares the capture capacity before capturing any
            # graph, so only callers without graphs ever grow the scratch)
            rows = max(n, self.scratch_rows)
            V, D = self.w.lm_head.shape
            ch = min(V, self.vocab_chunk)
            world = self.comm.size if self.comm is not None else 1
            f32 = dict(dtype=torch.float32, device=device)
            self._head_bufs = {"rows": rows, "world": world,
                               "stats": torch.empty(rows, 2 * (-(-V // 64)), **f32), "tgt": torch.empty(rows, **f32),
                               "part": torch.empty(rows, 3, **f32), "parts": torch.empty(world * rows * 3, **f32),
                               "lse": torch.empty(rows, **f32), "loss": torch.empty(rows, **f32),
                               "dlog": torch.empty(rows, ch, dtype=self.cdt, device=device),
                               "dh": torch.empty(rows, D, **f32)}
        b = self._head_bufs
        return {"stats": b["stats"][:n], "tgt": b["tgt"][:n], "part": b["part"][:n],
                "parts": b["parts"][:b["world"] * n * 3].view(b["world"], n, 3),
                "lse": b["lse"][:n], "loss": b["loss"][:n], "dlog": b["dlog"][:n], "dh": b["dh"][:n]}

    def head_backward(self, final_in: torch.Tensor, labels: torch.Tensor,
                      n_valid: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Final RMSNorm + LM head + cross-entropy on this rank's slice of the
        vocabulary (the serving head's shard: rows ``[rank * V_l, (rank + 1) * V_l)``).

        1. statistics pass: one GEMM whose epilogue keeps, per row and tile,
           the max logit and the sum of exponentials (and the label's logit),
           merged per row; under TP the ranks' (max, sum, label logit) rows are
           gathered (one small collective) into the row's log-sum-exp;
        2. gradient pass, per vocabulary chunk: the GEMM recomputes the
           logits and its epilogue writes ``(softmax - onehot) / n_valid`` in
           bf16; ``dh += dlog_chunk @ W_chunk`` (fp32);
        3. ``dh`` is this rank's partial over its slice: summed over the
           ranks, then the final-norm backward.

        No [n, V] logit tensor exists at any point (the reference's head,
        ``bwd_services/common/head.py:31-100``, materialises fp32 logits).
        Returns (summed loss as a 0-d device tensor, d final_in fp32); the
        loss is the sum over the ``n_valid`` labelled rows and the gradient is
        already divided by ``n_valid``. Under the fused TP path the returned
        gradient holds this rank's owned rows (the rest lives in
        :attr:`resid_bf16`)."""
        for _ in self.head_steps(final_in, labels, n_valid):
            pass
        return self._head_out

    def head_steps(self, final_in: torch.Tensor, labels: torch.Tensor, n_valid: int):
        """:meth:`head_backward` as a generator that yields between its
        pieces (statistics, then every vocabulary chunk): the trainer's pause
        boundaries inside the head. The result is left in ``_head_out``."""
        w = self.w
        eps = self.arch.rms_eps
        head = w.lm_head
        dev = final_in.device
        n, D = final_in.shape
        world = self.comm.size if self.comm is not None else 1
        v0 = (self.comm.rank if self.comm is not None else 0) * head.shape[0]
        if final_in.is_cuda:    # the norm kernels (bf16 out, fp32 inside)
            h = torch.empty(final_in.shape, dtype=self.cdt, device=dev)
            ops.rms_norm(final_in, w.final_norm, h, eps)
        else:
            h = rmsnorm_fwd(final_in, w.final_norm, eps)
        if n_valid == 0:
            self._head_out = (torch.zeros((), device=dev), torch.zeros(n, D, dtype=torch.float32, device=dev))
            self.resid_bf16 = None
            return
        h = _bf(h, self.cdt).contiguous()
        headc = _bf(head, self.cdt)
        st = self._head_scratch(n, dev)
        self._mark("head_norm")
        st["tgt"].zero_()
        tiles = ops.ce_stats(h, headc, labels, v0, st["stats"], st["tgt"], max_ctas=self.max_ctas)
        ops.ce_merge(st["stats"], tiles, st["tgt"], st["part"])
        if world > 1:
            self.comm.all_gather_into(st["parts"], st["part"])
            parts = st["parts"]
        else:
            parts = st["part"].view(1, n, 3)
        ops.ce_finalize(parts, labels, st["lse"], st["loss"])
        self._mark("head_stats")
        yield "head_stats"
        chunks = self.head_chunks()
        fused = self.tpws is not None and final_in.is_cuda
        dh = st["dh"]
        for i, (c0, c1) in enumerate(chunks):
            dlog = st["dlog"][:, :c1 - c0]
            ops.ce_grad(h, headc[c0:c1], labels, v0 + c0, st["lse"], 1.0 / n_valid, dlog, max_ctas=self.max_ctas)
            last = i == len(chunks) - 1
            if fused and last:
                # The last chunk's product goes straight to the row owners
                # (with the earlier chunks' fp32 sum added), then the owner
                # applies the final-norm backward and all-gathers the rows.
                ops.gemm_push(dlog, headc[c0:c1], self.tpws, add=dh if i > 0 else None, max_ctas=self.max_ctas)
            else:
                ops.gemm(dlog, headc[c0:c1], dh, b_mn=True, epi=EPI_F32 if i == 0 else EPI_F32_ACCUM,
                         max_ctas=self.max_ctas)
            self._mark("head_grad")
            if not last:
                yield "head_chunk"
        loss = st["loss"].sum()
        if fused:
            r32 = self._resid32(n, dev)[1]
            self.resid_bf16 = ops.tp_reduce_rows(self.tpws, n, 1, r32, x=final_in, w=w.final_norm, eps=eps)
            d_final = r32
        else:
            if world > 1:
                self.comm.all_reduce(dh)
            if final_in.is_cuda:
                d_final = ops.rms_norm_bwd(final_in, dh, w.final_norm, eps)
            else:
                d_final = rmsnorm_bwd(final_in, dh, w.final_norm, eps)
            self.resid_bf16 = None
        self._mark("head_norm")
        self._head_out = (loss, d_final)

    def _resid32(self, n: int, device) -> list[torch.Tensor]:
        """The fused TP path's two fp32 residual-gradient buffers [n, D]
        (only this rank's owned rows are ever written or read): views of two
        buffers allocated once for :attr:`scratch_rows` rows."""
        if self._r32 is None or n > self._r32[0].shape[0]:
            rows = max(n, self.scratch_rows)
            self._r32 = [torch.zeros(rows, self.arch.hidden, dtype=torch.float32, device=device) for _ in range(2)]
        return [t[:n] for t in self._r32]

    @staticmethod
    def tc_attention(t: torch.Tensor) -> bool:
        """Whether the attention of tensors like ``t`` runs on the tcgen05 kernels."""
        return ops.ATTN_TC and t.is_cuda

    def attn_stats(self, n: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        """(lse, dd) fp32 [Hq, rows] scratch of the tcgen05 attention: the
        forward's row log-sum-exp and the backward's rowsum(dO * O), indexed
        by packed row (allocated once for :attr:`scratch_rows` rows, so every
        captured graph sees the same buffers)."""
        if self._astats is None or n > self._astats[0].shape[1]:
            rows = max(n, self.scratch_rows)
            self._astats = (torch.zeros(self.hq, rows, dtype=torch.float32, device=device),
                            torch.zeros(self.hq, rows, dtype=torch.float32, device=device))
        return self._astats

    # ------------------------------------------------------------ recompute
    def _proj_lora(self, layer: int, g: str, X: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
        """fp32 ``X @ W^T`` plus the trained adapter's term for group ``g``
        (the forward's projection, for activations that were not captured)."""
        y = self._mm(X, W, b_mn=False)
        Z = self._mm(X, self.slot_A(layer, g), b_mn=False)
        self._mm(Z, self.slot_B(layer, g), b_mn=False, epi=EPI_F32_ACCUM, out=y)
        return y

    def recompute_qkv_raw(self, layer: int, layer_in: torch.Tensor) -> torch.Tensor:
        lw = self.w.layers[layer]
        x1 = torch.empty_like(layer_in)
        ops.rms_norm(layer_in, lw.in_ln, x1, self.arch.rms_eps)
        return self._proj_lora(layer, "qkv", x1, lw.qkv).to(layer_in.dtype)

    def recompute_ctx(self, layer: int, qkv_raw: torch.Tensor, ci, positions, cos_sin,
                      lse: torch.Tensor | None = None) -> torch.Tensor:
        """The attention output of the layer; with ``lse`` (and the tcgen05
        kernels) also its base-2 row log-sum-exp, which the attention
        backward then reuses instead of recomputing the forward."""
        qh, kh, vh = self.recompute_qkv(qkv_raw, positions, self.w.layers[layer], cos_sin)
        if qh.is_cuda:
            out = torch.zeros(qh.shape[0], self.hq * self.hd, dtype=qkv_raw.dtype, device=qh.device)
            t128 = self._tiles128(ci) if ops.ATTN_TC else None
            return ops.attn_fwd_dense(qh, kh, vh, self._tiles(ci), self.scale, out, tiles128=t128,
                                      lse=lse if t128 is not None else None)
        o = attn_forward(qh, kh, vh, ci.starts, ci.lens, self.scale, ci.attn_groups)
        return o.reshape(qh.shape[0], -1).to(qkv_raw.dtype)

    def _tiles(self, ci) -> torch.Tensor:
        g = ci.attn_groups
        if g is None or getattr(g, "tiles", None) is None:
            return ops.dense_attn_tiles(ci.starts, ci.lens, self.w.embed.device)
        return g.tiles

    def _tiles128(self, ci) -> torch.Tensor:
        g = ci.attn_groups
        if g is None or getattr(g, "tiles128", None) is None:
            return ops.dense_attn_tiles(ci.starts, ci.lens, self.w.embed.device, bm=128)
        return g.tiles128

    def recompute_resid_mid(self, layer: int, layer_in: torch.Tensor, ctx: torch.Tensor) -> torch.Tensor:
        o = self._proj_lora(layer, "o", ctx, self.w.layers[layer].o)
        if self.comm is not None:
            self.comm.all_reduce(o)        # row-parallel: partial sums
        return (layer_in.float() + o).to(layer_in.dtype)

    # ------------------------------------------------------------ layer
    def recompute_qkv(self, qkv_raw: torch.Tensor, positions: torch.Tensor, lw, cos_sin):
        """Post-norm/RoPE q, k (as the serving kernel produced them) and v."""
        t = qkv_raw.clone()
        ops.qk_norm_rope_cache(t, positions, cos_sin, lw.q_norm, lw.k_norm, self.arch.rms_eps,
                               self.hq, self.hkv)
        n = t.shape[0]
        ql, kl = self.hq * self.hd, self.hkv * self.hd
        return (t[:, :ql].view(n, self.hq, self.hd), t[:, ql:ql + kl].view(n, self.hkv, self.hd),
                t[:, ql + kl:].view(n, self.hkv, self.hd))

    def layer_backward(self, layer: int, dh: torch.Tensor, saved: dict, ci: CycleInputs,
                       positions: torch.Tensor, cos_sin: torch.Tensor,
                       need_input_grad: bool = True) -> torch.Tensor:
        """dh: fp32 [n, D] gradient w.r.t. the layer output. Returns the gradient
        w.r.t. the layer input (fp32); this layer's factor gradients are written.
        With ``need_input_grad`` False (the first layer: nothing below it is
        trained) the input gradient is not computed and ``dh`` comes back.

        Under TP the two residual-stream gradients (after the MLP and after
        the qkv input gradient) are per-rank partials. With the fused path
        (:attr:`tpws`) each dX GEMM pushes its bf16 partial rows to their
        owner rank, the owner sums them and applies the RMSNorm backward
        (plus the residual gradient) for its rows, and the bf16 rows are
        all-gathered — the reference's ``reduce_partial`` all-reduces
        (``bwd_services/llama3.py:178-180, 210-211``) as GEMM ->
        reduce-scatter -> norm -> all-gather over NVLink; the factor-gradient
        GEMMs run while the partials travel. Otherwise ``comm.all_reduce``
        sums them on a side stream."""
        w = self.w
        lw = w.layers[layer]
        eps = self.arch.rms_eps
        x, qkv_raw, ctx = saved["layer_in"], saved["qkv"], saved["ctx"]
        resid_mid, gate_up, act = saved["resid_mid"], saved["gate_up"], saved.get("act")
        n, D = x.shape
        dev = x.device
        cdt = self.cdt
        fused = self.tpws is not None and x.is_cuda
        # ---- MLP -------------------------------------------------------
        dh_c = self.resid_bf16 if fused else _bf(dh, cdt)
        dz = self.group_dz(layer, "down", dh_c)
        # d(act) = dh . W_down (+ adapter), then the SwiGLU backward gives
        # d(gate_up) (and the activation when it was not captured).
        act_out = None
        if act is None:
            act_out = torch.empty(n, gate_up.shape[1] // 2, dtype=x.dtype, device=dev)
        if FUSE_SWIGLU_BWD:
            d_gu = self.dx_gemm(layer, "down", dh_c, lw.down, dz, swiglu_gu=gate_up, act_out=act_out)
        else:
            d_act = self.dx_gemm(layer, "down", dh_c, lw.down, dz)     # [n, I_l] fp32
            d_gu = torch.empty(n, gate_up.shape[1], dtype=cdt, device=dev)
            ops.swiglu_bwd(gate_up, d_act, d_gu, act_out)
        if act is None:
            act = act_out
        dz_down = dz
        x2 = torch.empty(n, D, dtype=x.dtype, device=dev)
        ops.rms_norm(resid_mid, lw.post_ln, x2, eps)
        dz = self.group_dz(layer, "gate_up", d_gu)
        if fused:
            self.push_dx(layer, "gate_up", d_gu, lw.gate_up, dz)
            self._mark("mlp_dx")
            self.group_grads(layer, "down", act, dh_c, dz_down)
            self.group_grads(layer, "gate_up", x2, d_gu, dz)
            self._mark("mlp_factor_grads")
            r32 = self._resid32(n, dev)
            d_mid_c = ops.tp_reduce_rows(self.tpws, n, 0, r32[0], x=resid_mid, w=lw.post_ln, eps=eps, add=dh)
            d_mid = r32[0]
            self._mark("reduce_norm_mid")
        else:
            d_x2 = self.dx_gemm(layer, "gate_up", d_gu, lw.gate_up, dz)  # [n, D]
            self._mark("mlp_dx")
            # The TP sum of d_x2 runs while the factor gradients (which do not
            # read it) are computed.
            h = self.reduce_begin(d_x2)
            self.group_grads(layer, "down", act, dh_c, dz_down)
            self.group_grads(layer, "gate_up", x2, d_gu, dz)
            self._mark("mlp_factor_grads")
            self.reduce_end(h, dev)
            self._mark("wait_reduce_mid")
            d_mid_c = torch.empty(n, D, dtype=cdt, device=dev)
            d_mid = ops.rms_norm_bwd(resid_mid, d_x2, lw.post_ln, eps, add=dh, out_bf16=d_mid_c)
            self._mark("norm_bwd_mid")
        # ---- attention ---------------------------------------------------
        dz_o = self.group_dz(layer, "o", d_mid_c)
        tc_attn = self.tc_attention(x)
        d_ctx = self.dx_gemm(layer, "o", d_mid_c, lw.o, dz_o, bf16_out=tc_attn)      # [n, q_l]
        self._mark("o_dx")
        qh, kh, vh = self.recompute_qkv(qkv_raw, positions, lw, cos_sin)
        ql, kl = self.hq * self.hd, self.hkv * self.hd
        d_qkv = torch.empty(n, ql + 2 * kl, dtype=cdt, device=dev)
        if qh.is_cuda:
            # Fused flash-style backward; its epilogues undo RoPE and store
            # bf16 straight into d(qkv) (dq / dk stay fp32 for the Qwen3 q/k
            # norm backward). Rows past the samples carry no gradient.
            d_qkv[ci.n:].zero_()
            mask = 4 if self.arch.qk_norm else 7
            if tc_attn:
                lse, dd = self.attn_stats(n, dev)
                have_lse = saved.get("lse") is not None
                dq, dk, dv = ops.attn_bwd(qh, kh, vh, d_ctx, self._tiles(ci), self.scale, rope=(ci.cos, ci.sin),
                                          dqkv=d_qkv, bf16_mask=mask, o=ctx if have_lse else None,
                                          lse=lse if have_lse else None, tiles128=self._tiles128(ci), dd=dd)
            else:
                dq, dk, dv = ops.attn_bwd(qh, kh, vh, d_ctx, self._tiles(ci), self.scale, rope=(ci.cos, ci.sin),
                                          dqkv=d_qkv, bf16_mask=mask)
        else:
            dq, dk, dv = attn_backward(qh, kh, vh, d_ctx.view(n, self.hq, self.hd), ci.starts, ci.lens,
                                       self.scale, ci.attn_groups)
            dq = rope_backward(dq, ci.cos, ci.sin)
            dk = rope_backward(dk, ci.cos, ci.sin)
            d_qkv[:, ql + kl:] = dv.reshape(n, kl)
            if not self.arch.qk_norm:
                d_qkv[:, :ql] = dq.reshape(n, ql)
                d_qkv[:, ql:ql + kl] = dk.reshape(n, kl)
        if self.arch.qk_norm:
            q_pre = qkv_raw[:, :ql].reshape(n * self.hq, self.hd)
            k_pre = qkv_raw[:, ql:ql + kl].reshape(n * self.hkv, self.hd)
            dqn = ops.rms_norm_bwd(q_pre, dq.reshape(n * self.hq, self.hd), lw.q_norm, eps)
            dkn = ops.rms_norm_bwd(k_pre, dk.reshape(n * self.hkv, self.hd), lw.k_norm, eps)
            d_qkv[:, :ql] = dqn.view(n, ql)
            d_qkv[:, ql:ql + kl] = dkn.view(n, kl)
        self._mark("attention")
        x1 = torch.empty(n, D, dtype=x.dtype, device=dev)
        ops.rms_norm(x, lw.in_ln, x1, eps)
        dz = self.group_dz(layer, "qkv", d_qkv)
        if not need_input_grad:
            self.group_grads(layer, "o", ctx, d_mid_c, dz_o)
            self.group_grads(layer, "qkv", x1, d_qkv, dz)
            self._mark("attn_factor_grads")
            return dh
        if fused:
            self.push_dx(layer, "qkv", d_qkv, lw.qkv, dz)
            self._mark("qkv_dx")
            self.group_grads(layer, "o", ctx, d_mid_c, dz_o)
            self.group_grads(layer, "qkv", x1, d_qkv, dz)
            self._mark("attn_factor_grads")
            r32 = self._resid32(n, dev)
            self.resid_bf16 = ops.tp_reduce_rows(self.tpws, n, 1, r32[1], x=x, w=lw.in_ln, eps=eps, add=d_mid)
            self._mark("reduce_norm_x")
            return r32[1]
        d_x1 = self.dx_gemm(layer, "qkv", d_qkv, lw.qkv, dz)       # [n, D]
        self._mark("qkv_dx")
        h = self.reduce_begin(d_x1)
        self.group_grads(layer, "o", ctx, d_mid_c, dz_o)
        self.group_grads(layer, "qkv", x1, d_qkv, dz)
        self._mark("attn_factor_grads")
        self.reduce_end(h, dev)
        self._mark("wait_reduce_x")
        out = ops.rms_norm_bwd(x, d_x1, lw.in_ln, eps, add=d_mid)
        self._mark("norm_bwd_x")
        return out
