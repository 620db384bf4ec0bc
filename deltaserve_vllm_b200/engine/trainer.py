"""LoRA trainer that runs inside the serving process.

One backward *cycle* trains on the activations of one filled capture buffer:

1. head backward (final norm + LM head + CE, fp32 logits);
2. layers L-1 .. 0: hand-written layer backward (``models/lora_backward.py``);
   under TP the replicated factor gradients of every 8 layers are summed with
   one all-reduce of a contiguous slab (the reference buckets the same way,
   ``bwd_services/common/tp.py:186-236``);
3. per-layer gradient clipping to norm 1.0 (rank-symmetric under TP), AdamW on
   the flat fp32 masters (two launches), StepLR decay per epoch;
4. publish: bf16 ``A`` and ``B * alpha/r`` written straight into the served
   LoRA slot (``ops.lora_publish``), so inference uses the new weights from the
   next step.

The cycle is a generator that yields at every layer boundary: the engine
decides between yields whether to keep enqueueing backward work (pause on
request arrival, run-ahead bound) — the reference's pause contract
(``bwd_services/base.py:148-208``) without a second process.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import torch

from .. import dprint, ops
from ..adapters import peft_io
from ..models.decoder import CaptureBuffers
from ..models.lora import GROUPS, LoraServeBuffers, random_adapter
from ..models.lora_backward import CycleInputs, LoraBackward, LoraMasters, make_labels
from ..models.rope import cos_sin as rope_cos_sin
from ..models.weights import ModelWeights

BUCKET_LAYERS = 8
CLIP_NORM = 1.0


@dataclass
class CycleResult:
    loss: float
    n_tokens: int
    n_valid: int
    gpu_ms: float
    wall_ms: float
    step: int


class LoraTrainer:
    def __init__(self, weights: ModelWeights, served: LoraServeBuffers | None, ft_slot: int,
                 rank: int, alpha: float, lr: float = 1e-4, weight_decay: float = 0.0,
                 gamma: float = 1.0, comm=None, mask_prefix: int = 0, targets=None,
                 adapter_config: dict | None = None, cos_sin_table: torch.Tensor | None = None):
        self.w = weights
        self.arch = weights.arch
        self.served = served
        self.ft_slot = ft_slot
        self.rank_r = rank
        self.alpha = alpha
        self.scaling = alpha / rank
        self.comm = comm
        self.lr, self.wd, self.gamma = lr, weight_decay, gamma
        self.mask_prefix = mask_prefix
        self.targets = tuple(targets) if targets else None
        dev = weights.embed.device
        R = served.R if served is not None else rank
        self.masters = LoraMasters(self.arch, weights.tp, R, dev)
        self.bwd = LoraBackward(weights, self.masters, self.scaling, comm)
        self.adapter_config = adapter_config or peft_io.default_adapter_config(
            rank, alpha, self.targets or ("q", "k", "v", "o", "gate", "up", "down"))
        self.cos_sin = cos_sin_table
        self.step = 0
        self.epoch = 0
        self.total_tokens = 0
        self.losses: list[float] = []
        L = self.arch.num_layers
        self._sq_rep = torch.zeros(L, dtype=torch.float32, device=dev)
        self._sq_shard = torch.zeros(L, dtype=torch.float32, device=dev)

    # ------------------------------------------------------------ adapter state
    def load_adapter(self, tensors: dict[str, torch.Tensor], rank: int, alpha: float) -> None:
        """Copy a PEFT adapter into the existing masters (buffers keep their
        addresses, so captured graphs and tensor maps stay valid); optimizer
        state restarts."""
        self.rank_r, self.alpha = rank, alpha
        self.scaling = alpha / rank
        self.bwd.s = self.scaling
        self.masters.load_peft(tensors, rank)
        self.masters.exp_avg.zero_()
        self.masters.exp_avg_sq.zero_()
        self.step = 0

    def init_random(self, seed: int = 0) -> None:
        """PEFT-style init for a fresh adapter: A kaiming-uniform, B zero."""
        t = random_adapter(self.arch, self.rank_r, seed, targets=self.targets or
                           ("q", "k", "v", "o", "gate", "up", "down"), b_std=0.0)
        self.load_adapter(t, self.rank_r, self.alpha)

    @torch.no_grad()
    def publish(self) -> None:
        if self.served is None or self.ft_slot < 0:
            return
        sv = self.served
        for l in range(self.arch.num_layers):
            for g in GROUPS:
                gg = sv.geom[g]
                ops.lora_publish(self.masters.p(l, g, "A"), sv.A[l][g][self.ft_slot],
                                 self.masters.p(l, g, "Bt"), sv.B2[l][g],
                                 self.ft_slot * sv.seg[g], gg.b1, gg.b2, gg.interleave,
                                 self.scaling)
        sv.slot_rank[self.ft_slot] = self.rank_r

    # ------------------------------------------------------------ one cycle
    def _cycle_inputs(self, cap: CaptureBuffers, n: int, starts, lens) -> CycleInputs:
        n_pad = max(8, -(-n // 8) * 8)
        if n_pad > cap.layer_in.shape[1]:
            raise ValueError("capture buffer too small for the padded cycle")
        if n_pad > n:  # padded rows must be zero (they carry no sample)
            for t in (cap.layer_in, cap.qkv, cap.ctx, cap.resid_mid, cap.gate_up):
                t[:, n:n_pad].zero_()
            cap.final_in[n:n_pad].zero_()
            cap.ids[n:n_pad].zero_()
            cap.positions[n:n_pad].zero_()
        labels = make_labels(cap.ids[:n_pad], starts, lens, n_pad, self.mask_prefix)
        c, s = rope_cos_sin(cap.positions[:n_pad], self.arch.head_dim, self.arch.rope_theta,
                            self.arch.rope_scaling)
        return CycleInputs(n, n_pad, list(starts), list(lens), labels, c, s)

    def n_valid(self, lens) -> int:
        """Rows that carry a label (host-side, no device sync)."""
        return sum(max(0, ln - 1 - min(self.mask_prefix, max(0, ln - 1))) for ln in lens)

    def cycle(self, cap: CaptureBuffers, n: int, starts, lens, epoch: int | None = None,
              sync: bool = True):
        """Generator: yields at each pause boundary; its return value (via
        StopIteration.value) is a pending :class:`CycleResult` — with
        ``sync=False`` the loss and GPU time are resolved later by
        :meth:`finish_cycle`, so the host never waits on the backward."""
        t_wall = time.perf_counter()
        dev = self.masters.params.device
        ev0 = ev1 = None
        if dev.type == "cuda":
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        ci = self._cycle_inputs(cap, n, starts, lens)
        m = self.masters
        m.grads.zero_()
        n_valid = self.n_valid(lens)
        loss_sum, dh = self.bwd.head_backward(cap.final_in[:ci.n_pad], ci.labels, n_valid)
        yield "head"
        L = self.arch.num_layers
        cs = self.cos_sin
        pos = cap.positions[:ci.n_pad]
        pending = []
        for l in range(L - 1, -1, -1):
            saved = {k: getattr(cap, k)[l, :ci.n_pad] for k in
                     ("layer_in", "qkv", "ctx", "resid_mid", "gate_up")}
            dh = self.bwd.layer_backward(l, dh, saved, ci, pos, cs)
            if self.comm is not None and self.comm.size > 1 and (l % BUCKET_LAYERS == 0):
                # Layers [l, l + BUCKET_LAYERS) are done: one all-reduce of their
                # replicated factor gradients.
                self.comm.all_reduce(m.rep_block(m.grads, l, min(L, l + BUCKET_LAYERS)))
            yield l
        self._optimizer_step(epoch)
        self.publish()
        if ev1 is not None:
            ev1.record()
        res = CycleResult(0.0, n, n_valid, 0.0, 0.0, self.step)
        res._pending = (loss_sum, ev0, ev1, t_wall)
        return self.finish_cycle(res) if sync else res

    def finish_cycle(self, res: CycleResult) -> CycleResult:
        """Resolve a cycle's loss and GPU time (waits for its end event)."""
        pend = getattr(res, "_pending", None)
        if pend is None:
            return res
        loss_sum, ev0, ev1, t_wall = pend
        if ev1 is not None:
            ev1.synchronize()
            res.gpu_ms = ev0.elapsed_time(ev1)
        else:
            res.gpu_ms = (time.perf_counter() - t_wall) * 1e3
        res.wall_ms = (time.perf_counter() - t_wall) * 1e3
        res.loss = float(loss_sum) / max(1, res.n_valid) if res.n_valid else 0.0
        res._pending = None
        self.total_tokens += res.n_tokens
        self.losses.append(res.loss)
        if not math.isfinite(res.loss):
            dprint(f"[trainer] WARNING: non-finite loss at step {self.step}; training continues")
        return res

    def run_cycle(self, cap, n, starts, lens, epoch=None) -> CycleResult:
        g = self.cycle(cap, n, starts, lens, epoch)
        while True:
            try:
                next(g)
            except StopIteration as e:
                return e.value

    @torch.no_grad()
    def _optimizer_step(self, epoch: int | None) -> None:
        m = self.masters
        if epoch is not None and epoch > self.epoch:
            self.epoch = epoch
        lr = self.lr * (self.gamma ** self.epoch)
        self.step += 1
        ops.seg_sumsq(m.rep_block(m.grads), m.rep_per_layer, self._sq_rep)
        ops.seg_sumsq(m.shard_block(m.grads), m.shard_per_layer, self._sq_shard)
        if self.comm is not None and self.comm.size > 1:
            self.comm.all_reduce(self._sq_shard)
        total = self._sq_rep + self._sq_shard
        for blk, seg in ((m.rep_block, m.rep_per_layer), (m.shard_block, m.shard_per_layer)):
            ops.adamw(blk(m.params), blk(m.grads), blk(m.exp_avg), blk(m.exp_avg_sq), seg_len=seg,
                      seg_sumsq_t=total, max_norm=CLIP_NORM, grad_scale=1.0, lr=lr, wd=self.wd,
                      step=self.step)

    # ------------------------------------------------------------ checkpoints
    def export_full(self) -> dict[str, torch.Tensor] | None:
        """Full (TP-merged) PEFT tensors on rank 0, None on other ranks."""
        mine = self.masters.export_peft(self.rank_r, self.targets)
        if self.comm is None or self.comm.size == 1:
            return mine
        shards = self.comm.gather_objects(mine)
        return peft_io.merge_tp_shards(shards) if shards is not None else None

    def save_adapter(self, path: str, save_id: str = "", extra: dict | None = None) -> str | None:
        full = self.export_full()
        if full is None:
            return None
        state = {"save_id": save_id, "step": self.step, "epoch": self.epoch,
                 "total_tokens": self.total_tokens, "time": time.time(),
                 "last_loss": self.losses[-1] if self.losses else None, **(extra or {})}
        peft_io.write_peft_adapter(path, full, dict(self.adapter_config), state)
        return path
