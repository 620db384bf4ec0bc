"""LoRA trainer that runs inside the serving process.

One backward *cycle* trains on the activations of one filled capture buffer:

1. head backward (final norm + vocabulary-parallel LM head + cross-entropy,
   statistics then gradient per vocabulary chunk, no logits stored);
2. layers L-1 .. 0: hand-written layer backward (``models/lora_backward.py``);
   under TP the replicated factor gradients of every 8 layers (a contiguous
   slab; the reference buckets the same way, ``bwd_services/common/tp.py:186-236``)
   are pushed to their slice owners over peer memory while the next layer's
   backward runs (or, on the NCCL path, all-reduced from a side stream);
3. per-layer gradient clipping to norm 1.0 (rank-symmetric under TP) and
   AdamW on the flat fp32 masters; on the fused path each owner sums, clips
   and updates its slice of the replicated factors and sends the new values
   to every rank (``ops.fused_replicated_adamw``); StepLR decay per epoch;
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
import os
import time
from dataclasses import dataclass

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


def _copy_unless_same(dst: torch.Tensor, src: torch.Tensor) -> None:
    if src.data_ptr() != dst.data_ptr():
        dst.copy_(src)


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
        self.bwd = LoraBackward(weights, self.masters, self.scaling, comm, served=served, ft_slot=ft_slot)
        self.adapter_config = adapter_config or peft_io.default_adapter_config(
            rank, alpha, self.targets or ("q", "k", "v", "o", "gate", "up", "down"))
        self.cos_sin = cos_sin_table
        self.step = 0
        self.epoch = 0
        self.total_tokens = 0
        self._writer = None          # background checkpoint writer (one thread)
        self._pending_save = None
        self.losses: list[float] = []
        L = self.arch.num_layers
        # Captured per-layer backward graphs, keyed by the batch shape.
        self.use_graphs = dev.type == "cuda"
        self.max_graph_shapes = 4
        self._graphs: dict = {}
        self._groups_cache: dict = {}
        self._pool = None
        self._cap_stream = None
        self._seen_shapes: set = set()
        self._sq_rep = torch.zeros(L, dtype=torch.float32, device=dev)
        self._sq_shard = torch.zeros(L, dtype=torch.float32, device=dev)
        # Fused optimizer of the TP-replicated factors over peer memory
        # (``parallel.peer.OptPeerWorkspace``, set by the engine).
        self.optws = None
        self._opt_coef = torch.zeros(L, dtype=torch.float32, device=dev)
        self._opt_total = torch.zeros(L, dtype=torch.float32, device=dev)
        # DSERVE_TP_DIAG=N: for the first N cycles, recompute every captured
        # activation from the layer input and log its largest deviation from
        # the captured copy (forward capture vs backward recompute; the
        # reference's remat-vs-captured check). Runs eagerly, graphs off.
        self.diag_cycles = int(os.environ.get("DSERVE_TP_DIAG", "0") or 0)
        self.diag_log: list[dict] = []

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
            for t in (cap.layer_in, cap.qkv, cap.ctx, cap.resid_mid, cap.gate_up, cap.act):
                if t is not None:
                    t[:, n:n_pad].zero_()
            cap.final_in[n:n_pad].zero_()
            cap.ids[n:n_pad].zero_()
            cap.positions[n:n_pad].zero_()
        labels = make_labels(cap.ids[:n_pad], starts, lens, n_pad, self.mask_prefix)
        c, s = rope_cos_sin(cap.positions[:n_pad], self.arch.head_dim, self.arch.rope_theta,
                            self.arch.rope_scaling)
        return CycleInputs(n, n_pad, list(starts), list(lens), labels, c, s)

    def _attn_groups(self, ci: CycleInputs):
        key = (ci.n_pad, tuple(ci.starts), tuple(ci.lens))
        g = self._groups_cache.get(key)
        if g is None:
            from ..models.lora_backward import attention_groups
            g = attention_groups(ci.starts, ci.lens, self.masters.params.device)
            if len(self._groups_cache) > 64:
                self._groups_cache.clear()
            self._groups_cache[key] = g
        return g

    def n_valid(self, lens) -> int:
        """Rows that carry a label (host-side, no device sync)."""
        return sum(max(0, ln - 1 - min(self.mask_prefix, max(0, ln - 1))) for ln in lens)

    # ------------------------------------------------------------ CUDA graphs
    def _layer_step(self, cap, ci, l, dh):
        """Backward of layer ``l`` (+ the bucketed replicated-gradient
        all-reduce at bucket boundaries). Returns the new residual gradient."""
        L = self.arch.num_layers
        m = self.masters
        saved = {k: (None if getattr(cap, k) is None else getattr(cap, k)[l, :ci.n_pad]) for k in
                 ("layer_in", "qkv", "ctx", "resid_mid", "gate_up", "act")}
        pos = cap.positions[:ci.n_pad]
        # Activations the forward did not capture (save_attn_qkv / save_attn_ctx /
        # save_resid_mid off) are recomputed from the layer input.
        if saved["qkv"] is None:
            saved["qkv"] = self.bwd.recompute_qkv_raw(l, saved["layer_in"])
        if saved["ctx"] is None:
            # The tcgen05 recompute also leaves the row log-sum-exp, which the
            # attention backward reuses instead of running the forward again.
            lse = self.bwd.attn_stats(ci.n_pad, saved["qkv"].device)[0] if self.bwd.tc_attention(saved["qkv"]) else None
            saved["ctx"] = self.bwd.recompute_ctx(l, saved["qkv"], ci, pos, self.cos_sin, lse=lse)
            saved["lse"] = lse
        if saved["resid_mid"] is None:
            saved["resid_mid"] = self.bwd.recompute_resid_mid(l, saved["layer_in"], saved["ctx"])
        if self.diag_cycles > 0 and self.step < self.diag_cycles:
            self._diag_layer(l, saved, ci, pos)
        tp = self.comm is not None and self.comm.size > 1
        h = None
        if tp and (l + 1) % BUCKET_LAYERS == 0 and l + 1 < L:
            # Layers [l + 1, l + 1 + BUCKET_LAYERS) finished with the previous
            # step: their replicated factor gradients go to their slice owners
            # (fused optimizer) or into one all-reduce on a side stream, which
            # overlaps this layer's backward (it writes only layer l's).
            if self.optws is not None:
                ops.push_slices(m.rep_block(m.grads), (l + 1) * m.rep_per_layer,
                                min(L, l + 1 + BUCKET_LAYERS) * m.rep_per_layer, self.optws)
            else:
                h = self.bwd.reduce_begin(m.rep_block(m.grads, l + 1, min(L, l + 1 + BUCKET_LAYERS)))
        # The first layer's input gradient feeds nothing that is trained.
        dh = self.bwd.layer_backward(l, dh, saved, ci, pos, self.cos_sin, need_input_grad=l > 0)
        self.bwd.reduce_end(h, dh.device)
        self.bwd._mark("wait_bucket")
        if tp and l == 0:
            if self.optws is not None:
                ops.push_slices(m.rep_block(m.grads), 0, min(L, BUCKET_LAYERS) * m.rep_per_layer, self.optws)
            else:
                self.comm.all_reduce(m.rep_block(m.grads, 0, min(L, BUCKET_LAYERS)))
            self.bwd._mark("bucket_allreduce_last")
        return dh

    @torch.no_grad()
    def _diag_layer(self, l, saved, ci, pos) -> None:
        """Largest relative deviation of each recomputed activation from its
        captured copy over the cycle's rows (logged and kept in diag_log)."""
        n = ci.n
        rec = {"cycle": self.step, "layer": l}
        qkv = self.bwd.recompute_qkv_raw(l, saved["layer_in"])
        ctx = self.bwd.recompute_ctx(l, saved["qkv"], ci, pos, self.cos_sin)
        mid = self.bwd.recompute_resid_mid(l, saved["layer_in"], saved["ctx"])
        for name, got in (("qkv", qkv), ("ctx", ctx), ("resid_mid", mid)):
            ref = saved[name][:n].float()
            d = (got[:n].float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)
            rec[name] = float(d)
        self.diag_log.append(rec)
        dprint(f"[diag] cycle {self.step} layer {l}: recompute vs captured rel max "
               f"qkv {rec['qkv']:.2e} ctx {rec['ctx']:.2e} resid_mid {rec['resid_mid']:.2e}")

    def _graph_set(self, cap, ci, n_valid):
        """Per-batch-shape CUDA graphs: one for the head, one per layer, all in
        one memory pool (replayed in capture order, never concurrently). The
        residual gradient lives in a static buffer that every graph reads and
        overwrites. Captured on the first cycle of a shape (the kernels were
        already loaded by :meth:`warmup`)."""
        key = (ci.n_pad, tuple(ci.lens))
        gs = self._graphs.get(key)
        if gs is not None:
            return gs
        if not self.use_graphs or len(self._graphs) >= self.max_graph_shapes or self.diag_cycles > 0:
            return None
        if key not in self._seen_shapes:
            # First cycle of a shape runs eagerly (creates library handles and
            # loads kernels outside any capture); the second captures.
            self._seen_shapes.add(key)
            return None
        dev = self.masters.params.device
        # The residual gradient passes between graphs in a static buffer; the
        # fused TP path keeps it in its own persistent buffer already.
        dh_buf = (self.bwd._resid32(ci.n_pad, dev)[1] if self.bwd.tpws is not None else
                  torch.empty(ci.n_pad, self.arch.hidden, dtype=torch.float32, device=dev))
        gs = {"labels": torch.empty(ci.n_pad, dtype=torch.long, device=dev),
              "cos": torch.empty_like(ci.cos), "sin": torch.empty_like(ci.sin), "dh": dh_buf,
              "loss": torch.zeros((), dtype=torch.float32, device=dev), "n_valid": n_valid}
        gs["labels"].copy_(ci.labels)
        gs["cos"].copy_(ci.cos)
        gs["sin"].copy_(ci.sin)
        sci = CycleInputs(ci.n, ci.n_pad, ci.starts, ci.lens, gs["labels"], gs["cos"], gs["sin"],
                          ci.attn_groups)
        gs["ci"] = sci
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        stream = torch.cuda.current_stream(dev)
        if stream == torch.cuda.default_stream(dev):
            # Capture is not allowed on the legacy default stream; capture on a
            # side stream (replay works on any stream).
            if self._cap_stream is None:
                self._cap_stream = torch.cuda.Stream(dev)
            self._cap_stream.wait_stream(stream)
            stream = self._cap_stream
        # Kernels of this package inside each graph: a replay launches them
        # again, so the launch count (bench accounting) adds them per replay.
        gs["kernels"] = {}
        # The head in pieces (statistics, then each vocabulary chunk): one
        # graph per piece, each a pause boundary.
        gs["head"] = []
        head = self.bwd.head_steps(cap.final_in[:ci.n_pad], sci.labels, n_valid)
        done = False
        while not done:
            g = torch.cuda.CUDAGraph()
            k0 = ops.LAUNCHES[0]
            with torch.cuda.graph(g, pool=self._pool, stream=stream):
                try:
                    next(head)
                except StopIteration:
                    done = True
                    loss, dh = self.bwd._head_out
                    gs["loss"].copy_(loss)
                    _copy_unless_same(gs["dh"], dh)
            gs["kernels"][("head", len(gs["head"]))] = ops.LAUNCHES[0] - k0
            gs["head"].append(g)
        gs["layers"] = {}
        for l in range(self.arch.num_layers - 1, -1, -1):
            g = torch.cuda.CUDAGraph()
            k0 = ops.LAUNCHES[0]
            with torch.cuda.graph(g, pool=self._pool, stream=stream):
                dh = self._layer_step(cap, sci, l, gs["dh"])
                _copy_unless_same(gs["dh"], dh)
            gs["layers"][l] = g
            gs["kernels"][l] = ops.LAUNCHES[0] - k0
        ops.LAUNCHES[0] -= sum(gs["kernels"].values())     # capture launches nothing
        self._graphs[key] = gs
        return gs

    def num_steps(self) -> int:
        """``next`` calls of one :meth:`cycle` until it returns: the head's
        pieces (statistics + one per vocabulary chunk), every layer, then the
        optimizer step."""
        return len(self.bwd.head_chunks()) + 1 + self.arch.num_layers + 1

    def release_graphs(self) -> None:
        """Drop every captured graph (and its memory pool)."""
        self._graphs.clear()
        self._seen_shapes.clear()
        self._pool = None
        import gc
        gc.collect()

    def cycle(self, cap: CaptureBuffers, n: int, starts, lens, epoch: int | None = None,
              sync: bool = True):
        """Generator: yields at each pause boundary; its return value (via
        StopIteration.value) is a pending :class:`CycleResult` — with
        ``sync=False`` the loss and GPU time are resolved later by
        :meth:`finish_cycle`, so the host never waits on the backward.
        On CUDA every step replays a captured graph (a few microseconds of
        host time per layer)."""
        t_wall = time.perf_counter()
        dev = self.masters.params.device
        ev0 = ev1 = None
        if dev.type == "cuda":
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        ci = self._cycle_inputs(cap, n, starts, lens)
        if dev.type == "cuda":
            ci.attn_groups = self._attn_groups(ci)
        m = self.masters
        m.grads.zero_()
        n_valid = self.n_valid(lens)
        L = self.arch.num_layers
        self.bwd.prepare(ci.n_pad, dev, max_rows=cap.layer_in.shape[1])
        gs = self._graph_set(cap, ci, n_valid) if dev.type == "cuda" else None
        if gs is not None:
            gs["labels"].copy_(ci.labels)
            gs["cos"].copy_(ci.cos)
            gs["sin"].copy_(ci.sin)
            for i, g in enumerate(gs["head"]):
                g.replay()
                ops.LAUNCHES[0] += gs["kernels"][("head", i)]
                yield "head"
            loss_sum = gs["loss"]
            for l in range(L - 1, -1, -1):
                gs["layers"][l].replay()
                ops.LAUNCHES[0] += gs["kernels"][l]
                yield l
        else:
            for _ in self.bwd.head_steps(cap.final_in[:ci.n_pad], ci.labels, n_valid):
                yield "head"
            loss_sum, dh = self.bwd._head_out
            yield "head"
            for l in range(L - 1, -1, -1):
                dh = self._layer_step(cap, ci, l, dh)
                yield l
        self._optimizer_step(epoch)
        self.bwd._mark("optimizer")
        self.publish()
        self.bwd._mark("publish")
        if ev1 is not None:
            ev1.record()
        res = CycleResult(0.0, n, n_valid, 0.0, 0.0, self.step)
        res._pending = (loss_sum.clone(), ev0, ev1, t_wall)
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

    @torch.no_grad()
    def warmup(self, cap: CaptureBuffers, n: int, starts, lens) -> float:
        """Run one full cycle on the calling thread and restore every piece of
        optimizer and adapter state afterwards. Loads every kernel module the
        backward uses before the background feeder thread ever launches one,
        and measures the cycle. Returns its GPU milliseconds."""
        m = self.masters
        snap = [t.clone() for t in (m.params, m.exp_avg, m.exp_avg_sq)]
        step, epoch, tokens, losses = self.step, self.epoch, self.total_tokens, list(self.losses)
        # Eager first (loads kernels, creates library handles), then once more
        # through the CUDA-graph path, which captures this shape's graphs.
        use = self.use_graphs
        self.use_graphs = False
        res = self.run_cycle(cap, n, starts, lens)
        self.use_graphs = use
        if use:
            res = self.run_cycle(cap, n, starts, lens)
        for t, s in zip((m.params, m.exp_avg, m.exp_avg_sq), snap):
            t.copy_(s)
        self.step, self.epoch, self.total_tokens, self.losses = step, epoch, tokens, losses
        self.publish()
        if m.params.is_cuda:
            torch.cuda.synchronize(m.params.device)
        return res.gpu_ms

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
        if self.optws is not None:
            # Fused path: the replicated block's slices were pushed to their
            # owners during the backward; each owner sums its slice, the
            # ranks swap per-layer squared norms (replicated slice + own
            # shard), the owner runs AdamW on its slice and sends the new
            # values to every rank; the shard runs AdamW locally.
            ops.seg_sumsq(m.shard_block(m.grads), m.shard_per_layer, self._sq_shard)
            total = ops.fused_replicated_adamw(
                self.optws, m.rep_block(m.params), m.rep_block(m.grads), m.rep_block(m.exp_avg),
                m.rep_block(m.exp_avg_sq), m.rep_per_layer, self._sq_shard, max_norm=CLIP_NORM, lr=lr, wd=self.wd,
                step=self.step, coef=self._opt_coef, total=self._opt_total, sq=self._sq_rep)
            ops.adamw(m.shard_block(m.params), m.shard_block(m.grads), m.shard_block(m.exp_avg),
                      m.shard_block(m.exp_avg_sq), seg_len=m.shard_per_layer, seg_sumsq_t=total,
                      max_norm=CLIP_NORM, grad_scale=1.0, lr=lr, wd=self.wd, step=self.step)
            ops.fused_replicated_finish(self.optws, m.rep_block(m.params))
            return
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

    def save_adapter(self, path: str, save_id: str = "", extra: dict | None = None,
                     background: bool = False, after=None) -> str | None:
        """PEFT checkpoint of the trained adapter (merged across TP ranks, on
        rank 0). The tensors are gathered to host memory here; with
        ``background`` the files are written by a writer thread, so the
        serving loop does not wait on the disk — ``trainer_state.json`` (the
        completion marker) or ``save_error.json`` appears when it is done.
        ``after`` (e.g. pruning older checkpoints) runs once the files are
        written, on the same thread, so it sees the new directory."""
        full = self.export_full()
        if full is None:
            return None
        state = {"save_id": save_id, "step": self.step, "epoch": self.epoch,
                 "total_tokens": self.total_tokens, "time": time.time(),
                 "last_loss": self.losses[-1] if self.losses else None, **(extra or {})}
        cfg = dict(self.adapter_config)
        if not background:
            peft_io.write_peft_adapter(path, full, cfg, state)
            if after is not None:
                after()
            return path
        if self._writer is None:
            import concurrent.futures as cf
            self._writer = cf.ThreadPoolExecutor(max_workers=1, thread_name_prefix="dsv-save")

        def write():
            try:
                peft_io.write_peft_adapter(path, full, cfg, state)
            except Exception as e:  # reported through the save handshake
                peft_io.write_save_error(path, save_id, repr(e))
                return
            if after is not None:
                after()
        self._pending_save = self._writer.submit(write)
        return path

    def wait_saves(self) -> None:
        """Block until every background checkpoint write has finished."""
        if self._pending_save is not None:
            self._pending_save.result()
            self._pending_save = None
