"""Turns a scheduled step into device inputs, runs the forward, samples.

All per-step integer metadata (token ids, positions, KV slots, block tables,
varlen offsets, attention tile list, LoRA slot ids and per-tile slot masks,
logit rows) is packed on the host into ONE pinned int32/int64 staging buffer
and moved with ONE host-to-device copy; the device tensors are views into it.
"""

from __future__ import annotations

import time

import numpy as np
import torch

from .. import ops
from ..models.decoder import CaptureBuffers, DecoderModel, FTAborted, ForwardBatch
from .scheduler import SchedulerOutput


def _token_at(r, i: int) -> int:
    """Token ``i`` of a request's prompt + output (without joining the lists)."""
    n = len(r.prompt_ids)
    return r.prompt_ids[i] if i < n else r.output_ids[i - n]


def _token_slice(r, start: int, n: int) -> list[int]:
    npr = len(r.prompt_ids)
    if start + n <= npr:
        return r.prompt_ids[start:start + n]
    if start >= npr:
        return r.output_ids[start - npr:start - npr + n]
    return r.prompt_ids[start:] + r.output_ids[:start + n - npr]


class _Packer:
    """Accumulates int64 segments; one pinned buffer, one copy."""

    def __init__(self):
        self.parts: list[tuple[str, np.ndarray]] = []

    def add(self, name: str, arr) -> None:
        self.parts.append((name, np.ascontiguousarray(np.asarray(arr, dtype=np.int64).ravel())))

    def freeze(self) -> tuple[np.ndarray, list[tuple[str, int]]]:
        """One contiguous int64 array + (name, length) spans (what rank 0 sends
        to the other tensor-parallel ranks)."""
        arr = np.concatenate([a for _, a in self.parts]) if self.parts else np.zeros(0, np.int64)
        return arr, [(n, a.size) for n, a in self.parts]

    @classmethod
    def thaw(cls, arr: np.ndarray, spans: list[tuple[str, int]]) -> "_Packer":
        pk = cls()
        off = 0
        for n, k in spans:
            pk.parts.append((n, arr[off:off + k]))
            off += k
        return pk

    def ship(self, device, pinned: "PinnedRing | None"):
        total = sum(a.size for _, a in self.parts)
        slot = None
        if device.type == "cuda":
            host, slot = pinned.acquire(total)
        else:
            host = torch.empty(total, dtype=torch.int64)
        hn = host.numpy()
        off = 0
        spans = {}
        for name, a in self.parts:
            hn[off:off + a.size] = a
            spans[name] = (off, a.size)
            off += a.size
        dev = host.to(device, non_blocking=True) if device.type == "cuda" else host
        if slot is not None:
            pinned.release(slot)
        return {k: dev[o:o + n] for k, (o, n) in spans.items()}, pinned, total * 8


class PinnedRing:
    """Pinned host staging buffers for the per-step H2D copy. A buffer is
    reused only after the copy that last read it has executed (an event
    recorded right after the copy), so a host that runs ahead of the GPU (a
    follower rank, or steps that sample nothing) never overwrites step
    metadata the GPU has not fetched yet."""

    def __init__(self, n: int = 4):
        self.bufs: list[torch.Tensor | None] = [None] * n
        self.events: list = [None] * n
        self.i = 0

    def acquire(self, numel: int):
        k = self.i
        self.i = (self.i + 1) % len(self.bufs)
        if self.events[k] is not None:
            self.events[k].synchronize()
        b = self.bufs[k]
        if b is None or b.numel() < numel:
            b = torch.empty(max(numel, 1 << 16) * 2, dtype=torch.int64, pin_memory=True)
            self.bufs[k] = b
        return b[:numel], k

    def release(self, k: int) -> None:
        ev = torch.cuda.Event()
        ev.record()
        self.events[k] = ev


DECODE_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256)


class DecodeGraphs:
    """CUDA graphs of a decode-only step (forward + sampling), one per padded
    batch size and LoRA on/off, replayed with one host->device copy of the
    step's metadata into static buffers. A decode step otherwise costs a few
    hundred kernel launches from Python, which is more host time than the GPU
    needs for the step.

    Padded rows carry no token: slot -1 (no KV write), context 0 (attention
    skips them), LoRA slot -1; their logits and samples are ignored. The
    attention splits each sequence's context itself (keys_per_split 0), so
    a graph is valid for any context length up to ``max_model_len``."""

    def __init__(self, model: DecoderModel, device, block_size: int, max_model_len: int, num_sms: int):
        self.model = model
        self.device = device
        self.maxb = -(-max_model_len // block_size)
        self.max_model_len = max_model_len
        self.num_sms = num_sms
        self.graphs: dict[tuple[int, bool], dict] = {}
        self.pool = None
        self.replays = 0
        self.eos_ids: tuple[int, ...] = ()   # set by the engine (min_tokens masks them)
        self._host: torch.Tensor | None = None
        self._host_f: torch.Tensor | None = None
        self._evt = None
        self._side = None

    @staticmethod
    def bucket(n: int) -> int | None:
        for b in DECODE_BUCKETS:
            if b >= n:
                return b
        return None

    def _layout(self, Bp: int, lora: bool) -> dict:
        sizes = [("ids", Bp), ("pos", Bp), ("slot", Bp), ("btab", Bp * self.maxb), ("ctx", Bp),
                 ("seeds", Bp)]
        if lora:
            sizes += [("lslot", Bp), ("tile", -(-Bp // 128))]
        lay, off = {}, 0
        for k, n in sizes:
            lay[k] = (off, n)
            off += n
        return {"spans": lay, "total": off}

    def _forward(self, st: dict, Bp: int, lora: bool):
        m = self.model
        i32 = lambda t: t.to(torch.int32)
        splits = ops.decode_splits(Bp, m.hkv_l, self.max_model_len, self.num_sms)[0]
        b = ForwardBatch(
            input_ids=st["ids"], positions=st["pos"], slot_mapping=st["slot"], num_decode=Bp,
            dec_block_tables=i32(st["btab"]).view(Bp, self.maxb), dec_ctx_lens=i32(st["ctx"]),
            dec_splits=splits, dec_keys_per_split=0,
            slot_ids=i32(st["lslot"]) if lora else None, tile_slots=i32(st["tile"]) if lora else None,
            logits_idx=st["rows"])
        logits = m.forward(b, None)
        ops.sample(logits, st["temps"], st["seeds"], st["toks"])
        return logits

    def _capture(self, Bp: int, lora: bool) -> dict:
        lay = self._layout(Bp, lora)
        flat = torch.zeros(lay["total"], dtype=torch.int64, device=self.device)
        st = {k: flat[o:o + n] for k, (o, n) in lay["spans"].items()}
        st["rows"] = torch.arange(Bp, dtype=torch.int64, device=self.device)
        st["temps"] = torch.zeros(Bp, dtype=torch.float32, device=self.device)
        st["toks"] = torch.zeros(Bp, dtype=torch.int64, device=self.device)
        st["slot"].fill_(-1)
        if lora:
            st["lslot"].fill_(-1)
        stream = torch.cuda.current_stream(self.device)
        n0 = ops.LAUNCHES[0]
        self._forward(st, Bp, lora)            # eager warm-up: lazy set-up outside the capture
        stream.synchronize()
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        k0 = ops.LAUNCHES[0]
        # Capture needs a non-default stream; replays may run on any stream.
        cap_stream = stream
        if stream == torch.cuda.default_stream(self.device):
            if self._side is None:
                self._side = torch.cuda.Stream(self.device)
            cap_stream = self._side
            cap_stream.wait_stream(stream)
        with torch.cuda.graph(g, pool=self.pool, stream=cap_stream):
            logits = self._forward(st, Bp, lora)
        if cap_stream is not stream:
            stream.wait_stream(cap_stream)
        kernels = ops.LAUNCHES[0] - k0
        ops.LAUNCHES[0] = n0                   # counted per replay from now on
        # `logits` lives in the graph's pool: every replay rewrites it.
        ent = {"graph": g, "flat": flat, "st": st, "lay": lay, "kernels": kernels, "logits": logits}
        self.graphs[(Bp, lora)] = ent
        return ent

    def capture_all(self, max_seqs: int, lora: bool) -> int:
        """Capture every bucket up to ``max_seqs`` (with and without LoRA)
        before serving, so no request waits on a capture. Returns how many."""
        top = self.bucket(min(max_seqs, DECODE_BUCKETS[-1])) or DECODE_BUCKETS[-1]
        n = 0
        for Bp in DECODE_BUCKETS:
            if Bp > top:
                break
            for lo in ((False, True) if lora else (False,)):
                if (Bp, lo) not in self.graphs:
                    self._capture(Bp, lo)
                    n += 1
        return n

    def run(self, meta: dict, pk: "_Packer", temps=None, seeds=None) -> tuple[torch.Tensor, int]:
        """Replay the graph for this decode step; returns (tokens [Bp] on the
        device, H2D bytes)."""
        nd = meta["nd"]
        Bp = self.bucket(nd)
        lora = bool(meta["use_lora"])
        ent = self.graphs.get((Bp, lora)) or self._capture(Bp, lora)
        lay = ent["lay"]
        parts = dict(pk.parts)
        total = lay["total"]
        if self._host is None or self._host.numel() < total:
            self._host = torch.zeros(max(total, 1 << 16), dtype=torch.int64, pin_memory=True)
            self._host_f = torch.zeros(256, dtype=torch.float32, pin_memory=True)
        if self._evt is not None:
            self._evt.synchronize()            # the previous step's copy has read the pinned buffer
        h = self._host.numpy()
        sp = lay["spans"]

        def put(name, arr, fill=0):
            o, n = sp[name]
            h[o:o + n] = fill
            h[o:o + len(arr)] = arr
        put("ids", parts["ids"])
        put("pos", parts["pos"])
        put("slot", parts["slot_mapping"], fill=-1)
        o, n = sp["btab"]
        h[o:o + n] = 0
        bt = parts["dec_btab"].reshape(nd, meta["maxb"])
        h[o:o + n].reshape(Bp, self.maxb)[:nd, :meta["maxb"]] = bt
        put("ctx", parts["dec_ctx"])
        put("seeds", seeds if seeds is not None else np.zeros(nd, np.int64))
        if lora:
            put("lslot", parts["lslot"], fill=-1)
            put("tile", parts["tile_slots"])
        hf = self._host_f.numpy()
        hf[:Bp] = 0.0
        if temps is not None:
            hf[:nd] = temps
        ent["flat"].copy_(self._host[:total], non_blocking=True)
        ent["st"]["temps"].copy_(self._host_f[:Bp], non_blocking=True)
        self._evt = torch.cuda.Event()
        self._evt.record()
        ent["graph"].replay()
        ops.LAUNCHES[0] += ent["kernels"]
        self.replays += 1
        self.last_logits = ent["logits"][:nd]
        return ent["st"]["toks"], total * 8 + Bp * 4

    def release(self) -> None:
        self.graphs.clear()
        self.pool = None


class ModelRunner:
    def __init__(self, model: DecoderModel, block_size: int, device, num_sms: int = 148,
                 ft_slot: int = -1, max_model_len: int = 4096, decode_graphs: bool = True):
        self.model = model
        self.block_size = block_size
        self.device = torch.device(device)
        self.num_sms = num_sms
        self.ft_slot = ft_slot
        self._pinned = PinnedRing() if self.device.type == "cuda" else None
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0
        self.graphs = (DecodeGraphs(model, self.device, block_size, max_model_len, num_sms)
                       if (decode_graphs and self.device.type == "cuda") else None)

    def graph_eligible(self, meta: dict) -> bool:
        return (self.graphs is not None and meta["npf"] == 0 and meta["nd"] > 0
                and not meta.get("full_sampler", False)
                and DecodeGraphs.bucket(meta["nd"]) is not None)

    def abort_hook(self, should_abort, vote=None, ahead: int = 2):
        """Per-layer pre-emption check of an FT-only forward (tier C): the host
        never runs more than ``ahead`` layers ahead of the GPU (an event per
        layer), so an abort lands within a couple of layers; under TP the
        decision is a MAX vote so every rank stops at the same layer."""
        events = []

        def hook(l: int) -> bool:
            if self.device.type == "cuda":
                if l >= ahead:
                    events[l - ahead].synchronize()
                ev = torch.cuda.Event()
                ev.record()
                events.append(ev)
            flag = 1 if should_abort() else 0
            if vote is not None:
                flag = vote(flag)
            return bool(flag)
        return hook

    def forward_follower(self, meta: dict, pk: "_Packer", cap, vote=None) -> bool:
        """A follower rank's replay of a step: the same graph or kernels as rank 0.
        Returns False when the step was pre-empted (tier C, same layer as rank 0)."""
        if self.graph_eligible(meta):
            self.graphs.run(meta, pk)
            return True
        b = self.batch_from(meta, pk)
        hook = self.abort_hook(lambda: False, vote) if meta.get("abortable") else None
        try:
            self.model.forward(b, cap, layer_hook=hook)
        except FTAborted:
            return False
        return True

    def build_host(self, out: SchedulerOutput, ft_dst: int = 0) -> tuple[dict, _Packer, list]:
        bs = self.block_size
        ids, pos, slots, lslot = [], [], [], []
        sample_rows, sample_reqs = [], []
        # Decode rows (one token each, first in the batch) in one vectorised
        # pass: per-sequence numpy calls cost ~10 us each at 256 sequences.
        nd0 = len(out.decode)
        if nd0:
            dec = [s.req for s in out.decode]
            p = np.fromiter((s.start for s in out.decode), dtype=np.int64, count=nd0)
            ids.append(np.fromiter((_token_at(r, int(q)) for r, q in zip(dec, p)), dtype=np.int64, count=nd0))
            pos.append(p)
            blk = np.fromiter((r.block_ids[int(q) // bs] for r, q in zip(dec, p)), dtype=np.int64, count=nd0)
            slots.append(blk * bs + p % bs)
            lslot.append(np.fromiter((self.ft_slot if r.is_ft else r.lora_slot for r in dec), dtype=np.int64,
                                     count=nd0))
            sample_rows.extend(range(nd0))
            sample_reqs.extend(dec)
        row = nd0
        for s in out.prefill + out.ft:
            r = s.req
            toks = _token_slice(r, s.start, s.num_new)
            p = np.arange(s.start, s.start + s.num_new)
            blk = np.asarray(r.block_ids, dtype=np.int64)
            ids.append(toks)
            pos.append(p)
            slots.append(blk[p // bs] * bs + p % bs)
            lslot.append(np.full(s.num_new, self.ft_slot if r.is_ft else r.lora_slot, dtype=np.int64))
            row += s.num_new
            if s.sample:
                sample_rows.append(row - 1)
                sample_reqs.append(r)
        T = row
        pk = _Packer()
        pk.add("ids", np.concatenate(ids) if ids else [])
        pk.add("pos", np.concatenate(pos) if pos else [])
        pk.add("slot_mapping", np.concatenate(slots) if slots else [])
        nd = len(out.decode)
        maxb = max([len(s.req.block_ids) for s in out.seqs] + [1])
        splits, kps = 1, 64
        if nd:
            btab = np.zeros((nd, maxb), dtype=np.int64)
            for i, s in enumerate(out.decode):
                btab[i, :len(s.req.block_ids)] = s.req.block_ids
            ctx = [s.req.num_computed + 1 for s in out.decode]
            pk.add("dec_btab", btab)
            pk.add("dec_ctx", ctx)
            hkv = self.model.hkv_l
            splits, kps = ops.decode_splits(nd, hkv, max(ctx), self.num_sms)
        pf = out.prefill + out.ft
        if pf:
            btab = np.zeros((len(pf), maxb), dtype=np.int64)
            cu = [0]
            ctx = []
            for i, s in enumerate(pf):
                btab[i, :len(s.req.block_ids)] = s.req.block_ids
                cu.append(cu[-1] + s.num_new)
                ctx.append(s.start + s.num_new)
            tiles = ops.prefill_tiles(cu)
            pk.add("pf_btab", btab)
            pk.add("pf_cu", cu)
            pk.add("pf_ctx", ctx)
            pk.add("pf_tiles", np.asarray(tiles, dtype=np.int64).reshape(-1))
        ls = np.concatenate(lslot) if lslot else np.zeros(0, dtype=np.int64)
        use_lora = self.model.lora is not None and bool((ls >= 0).any())
        if use_lora:
            pk.add("lslot", ls)
            nt = -(-T // 128)
            mask = np.zeros(nt, dtype=np.int64)
            for t in range(nt):
                seg = ls[t * 128:(t + 1) * 128]
                seg = seg[seg >= 0]
                m = 0
                for v in np.unique(seg):
                    m |= 1 << int(v)
                mask[t] = m if m < (1 << 31) else m - (1 << 32)
            pk.add("tile_slots", mask)
        pk.add("logits_idx", sample_rows)
        meta = {"full_sampler": any(r.params.needs_full_sampler for r in sample_reqs),
                "nd": nd, "maxb": maxb, "splits": splits, "kps": kps, "npf": len(pf),
                "use_lora": use_lora, "T": T, "ft_rows": sum(s.num_new for s in out.ft),
                "ft_dst": ft_dst}
        return meta, pk, sample_reqs

    def prepare(self, out: SchedulerOutput, ft_dst: int = 0) -> tuple[ForwardBatch, list]:
        meta, pk, reqs = self.build_host(out, ft_dst)
        return self.batch_from(meta, pk), reqs

    def batch_from(self, meta: dict, pk: _Packer) -> ForwardBatch:
        """Device batch from host metadata (also used by the follower ranks)."""
        d, self._pinned, nbytes = pk.ship(self.device, self._pinned)
        self.last_h2d_bytes = nbytes
        i32 = lambda t: t.to(torch.int32)
        nd, maxb, npf, use_lora = meta["nd"], meta["maxb"], meta["npf"], meta["use_lora"]
        splits, kps, T, ft_rows, ft_dst = meta["splits"], meta["kps"], meta["T"], meta["ft_rows"], meta["ft_dst"]
        pf = npf
        b = ForwardBatch(
            input_ids=d["ids"], positions=d["pos"], slot_mapping=d["slot_mapping"],
            num_decode=nd,
            dec_block_tables=i32(d["dec_btab"]).view(nd, maxb) if nd else None,
            dec_ctx_lens=i32(d["dec_ctx"]) if nd else None,
            dec_splits=splits, dec_keys_per_split=kps,
            num_prefill_seqs=pf,
            pf_cu_q=i32(d["pf_cu"]) if pf else None,
            pf_ctx_lens=i32(d["pf_ctx"]) if pf else None,
            pf_block_tables=i32(d["pf_btab"]).view(pf, maxb) if pf else None,
            pf_tile_info=i32(d["pf_tiles"]).view(-1, 2) if pf else None,
            slot_ids=i32(d["lslot"]) if use_lora else None,
            tile_slots=i32(d["tile_slots"]) if use_lora else None,
            logits_idx=d["logits_idx"],
            ft_lo=T - ft_rows, ft_hi=T, ft_dst=ft_dst)
        return b

    def execute(self, out: SchedulerOutput, cap: CaptureBuffers | None = None, ft_dst: int = 0,
                on_host_plan=None, before_sample=None, abort_check=None, vote=None):
        """Forward + sampling. Returns ({seq_no: token}, logits). ``on_host_plan``
        (rank 0 under TP) receives the host metadata before the forward is
        enqueued, so the other ranks can replay the same step."""
        self.last_aborted = False
        self.last_phases = (0.0, 0.0, 0.0, 0.0)
        if out.is_empty():
            return {}, None
        t0 = time.perf_counter()
        meta, pk, reqs = self.build_host(out, ft_dst)
        # Tier C: an FT-only step can be abandoned between layers.
        meta["abortable"] = bool(abort_check is not None and out.ft and not out.decode and not out.prefill)
        if on_host_plan is not None:
            on_host_plan(meta, pk)
        t1 = time.perf_counter()
        # Host seconds of this call: (pack + plan send, enqueue, backward feed,
        # sampling incl. the wait for the GPU).
        self.last_phases = (t1 - t0, 0.0, 0.0, 0.0)
        if self.graph_eligible(meta) and len(reqs) == meta["nd"]:
            temps = np.array([r.params.temperature for r in reqs], dtype=np.float32)
            seeds = np.array([(r.params.seed if r.params.seed is not None else r.seq_no) * 1000003
                              + len(r.output_ids) for r in reqs], dtype=np.int64)
            toks, nbytes = self.graphs.run(meta, pk, temps, seeds)
            self.last_h2d_bytes = nbytes
            t2 = time.perf_counter()
            self.last_enqueue_s = t2 - t0
            if before_sample is not None:
                before_sample()
            t3 = time.perf_counter()
            host = toks[:len(reqs)].cpu()
            self.last_d2h_bytes = len(reqs) * 8
            res = {r.seq_no: int(v) for r, v in zip(reqs, host.tolist())}
            self.last_phases = (t1 - t0, t2 - t1, t3 - t2, time.perf_counter() - t3)
            return res, self.graphs.last_logits
        b = self.batch_from(meta, pk)
        hook = self.abort_hook(abort_check, vote) if meta["abortable"] else None
        try:
            logits = self.model.forward(b, cap if out.ft else None, layer_hook=hook)
        except FTAborted:
            self.last_aborted = True
            self.last_enqueue_s = time.perf_counter() - t0
            return {}, None
        t2 = time.perf_counter()
        self.last_enqueue_s = t2 - t0   # host time to enqueue the forward
        if before_sample is not None:
            before_sample()
        t3 = time.perf_counter()
        res = self.sample(logits, reqs)
        self.last_phases = (t1 - t0, t2 - t1, t3 - t2, time.perf_counter() - t3)
        return res, logits

    def sample(self, logits, reqs) -> dict:
        if not reqs:
            self.last_d2h_bytes = 0
            return {}
        R = len(reqs)
        t = torch.tensor([r.params.temperature for r in reqs], dtype=torch.float32)
        sd = torch.tensor([(r.params.seed if r.params.seed is not None else r.seq_no) * 1000003
                           + len(r.output_ids) for r in reqs], dtype=torch.int64)
        toks = torch.empty(R, dtype=torch.int64, device=logits.device)
        dev = logits.device
        topk = topp = lps = None
        if any(r.params.has_penalties for r in reqs):
            from .penalties import apply_penalties
            self.last_h2d_bytes += apply_penalties(logits, reqs, self.eos_ids)
        if any(r.params.needs_full_sampler for r in reqs):
            topk = torch.tensor([r.params.top_k for r in reqs], dtype=torch.int32).to(dev, non_blocking=True)
            topp = torch.tensor([r.params.top_p for r in reqs], dtype=torch.float32).to(dev, non_blocking=True)
            if any(r.params.logprobs for r in reqs):
                lps = torch.empty(R, dtype=torch.float32, device=dev)
            self.last_h2d_bytes += R * 8
        ops.sample(logits, t.to(dev, non_blocking=True), sd.to(dev, non_blocking=True), toks, topk, topp, lps)
        host = toks.cpu()
        self.last_h2d_bytes += R * 12
        self.last_d2h_bytes = R * 8
        if lps is not None:
            for r, v in zip(reqs, lps.cpu().tolist()):
                if r.params.logprobs:
                    r.output_logprobs.append(float(v))
            self.last_d2h_bytes += R * 4
        k = max((r.params.top_logprobs for r in reqs if r.params.logprobs), default=0)
        if k > 0:
            # the k most likely tokens of each position under the model's
            # distribution (log-softmax of the logits)
            vals, idx = torch.log_softmax(logits[:R].float(), dim=-1).topk(k, dim=-1)
            vals, idx = vals.cpu().tolist(), idx.cpu().tolist()
            self.last_d2h_bytes += R * k * 12
            for r, v, i in zip(reqs, vals, idx):
                if r.params.logprobs and r.params.top_logprobs > 0:
                    n = r.params.top_logprobs
                    r.output_top_logprobs.append(list(zip(i[:n], v[:n])))
        return {r.seq_no: int(v) for r, v in zip(reqs, host.tolist())}
