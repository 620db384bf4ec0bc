"""Turns a scheduled step into device inputs, runs the forward, samples.

All per-step integer metadata (token ids, positions, KV slots, block tables,
varlen offsets, attention tile list, LoRA slot ids and per-tile slot masks,
logit rows) is packed on the host into ONE pinned int32/int64 staging buffer
and moved with ONE host-to-device copy; the device tensors are views into it.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import ops
from ..models.decoder import CaptureBuffers, DecoderModel, ForwardBatch
from .scheduler import SchedulerOutput


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


class ModelRunner:
    def __init__(self, model: DecoderModel, block_size: int, device, num_sms: int = 148,
                 ft_slot: int = -1):
        self.model = model
        self.block_size = block_size
        self.device = torch.device(device)
        self.num_sms = num_sms
        self.ft_slot = ft_slot
        self._pinned = PinnedRing() if self.device.type == "cuda" else None
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0

    def build_host(self, out: SchedulerOutput, ft_dst: int = 0) -> tuple[dict, _Packer, list]:
        bs = self.block_size
        ids, pos, slots, lslot = [], [], [], []
        sample_rows, sample_reqs = [], []
        row = 0
        for s in out.seqs:
            r = s.req
            toks = r.all_ids[s.start:s.start + s.num_new]
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
        meta = {"nd": nd, "maxb": maxb, "splits": splits, "kps": kps, "npf": len(pf),
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
                on_host_plan=None, before_sample=None):
        """Forward + sampling. Returns ({seq_no: token}, logits). ``on_host_plan``
        (rank 0 under TP) receives the host metadata before the forward is
        enqueued, so the other ranks can replay the same step."""
        if out.is_empty():
            return {}, None
        meta, pk, reqs = self.build_host(out, ft_dst)
        if on_host_plan is not None:
            on_host_plan(meta, pk)
        b = self.batch_from(meta, pk)
        logits = self.model.forward(b, cap if out.ft else None)
        if before_sample is not None:
            before_sample()
        return self.sample(logits, reqs), logits

    def sample(self, logits, reqs) -> dict:
        if not reqs:
            self.last_d2h_bytes = 0
            return {}
        R = len(reqs)
        t = torch.tensor([r.params.temperature for r in reqs], dtype=torch.float32)
        sd = torch.tensor([(r.params.seed if r.params.seed is not None else r.seq_no) * 1000003
                           + len(r.output_ids) for r in reqs], dtype=torch.int64)
        toks = torch.empty(R, dtype=torch.int64, device=logits.device)
        ops.sample(logits, t.to(logits.device, non_blocking=True), sd.to(logits.device, non_blocking=True),
                   toks)
        host = toks.cpu()
        self.last_h2d_bytes += R * 12
        self.last_d2h_bytes = R * 8
        return {r.seq_no: int(v) for r, v in zip(reqs, host.tolist())}
