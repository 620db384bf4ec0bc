"""The co-serving engine: inference with continuous batching and multi-LoRA,
plus LoRA finetuning on the same GPU(s).

One process per GPU. Rank 0 owns every decision (scheduling, FT admission,
backward triggers, pauses) and sends each step's *plan* (packed integer
metadata + a few flags) to the other tensor-parallel ranks, which replay it;
every rank therefore issues the same kernels and collectives in the same order
(rank-symmetric by construction — no per-layer host votes).

Step (rank 0):

1. ingest arrivals; throttles; job tick;
2. inference schedule (decode, then chunked prefill);
3. FT admission against the SLOs using the step's exact composition; the
   admitted samples are appended as whole prefill-only rows and get capture
   offsets in the activation buffer;
4. forward on the high-priority stream (activations of FT rows captured by
   the kernels), sampling, scheduler update, per-step CUDA-event timing into
   the estimator (read one step late so the host never waits for it);
5. a full buffer starts a backward cycle; the cycle advances on the
   low-priority stream between steps, one layer per boundary, unless an
   inference prefill is pending (pause-on-arrival) or the run-ahead bound is
   reached; its completion (an event) publishes the adapter and reopens
   admission.
"""

from __future__ import annotations

import json
import threading
import os
import time
from collections import deque
from dataclasses import dataclass

import numpy as np
import torch

from .. import dprint, ops
from ..config import AdapterRoutingConfig, EngineConfig, FinetuneConfig
from ..models.configs import ModelArch, resolve_arch
from ..models.decoder import CaptureBuffers, DecoderModel
from ..models.lora import LoraServeBuffers, random_adapter
from ..models.weights import TPInfo, init_weights
from .ft.admission import FinetuneAdmission
from .ft.coordinator import FinetuneCoordinator
from .ft.estimator import MergedExecutionEstimator, StepFeatures, StepLog
from .ft.store import FinetuningStore
from .ft.tbt_window import DecodeGapWindow
from .ft_job import FinetuneJobSpec, FtJobManager
from .kv_cache import KVCache
from .model_runner import ModelRunner
from .request import Request, SamplingParams
from .scheduler import Scheduler, SchedulerOutput
from .trainer import LoraTrainer

FT_ADAPTER_NAME = "__finetune__"
# Host-side fault injection for tests: raise in the backward after this many
# layer steps (-1 = off); nothing is done to the GPU.
_FAIL_BACKWARD_AT = int(os.environ.get("DSERVE_TEST_FAIL_BACKWARD", "-1"))


@dataclass
class StepRecord:
    features: StepFeatures
    start: object          # cuda event or float
    end: object
    predicted: float | None
    kind: str


def _generation_eos_ids(model: str) -> tuple[int, ...]:
    """``eos_token_id`` of a model directory's ``generation_config.json`` (an
    int or a list), else ()."""
    path = os.path.join(model, "generation_config.json") if model and os.path.isdir(model) else None
    if path is None or not os.path.isfile(path):
        return ()
    try:
        with open(path) as f:
            e = json.load(f).get("eos_token_id")
    except (OSError, ValueError):
        return ()
    if isinstance(e, int):
        return (e,)
    if isinstance(e, list):
        return tuple(int(x) for x in e if isinstance(x, int))
    return ()


class CoServingEngine:
    def __init__(self, ecfg: EngineConfig, ftcfg: FinetuneConfig | None = None,
                 rcfg: AdapterRoutingConfig | None = None, comm=None,
                 arch: ModelArch | None = None, adapters: dict | None = None,
                 tokenizer=None, ft_store: FinetuningStore | None = None,
                 ft_adapter: tuple[dict, int, float] | None = None):
        self.ecfg = ecfg
        self.ftcfg = ftcfg or FinetuneConfig()
        self.rcfg = rcfg or AdapterRoutingConfig()
        self.comm = comm
        self.tp = TPInfo(comm.rank, comm.size) if comm is not None else TPInfo()
        self.is_driver = self.tp.rank == 0
        dev = ecfg.device or ("cuda" if torch.cuda.is_available() else "cpu")
        if dev == "cuda":
            dev = f"cuda:{torch.cuda.current_device()}"
        self.device = torch.device(dev)
        self.cuda = self.device.type == "cuda"
        self.dtype = torch.bfloat16 if self.cuda else torch.float32
        self.arch = arch or resolve_arch(ecfg.model)
        self.tokenizer = tokenizer
        t0 = time.perf_counter()
        self.weights = self._load_weights(ecfg)
        self._gen_eos = _generation_eos_ids(ecfg.model)
        # ---- LoRA slots: inference adapters + the pinned FT slot
        self.adapter_slots: dict[str, int] = {}
        self.adapter_meta: dict[str, dict] = {}
        n_slots = max(1, ecfg.max_loras) if ecfg.enable_lora else 0
        self.lora = (LoraServeBuffers(self.arch, self.tp, n_slots, ecfg.max_lora_rank, self.device,
                                      self.dtype) if n_slots else None)
        self.ft_slot = -1
        # ---- finetuning
        self.ft_enabled = bool(self.ftcfg.enable_finetuning) and self.lora is not None
        cap_tokens = self.ftcfg.max_saved_finetuning_tokens
        # save_activations off: FT rows are forwarded but nothing is captured or
        # trained (measures the capture overhead).
        fc = self.ftcfg
        self.capture = (CaptureBuffers.allocate(self.weights, cap_tokens + 8, self.device, self.dtype,
                                                save_qkv=fc.save_attn_qkv, save_ctx=fc.save_attn_ctx,
                                                save_resid_mid=fc.save_resid_mid)
                        if self.ft_enabled and fc.save_activations else None)
        # ---- fused GEMM + all-reduce workspace (row-parallel o / down under TP)
        self.peer_ws = None
        if self.cuda and comm is not None and comm.size > 1 and ecfg.tp_comm == "fused":
            from ..parallel.peer import PeerWorkspace
            rows = ecfg.max_num_batched_tokens + (cap_tokens if self.ft_enabled else 0) + 128
            self.peer_ws = PeerWorkspace(comm, rows, self.arch.hidden)
            comm.peer_ws = self.peer_ws
            if not self._self_test_fused(comm):
                self.peer_ws.close()
                self.peer_ws = comm.peer_ws = None
        # ---- vocabulary-parallel embedding read over peer memory (no all-reduce)
        self.embed_peer = None
        if self.cuda and comm is not None and comm.size > 1 and ecfg.tp_comm == "fused":
            self._setup_embed_peer(comm)
        # ---- KV cache sized from what is left
        self.kv = self._alloc_kv()
        self.model = DecoderModel(self.weights, self.kv.k, self.kv.v, self.lora, comm)
        self.model.embed_peer = self.embed_peer
        num_sms = (torch.cuda.get_device_properties(self.device).multi_processor_count
                   if self.cuda else 148)
        self.scheduler = Scheduler(self.kv.allocator, ecfg.block_size, ecfg.max_num_seqs,
                                   ecfg.max_num_batched_tokens, ecfg.max_model_len,
                                   ecfg.enable_chunked_prefill, cache_key=self._cache_key)
        self.runner = ModelRunner(self.model, ecfg.block_size, self.device, num_sms,
                                  max_model_len=ecfg.max_model_len, decode_graphs=not ecfg.enforce_eager)
        # Backward collectives use their own communicator: forward and backward
        # run on different streams and must never share an NCCL queue.
        self.bwd_comm = comm
        if comm is not None and comm.size > 1:
            import torch.distributed as dist
            from ..parallel.comm import TPComm
            from ..parallel.comm import new_backward_group
            self.bwd_comm = new_backward_group(comm)
        self._actions: list = []
        self._actions_lock = threading.Lock()
        # Step plans reach the follower ranks through shared memory (a memory
        # copy per step); DSERVE_TP_PLAN_CHANNEL=gloo sends them through the
        # process group instead.
        self.plan_chan = None
        if comm is not None and comm.size > 1 and os.environ.get("DSERVE_TP_PLAN_CHANNEL", "shm") == "shm":
            from ..parallel.shm_channel import ChannelUnavailable, ShmChannel
            try:
                self.plan_chan = ShmChannel(comm)
            except ChannelUnavailable as e:
                dprint(f"[tp] {e}; step plans go through the process group")
        self.estimator = MergedExecutionEstimator()
        self.estimator.set_margin(self.ftcfg.admission_margin, self.ftcfg.admission_margin_k)
        self.estimator.split_mixed = bool(self.ftcfg.graph_ft_batches)
        self.tracker = StepLog()
        self.tbt_window = DecodeGapWindow(self.ftcfg.avg_tbt_window_s) if self.ftcfg.avg_tbt_window_s > 0 else None
        self.coord = FinetuneCoordinator(cap_tokens, ft_started=self.ftcfg.start_on_launch,
                                         bwd_log_path=self.ftcfg.bwd_log_path)
        self.jobs = FtJobManager()
        self.store = ft_store
        self.trainer: LoraTrainer | None = None
        if self.ft_enabled:
            self.ft_slot = n_slots - 1
            self.adapter_slots[FT_ADAPTER_NAME] = self.ft_slot
            self.runner.ft_slot = self.ft_slot
            self._init_finetuning(ft_adapter)
        # ---- the backward's residual-gradient reductions over peer memory
        self.bwd_ws = None
        self.opt_ws = None
        if (self.cuda and comm is not None and comm.size > 1 and ecfg.tp_comm == "fused"
                and self.trainer is not None and self.capture is not None):
            from ..parallel.peer import BwdPeerWorkspace
            self.bwd_ws = BwdPeerWorkspace(comm, cap_tokens + 8, self.arch.hidden)
            if self._self_test_bwd(comm):
                self.trainer.bwd.tpws = self.bwd_ws
                # ... and the replicated factors' optimizer over peer memory
                from ..parallel.peer import OptPeerWorkspace
                m = self.trainer.masters
                self.opt_ws = OptPeerWorkspace(comm, m.rep_total, self.arch.num_layers)
                self.trainer.optws = self.opt_ws
            else:
                self.bwd_ws.close()
                self.bwd_ws = None
        # Every rank builds with the same constructor adapters; later loads
        # are made by the driver and replayed by the followers.
        self._replicate = False
        for name, spec in (adapters or {}).items():
            self.load_inference_adapter(name, **spec)
        self._replicate = True
        # ---- streams: forward high priority, backward low priority
        if self.cuda:
            self.fwd_stream = torch.cuda.Stream(self.device, priority=-2)
            self.bwd_stream = torch.cuda.Stream(self.device, priority=0)
        else:
            self.fwd_stream = self.bwd_stream = None
        # Backward layers are CUDA-graph replays enqueued inline by this thread
        # (a background feeder thread loses the GIL to the serving loop after
        # every PyTorch call, so the work stays on the engine thread).
        self._bwd_remaining = 0
        self._bwd_gen = None
        self._bwd_events: deque = deque()
        self._bwd_done_evt = None
        self._bwd_meta: dict | None = None
        self._bwd_result = None
        self._publish_evt = None
        self._pending_timing: deque[StepRecord] = deque()
        self.requests: dict[str, Request] = {}
        self.finished: list[Request] = []
        self.step_no = 0
        self.profiling = False
        self.last_admit = None
        # Host seconds per step phase (rank 0), for the bench's breakdown.
        self.host_s: dict[str, float] = {}
        self.stats = {"ft_tokens_forwarded": 0, "ft_tokens_trained": 0, "steps": 0,
                      "bwd_layers": 0, "h2d_bytes": 0, "d2h_bytes": 0}
        self.arrival_flag = False
        self._forced_ft = None
        if self.cuda:
            torch.cuda.synchronize(self.device)
        self.init_s = time.perf_counter() - t0
        self.step_listeners: list = []
        self.request_listeners: list = []
        self.backward_listeners: list = []
        self.metrics = None
        self.step_trace = None
        self.router = None
        self._job_owner = None
        if self.is_driver and (self.ftcfg.metrics_dir or self.ftcfg.step_trace_path):
            self.start_telemetry(self.ftcfg.metrics_dir)
        if self.ftcfg.print_weight_hash:
            dprint(f"[weights] rank {self.tp.rank} hash {self.weight_hash():.6e}")
        if self.ftcfg.backward_mps_percentage and self.trainer is not None and self.cuda:
            # The backward is a low-priority stream of this process, not an MPS
            # client: its share of the GPU becomes a cap on its GEMM grids.
            sms = torch.cuda.get_device_properties(self.device).multi_processor_count
            self.trainer.bwd.set_sm_share(float(self.ftcfg.backward_mps_percentage), sms)

    # ------------------------------------------------------------------ setup
    def _alloc_kv(self) -> KVCache:
        e = self.ecfg
        hkv = self.arch.num_kv_heads // self.tp.size
        per_block = KVCache.bytes_per_block(self.arch.num_layers, hkv, e.block_size,
                                            self.arch.head_dim, 2 if self.cuda else 4)
        if e.num_gpu_blocks_override:
            nb = e.num_gpu_blocks_override
        elif self.cuda:
            free, total = torch.cuda.mem_get_info(self.device)
            reserve = total * (1 - e.gpu_memory_utilization) + 6 * (1 << 30)  # workspaces
            nb = int(max(0, free - reserve) // per_block)
            # Enough for max_num_seqs full contexts is plenty.
            nb = min(nb, e.max_num_seqs * -(-e.max_model_len // e.block_size) + 64)
        else:
            nb = 4 * (-(-e.max_model_len // e.block_size)) + 16
        if self.comm is not None and self.comm.size > 1:
            # Rank 0 hands out page ids for every rank: all ranks must hold the
            # same number of pages (the smallest any rank can afford).
            nb = -self.comm.all_reduce_max_int(-nb)
        if nb < 2:
            raise MemoryError("no room for the KV cache")
        return KVCache(self.arch.num_layers, nb, hkv, e.block_size, self.arch.head_dim, self.device,
                       self.dtype, prefix_caching=e.enable_prefix_caching)

    def _check_stop_strings(self, out, now: float) -> list:
        """Requests whose decoded output now contains one of their stop strings."""
        ended = []
        for s in out.decode + out.prefill:
            r = s.req
            if (not r.params.stop or r.finished() or not s.sample or not r.output_ids
                    or len(r.output_ids) < r.params.min_tokens):
                continue
            text = self.tokenizer.decode(r.output_ids)
            hit = next((st for st in r.params.stop if st and st in text), None)
            if hit is not None:
                r.stop_reason = hit
                self.scheduler.finish(r, now)
                ended.append(r)
        return ended

    def _cache_key(self, req: Request):
        """What besides the tokens shaped a request's K/V, for prefix caching:
        its LoRA slot and the slot's load version. Requests on the adapter
        being trained never share pages (its weights change every cycle)."""
        slot = req.lora_slot
        if slot < 0:
            return (-1, 0)
        if slot == self.ft_slot:
            return None
        return (slot, self.lora.version[slot] if self.lora is not None else 0)

    def _init_finetuning(self, ft_adapter) -> None:
        from ..adapters import peft_io
        cfg = self.ftcfg
        tensors, rank, alpha, acfg = None, self.ecfg.max_lora_rank, 2.0 * self.ecfg.max_lora_rank, None
        if ft_adapter is not None:
            tensors, rank, alpha = ft_adapter
        elif cfg.finetuning_lora_path and os.path.isfile(
                os.path.join(cfg.finetuning_lora_path, peft_io.CONFIG_FILE)):
            tensors, acfg = peft_io.read_adapter(cfg.finetuning_lora_path)
            rank, alpha = peft_io.adapter_rank_alpha(acfg)
        self.trainer = LoraTrainer(self.weights, self.lora, self.ft_slot, rank, alpha,
                                   lr=cfg.learning_rate, weight_decay=cfg.weight_decay,
                                   gamma=cfg.gamma, comm=self.bwd_comm, mask_prefix=cfg.loss_mask_prefix,
                                   targets=cfg.ft_target_modules, adapter_config=acfg,
                                   cos_sin_table=self.model_cos_sin())
        self.trainer.use_graphs = self.cuda and bool(cfg.backward_cuda_graph)
        if cfg.backward_fp32 and self.cuda:
            dprint("[config] backward_fp32 is not available on the sm_100a path: backward GEMMs "
                   "take bf16 operands with fp32 accumulation (masters, norms, softmax and the "
                   "LM head stay fp32)")
        if tensors:
            self.trainer.load_adapter(tensors, rank, alpha)
        else:
            self.trainer.init_random(self.ecfg.seed + 1)
        self.trainer.publish()
        self.adapter_meta[FT_ADAPTER_NAME] = {"rank": rank, "alpha": alpha, "trainable": True}
        if self.store is None:
            tok = self.tokenizer.encode if self.tokenizer is not None else None
            self.store = FinetuningStore(cfg.data_path, tok, FT_ADAPTER_NAME, cfg.num_epochs,
                                         cfg.max_saved_finetuning_tokens, cfg.max_prepare)
            if cfg.data_path:
                self.store.load()
        self.coord.min_sample_len = max(1, self.store.min_len() or 1)
        self.admission = FinetuneAdmission(cfg, self.estimator, self.coord, self.store,
                                           self.ecfg.max_num_batched_tokens, self.tbt_window)
        self.jobs.submit(FinetuneJobSpec.from_finetune_config(cfg), self.rcfg.enable_adapter_routing)

    def _self_test_fused(self, comm) -> bool:
        """Check the fused GEMM + all-reduce against GEMM + NCCL on this
        machine's ranks before serving with it (every rank takes the same
        decision: the verdict is the MIN over ranks). A failure falls back to
        the NCCL path for the whole run."""
        import torch.distributed as dist
        ok = 1
        try:
            g = torch.Generator(device=self.device).manual_seed(1234 + comm.rank)
            for M in (3, 200):
                K = 256
                a = torch.randn(M, K, generator=g, device=self.device).to(self.dtype)
                b = (torch.randn(self.arch.hidden, K, generator=g, device=self.device) * 0.05).to(self.dtype)
                fused = ops.gemm_ar(a, b, self.peer_ws).float().clone()
                ref = a.float() @ b.float().t()
                dist.all_reduce(ref, group=comm.group)
                err = float((fused - ref).abs().max()) / max(1e-6, float(ref.abs().max()))
                if not err < 2e-2:
                    ok = 0
            torch.cuda.synchronize(self.device)
            if ops.check_device_error() != 0:
                ok = 0
        except Exception as e:  # a failing launch must not take serving down
            dprint(f"[tp] fused all-reduce self-test raised {e!r}")
            ok = 0
        ok = -comm.all_reduce_max_int(-ok)
        if not ok:
            dprint("[tp] fused GEMM + all-reduce failed its self-test: using GEMM + NCCL")
        return bool(ok)

    def _setup_embed_peer(self, comm) -> None:
        """Move this rank's embedding shard into peer-mapped memory and check
        the peer-read embedding against embedding + NCCL all-reduce (the MIN
        over ranks decides; a failure keeps the all-reduce path)."""
        from ..parallel.peer import PeerTable
        w = self.weights
        tied = w.lm_head.data_ptr() == w.embed.data_ptr()
        ok = 1
        pt = None
        try:
            pt = PeerTable(comm, w.embed, self.arch.vocab)
            vl, V = w.v_local, self.arch.vocab
            ids = torch.tensor([0, vl - 1, vl, V - 1, (V * 7) // 13, -1], dtype=torch.int64, device=self.device)
            ref = torch.empty(ids.numel(), self.arch.hidden, dtype=self.dtype, device=self.device)
            ops.embedding(ids, w.embed, ref, comm.rank * vl)
            comm.all_reduce(ref)
            got = torch.empty_like(ref)
            ops.embedding_peer(ids, pt, got)
            torch.cuda.synchronize(self.device)
            if not torch.equal(ref, got) or ops.check_device_error() != 0:
                ok = 0
        except Exception as e:  # a failing setup must not take serving down
            dprint(f"[tp] peer embedding setup raised {e!r}")
            ok = 0
        ok = -comm.all_reduce_max_int(-ok)
        if ok and pt is not None:
            w.embed = pt.local
            if tied:
                w.lm_head = pt.local
            self.embed_peer = pt
        else:
            if pt is not None:
                pt.close()
            dprint("[tp] peer embedding failed its self-test: embedding + NCCL all-reduce")

    def _self_test_bwd(self, comm) -> bool:
        """Check the backward's push + reduce over peer memory against a GEMM
        and an NCCL all-reduce before training with it (the decision is the
        MIN over ranks; a failure keeps the NCCL path for the whole run)."""
        import torch.distributed as dist
        ok = 1
        try:
            g = torch.Generator(device=self.device).manual_seed(4321 + comm.rank)
            D = self.arch.hidden
            for M in (8, 300):
                a = torch.randn(M, 192, generator=g, device=self.device).to(self.dtype)
                b = (torch.randn(192, D, generator=g, device=self.device) * 0.05).to(self.dtype)
                out = torch.zeros(M, D, dtype=torch.float32, device=self.device)
                ops.gemm_push(a, b, self.bwd_ws)
                got = ops.tp_reduce_rows(self.bwd_ws, M, 0, out).float().clone()
                ref = a.float() @ b.float()
                dist.all_reduce(ref, group=comm.group)
                err = float((got - ref).abs().max()) / max(1e-6, float(ref.abs().max()))
                if not err < 2e-2:
                    ok = 0
            torch.cuda.synchronize(self.device)
            if ops.check_device_error() != 0:
                ok = 0
        except Exception as e:  # a failing launch must not take serving down
            dprint(f"[tp] backward peer reduction self-test raised {e!r}")
            ok = 0
        ok = -comm.all_reduce_max_int(-ok)
        if not ok:
            dprint("[tp] backward peer reduction failed its self-test: using NCCL all-reduces")
        return bool(ok)

    def weight_hash(self) -> float:
        """Order-sensitive checksum of this rank's base weights (debug)."""
        h = 0.0
        for i, t in enumerate([self.weights.embed] + [getattr(L, f) for L in self.weights.layers
                                                      for f in ("qkv", "o", "gate_up", "down")]):
            h += (i + 1) * float(t.float().flatten()[:: max(1, t.numel() // 4096)].double().sum())
        return h

    def begin_job(self, job) -> bool:
        """Switch finetuning to ``job`` (its init stage). The launch job is
        already loaded. A later job waits until nothing of the previous one is
        in flight, then re-initialises the trainable adapter (its PEFT
        directory, or ``adapter_init`` random/zeros) with the job's optimiser
        settings and loads its corpus. The adapter rank stays the trainer's:
        the masters, graphs and slot keep their shapes."""
        if job.data.get("begun"):
            return True
        if self._job_owner is None:
            self._job_owner = job.job_id
            job.data["begun"] = True
            return True
        if (self.coord.fill_count or self.coord.reserved_fill or self.coord.pending_backward
                or self.bwd_active or self._bwd_done_evt is not None):
            return False
        spec = job.spec
        if spec.adapter_path and os.path.isdir(spec.adapter_path):
            from ..adapters import peft_io
            _, acfg = peft_io.read_adapter(spec.adapter_path)
            r, _ = peft_io.adapter_rank_alpha(acfg)
            if r != self.trainer.rank_r:
                raise ValueError(f"job adapter rank {r} != the trainer's rank {self.trainer.rank_r}")
        action = ("job", spec.adapter_path, spec.adapter_init, spec.learning_rate, spec.weight_decay,
                  spec.gamma, self.ecfg.seed + 1 + job.job_id)
        if self.tp_size > 1:
            self._record(action)
            self._flush_actions()
        self._apply_job(*action[1:])
        tok = self.tokenizer.encode if self.tokenizer is not None else None
        store = FinetuningStore(spec.data_path, tok, FT_ADAPTER_NAME, spec.num_epochs,
                                self.ftcfg.max_saved_finetuning_tokens, self.ftcfg.max_prepare)
        if spec.data_path:
            store.load()
        self.store = self.admission.store = store
        self.coord.min_sample_len = max(1, store.min_len() or 1)
        self._job_owner = job.job_id
        job.data["begun"] = True
        dprint(f"[ft-job] {spec.name}: {len(store)} samples, lr {spec.learning_rate}")
        return True

    def _apply_job(self, adapter_path, adapter_init, lr, wd, gamma, seed) -> None:
        tr = self.trainer
        if self.cuda:
            torch.cuda.synchronize(self.device)
        if adapter_path and os.path.isdir(adapter_path):
            from ..adapters import peft_io
            tensors, acfg = peft_io.read_adapter(adapter_path)
            tr.load_adapter(tensors, *peft_io.adapter_rank_alpha(acfg))
        else:                  # no checkpoint: PEFT init (A random, B zero)
            tr.init_random(seed)
        tr.lr, tr.wd, tr.gamma = lr, wd, gamma
        tr.epoch, tr.total_tokens, tr.losses = 0, 0, []
        tr.publish()
        if self.cuda:
            torch.cuda.synchronize(self.device)

    def model_cos_sin(self):
        from ..ops.reference import rope_cos_sin_table
        return rope_cos_sin_table(max(self.arch.max_position, 8192), self.arch.head_dim,
                                  self.arch.rope_theta, self.arch.rope_scaling, device=self.device)

    def load_inference_adapter(self, name: str, path: str | None = None, tensors=None,
                               rank: int | None = None, alpha: float | None = None,
                               seed: int | None = None) -> int:
        """Put an inference LoRA into a free slot (PEFT dir, tensors, or random).
        With TP the driver records the load so every rank writes the same
        slot at the same point of the step sequence."""
        from ..adapters import peft_io
        if self.lora is None:
            raise RuntimeError("LoRA is disabled (enable_lora: false)")
        if name in self.adapter_slots:
            return self.adapter_slots[name]
        used = set(self.adapter_slots.values())
        free = [s for s in range(self.lora.slots) if s not in used]
        if not free:
            raise RuntimeError("no free LoRA slot (raise max_loras)")
        slot = free[0]
        explicit = tensors is not None
        if tensors is None and path is not None:
            tensors, acfg = peft_io.read_adapter(path)
            rank, alpha = peft_io.adapter_rank_alpha(acfg)
        elif tensors is None:
            rank = rank or self.ecfg.max_lora_rank
            alpha = alpha if alpha is not None else 2.0 * rank
            seed = seed if seed is not None else 1000 + slot
            tensors = random_adapter(self.arch, rank, seed)
        if self.is_driver and self.tp_size > 1 and self._replicate:
            # Followers re-read the PEFT directory or regenerate the seeded
            # adapter; only tensors with neither source travel in the action.
            payload = None if (path is not None or not explicit) else tensors
            self._record(("adapter_load", slot, path, rank, alpha, seed, payload))
            self._flush_actions()
        self._write_slot(slot, tensors, rank, alpha)
        self.adapter_slots[name] = slot
        self.adapter_meta[name] = {"rank": rank, "alpha": alpha, "path": path}
        return slot

    def _write_slot(self, slot: int, tensors, rank: int, alpha: float) -> None:
        if self.cuda:
            # In-flight forwards may read other slots of the same buffers;
            # the write goes after everything queued so far.
            torch.cuda.synchronize(self.device)
        self.lora.load_slot(slot, tensors, rank, alpha)
        if self.cuda:
            torch.cuda.synchronize(self.device)

    def unload_inference_adapter(self, name: str) -> int:
        if name == FT_ADAPTER_NAME:
            raise ValueError("the trainable adapter cannot be unloaded")
        slot = self.adapter_slots.pop(name, None)
        if slot is None:
            raise KeyError(f"adapter {name!r} is not loaded")
        if self.is_driver and self.tp_size > 1 and self._replicate:
            self._record(("adapter_clear", slot))
            self._flush_actions()
        self._clear_slot(slot)
        self.adapter_meta.pop(name, None)
        return slot

    def _clear_slot(self, slot: int) -> None:
        if self.cuda:
            torch.cuda.synchronize(self.device)
        self.lora.clear_slot(slot)
        if self.cuda:
            torch.cuda.synchronize(self.device)

    def _save_trainer(self, path: str, save_id: str = "", extra: dict | None = None,
                      background: bool = False, after=None) -> str | None:
        """PEFT save of the trained adapter, merged across TP ranks (every
        rank takes part in the gather, so the driver records it first)."""
        if self.is_driver and self.tp_size > 1:
            self._record(("save",))
            self._flush_actions()
        if self.cuda:
            torch.cuda.synchronize(self.device)
        return self.trainer.save_adapter(path, save_id, extra, background=background, after=after)

    # ------------------------------------------------------------------ requests
    def add_request(self, request_id: str, prompt_ids: list[int], params: SamplingParams | None = None,
                    adapter: str | None = None, arrival_time: float | None = None) -> Request:
        r = Request(request_id, list(prompt_ids), params or SamplingParams(), adapter,
                    arrival_time if arrival_time is not None else time.perf_counter())
        if adapter is not None:
            if adapter not in self.adapter_slots:
                raise KeyError(f"unknown adapter {adapter!r}")
            r.lora_slot = self.adapter_slots[adapter]
        self.scheduler.add(r)
        self.requests[request_id] = r
        if self.ftcfg.print_engine_req_recv:
            dprint(f"[req] {request_id}: {len(r.prompt_ids)} prompt tokens, max {r.params.max_tokens}, "
                   f"adapter {adapter}")
        self.coord.note_arrival(r.arrival_time)
        self.arrival_flag = True
        for cb in self.request_listeners:
            cb("add", r)
        return r

    def abort_request(self, request_id: str) -> bool:
        if self.router is not None and self.router.cancel(request_id):
            return True
        r = self.scheduler.abort(request_id)
        if r is not None:
            self.requests.pop(request_id, None)
            r.finish_time = time.perf_counter()
            for cb in self.request_listeners:
                cb("abort", r)
        return r is not None

    def has_unfinished(self) -> bool:
        return self.scheduler.has_unfinished() or (self.router is not None and self.router.has_pending())

    # ------------------------------------------------------------------ control
    def start_finetuning(self) -> None:
        self.coord.start()

    def stop_finetuning(self) -> None:
        self.coord.stop()

    def finetuning_status(self) -> dict:
        st = self.coord.status()
        st.update({"enabled": self.ft_enabled,
                   "trainer_step": self.trainer.step if self.trainer else 0,
                   "store_untrained": self.store.num_untrained() if self.store else 0,
                   "store_epoch": self.store.current_epoch if self.store else 0,
                   "losses_tail": self.trainer.losses[-8:] if self.trainer else [],
                   "jobs": self.jobs.status()})
        return st

    def save_adapter(self, path: str | None = None, save_id: str = "", background: bool = False) -> str | None:
        if self.trainer is None:
            raise RuntimeError("finetuning is not enabled")
        if path is None:
            if not self.ftcfg.adapter_save_path:
                raise ValueError("no path given and finetune_param.adapter_save_path is unset")
            path = os.path.join(self.ftcfg.adapter_save_path, f"manual-{int(time.time())}")
        self._drain_backward()
        return self._save_trainer(path, save_id, background=background)

    def _load_weights(self, ecfg: EngineConfig):
        """Base weights: the model directory's safetensors checkpoint (this
        rank's shards only) or the seeded random initialisation."""
        from ..models.loader import checkpoint_files, load_hf_weights
        fmt = ecfg.load_format
        if fmt not in ("auto", "safetensors", "dummy"):
            raise ValueError(f"load_format must be auto, safetensors or dummy, got {fmt!r}")
        files = [] if fmt == "dummy" else checkpoint_files(ecfg.model)
        if fmt == "safetensors" and not files:
            raise FileNotFoundError(f"load_format=safetensors but {ecfg.model!r} has no *.safetensors")
        # The finetuning head works on the serving head's vocabulary shard:
        # no full copy of the LM head is kept.
        keep = False
        if files:
            dprint(f"loading {len(files)} safetensors file(s) from {ecfg.model} (tp rank {self.tp.rank})")
            return load_hf_weights(self.arch, ecfg.model, self.tp, device=self.device, dtype=self.dtype,
                                   keep_full_head=keep)
        return init_weights(self.arch, self.tp, seed=ecfg.seed, device=self.device, dtype=self.dtype,
                            keep_full_head=keep)

    # ------------------------------------------------------------------ estimator state
    def save_estimator_state(self, path: str | None = None) -> str | None:
        """Estimator coefficients plus the tracker's step samples as one JSON
        file, written atomically; with no ``path`` the configured
        ``estimator_state_save_path`` is used once (shutdown). Reference:
        ``deltaserve-plugin/deltaserve/ft_scheduler.py:1131-1156``."""
        if path is None:
            path = self.ftcfg.estimator_state_save_path
            if not path or getattr(self, "_estimator_state_saved", False):
                return None
            self._estimator_state_saved = True
        self._drain_timing(block=True)
        state = {"version": 1, "estimator": self.estimator.export_state(),
                 "tracker": self.tracker.export_state()}
        from ..adapters.peft_io import write_json_atomic
        write_json_atomic(path, state, indent=None)
        dprint(f"[estimator] state saved to {path}: {self.tracker.size()} samples")
        return path

    def load_estimator_state(self, path: str | None = None) -> bool:
        """Replace the fitted estimator with a saved state (after the launch
        profile, which still runs to warm the finetuning paths). A missing file
        is a warning, not an error (first run of a replayed trace)."""
        path = path or self.ftcfg.estimator_state_load_path
        if not path:
            return False
        if not os.path.isfile(path):
            dprint(f"[estimator] estimator_state_load_path={path} does not exist; "
                   "keeping the launch-time profile")
            return False
        with open(path) as f:
            state = json.load(f)
        self.tracker.import_state(state["tracker"])
        self.estimator.import_state(state["estimator"])
        dprint(f"[estimator] state restored from {path}: {self.tracker.size()} samples")
        return True

    # ------------------------------------------------------------------ telemetry
    def start_telemetry(self, metrics_dir: str | None = None) -> None:
        """Attach the run recorder (CSV/JSONL outputs when ``metrics_dir`` is
        set, live feed only otherwise) and, if configured, the step trace."""
        from ..utils.metrics import MetricsRecorder
        from ..utils.step_trace import attach_step_trace
        self.stop_telemetry()
        cfg = self.ftcfg
        self.metrics = MetricsRecorder(self, metrics_dir, cfg.metrics_interval_s, cfg.steps_log_max_mb,
                                       rank=self.tp.rank)
        if cfg.step_trace_path and self.step_trace is None:
            self.step_trace = attach_step_trace(self, cfg.step_trace_path)

    def stop_telemetry(self) -> None:
        m = self.metrics
        if m is None:
            return
        self.metrics = None
        for lst, cb in ((self.step_listeners, m.on_step), (self.request_listeners, m.on_request),
                        (self.backward_listeners, m.on_backward)):
            if cb in lst:
                lst.remove(cb)
        m.close()

    # ------------------------------------------------------------------ adapters
    def adapter_op(self, name: str, op: str):
        """Adapter lifecycle by name. With adapter routing the pool owns the
        lifecycle (``load``/``offload``/``retire``/``reactivate``/``pin``/
        ``unpin``/``remove``); without it ``unload``/``remove`` free the slot
        and ``load`` re-reads the adapter's path."""
        if self.router is not None and name in self.router.pool:
            return self.router.pool.op(name, op)
        if op in ("unload", "remove"):
            return {"slot": self.unload_inference_adapter(name)}
        if op == "load":
            meta = self.adapter_meta.get(name) or {}
            if not meta.get("path"):
                raise KeyError(f"adapter {name!r} has no known path")
            return {"slot": self.load_inference_adapter(name, path=meta["path"])}
        raise ValueError(f"unknown adapter op {op!r} (load, unload, remove)")

    # ------------------------------------------------------------------ stepping
    def _ft_rows_in(self, out: SchedulerOutput) -> int:
        return sum(s.num_new for s in out.ft)

    def _earliest_waiting_arrival(self, out: SchedulerOutput) -> float | None:
        t = [s.req.arrival_time for s in out.prefill if s.req.first_token_time is None]
        t += [r.arrival_time for r in self.scheduler.waiting]
        return min(t) if t else None

    def _drain_timing(self, block: bool = False) -> None:
        while self._pending_timing:
            rec = self._pending_timing[0]
            if self.cuda:
                if not block and not rec.end.query():
                    return
                dur = rec.start.elapsed_time(rec.end) / 1e3
            else:
                dur = rec.end - rec.start
            self._pending_timing.popleft()
            self.tracker.add(rec.features, dur, rec.predicted)
            for cb in self.step_listeners:
                cb(rec, dur)
            if self.tracker.due_for_refit():
                self.estimator.data_fit(self.tracker)

    def _host(self, phase: str, t0: float) -> float:
        """Accumulate host seconds of a step phase since ``t0``; returns now."""
        t = time.perf_counter()
        self.host_s[phase] = self.host_s.get(phase, 0.0) + (t - t0)
        return t

    def step(self) -> list[Request]:
        """One engine step (rank 0). Returns requests that finished."""
        now = time.perf_counter()
        self.step_no += 1
        self._drain_timing()
        self._poll_backward()
        if self.router is not None:
            self.router.tick()          # encode step + slot placement of routed requests
        cfg = self.ftcfg
        if self.ft_enabled:
            if cfg.rps_throttle_enable:
                self.coord.check_rps_throttle(now, cfg.rps_throttle_close_rps, cfg.rps_throttle_open_rps,
                                              cfg.rps_throttle_window_s, cfg.rps_throttle_close_time)
            self.coord.check_stuck(True)
            self.jobs.tick(self)
            if self.coord.try_flush():
                self._start_backward()
        t_h = self._host("housekeeping", now)
        out = self.scheduler.schedule()
        t_h = self._host("schedule", t_h)
        if self.ftcfg.print_scheduler_add and out.prefill:
            dprint(f"[sched] step {self.step_no}: prefill {[s.num_new for s in out.prefill]} "
                   f"decode {len(out.decode)}")
        bwd_busy = self.bwd_active or self._bwd_done_evt is not None
        adm = None
        ft_dst = 0
        if self.profiling and getattr(self, "_forced_ft", None):
            self.scheduler.add_ft(out, self._forced_ft)
            self._forced_ft = None
        if self.ft_enabled and not self.profiling:
            adm = self.admission.admit(out, self._earliest_waiting_arrival(out), now,
                                       bwd_in_flight=bwd_busy)
            self.last_admit = adm
            if adm.samples:
                reqs = [Request(f"__ft__{s.request_id[:8]}_{self.step_no}", s.prompt_ids,
                                SamplingParams(max_tokens=1), FT_ADAPTER_NAME, now, is_ft=True,
                                ft_sample=s) for s in adm.samples]
                rejected = self.scheduler.add_ft(out, reqs)
                if rejected:
                    self.store.release_claimed([r.ft_sample for r in rejected])
                kept = [s.req.ft_sample for s in out.ft]
                ft_dst = self.coord.reserve(self._ft_rows_in(out), kept)
                nxt = self.store.pop_next()
                self.coord.note_injection(nxt.input_len if nxt else None)
            # Tier B: an FT-only step about to run while an arrival is pending.
            if (cfg.forward_interruptible and out.ft and not out.decode and not out.prefill
                    and self.scheduler.waiting):
                self._rollback_ft(out)
            # Tier A: before an FT-only step, give a request that is arriving
            # right now (flagged by the HTTP thread) a short grace to join.
            elif (cfg.forward_interruptible and cfg.ft_only_admission_grace_ms > 0 and out.ft
                  and not out.decode and not out.prefill):
                t_end = time.perf_counter() + cfg.ft_only_admission_grace_ms / 1e3
                while not self.arrival_flag and time.perf_counter() < t_end:
                    time.sleep(0.0002)
                if self.arrival_flag:
                    self._rollback_ft(out)
        t_h = self._host("admission", t_h)
        if out.is_empty():
            self._advance_backward(idle=not self.has_unfinished())
            self._flush_actions()
            self._host("backward_feed", t_h)
            return []
        return self._run(out, ft_dst, bwd_busy)

    def _rollback_ft(self, out: SchedulerOutput) -> None:
        reqs = self.scheduler.rollback_ft(out)
        samples = [r.ft_sample for r in reqs]
        self.coord.unreserve(sum(r.num_prompt for r in reqs), samples)
        self.store.release_claimed(samples)

    def _run(self, out: SchedulerOutput, ft_dst: int, bwd_busy: bool,
             record_capture: bool = True) -> list[Request]:
        feats = StepFeatures(t_in=float(out.t_in), p=len(out.prefill) + len(out.ft),
                             t_ft=float(out.t_ft), b_d=out.b_d, k=float(out.k_decode),
                             prefill_lens=out.prefill_lens() or None, bwd=bwd_busy)
        pred = self.estimator.predict(feats) if self.estimator.is_ready else None
        # Pause: a step carrying inference prefill stops feeding the backward.
        has_inf_prefill = bool(out.prefill)
        pause_now = has_inf_prefill and (self.ftcfg.pause_on_arrival or self.ftcfg.pause_until_prefill_done
                                         or self.ftcfg.pause_prefill_always)
        # fwd_token_throttle: a large step keeps the backward paused while it runs.
        big_step = (self.ftcfg.fwd_token_throttle_enable
                    and out.t_in + out.b_d >= self.ftcfg.fwd_token_throttle)
        pause_now = pause_now or big_step
        # Queue backward layers while the forward runs (before the host blocks
        # on the sampled tokens); the low-priority stream fills GPU gaps.
        feed = (lambda: self._advance_backward(idle=False, paused=pause_now)) \
            if (self.cuda and not self.profiling) else None
        uses_ft_slot = bool(out.ft) or any(s.req.lora_slot == self.ft_slot for s in out.seqs
                                           if self.ft_slot >= 0)
        if self.ftcfg.print_engine_batch_exec or self.ftcfg.print_step_mode:
            mode = ("ft-only" if out.ft and not (out.prefill or out.decode) else
                    "mixed" if out.ft else "prefill" if out.prefill else "decode")
            dprint(f"[batch-exec] step {self.step_no} mode={mode} decode={len(out.decode)} "
                   f"prefill={len(out.prefill)} ft={len(out.ft)} t_in={out.t_in} t_ft={out.t_ft} "
                   f"bwd={'busy' if bwd_busy else 'idle'} pred_ms="
                   f"{'-' if pred is None else round(pred * 1e3, 3)}")
        # Tier C: an FT-only step is abandoned between layers if a request
        # arrives meanwhile (every rank stops at the same layer).
        abort_check = ((lambda: self.arrival_flag)
                       if (self.ftcfg.forward_interruptible and not self.profiling and self.ft_enabled) else None)
        self.runner.eos_ids = self.eos_ids()
        vote = self._abort_vote() if self.tp_size > 1 else None
        t_h = time.perf_counter()
        if self.cuda:
            with torch.cuda.stream(self.fwd_stream):
                if uses_ft_slot and self._publish_evt is not None:
                    self.fwd_stream.wait_event(self._publish_evt)
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record()
                toks, _ = self.runner.execute(out, self.capture, ft_dst, self._plan_hook(bool(out.ft)),
                                              before_sample=feed, abort_check=abort_check, vote=vote)
                ev1.record()
        else:
            ev0 = time.perf_counter()
            toks, _ = self.runner.execute(out, self.capture, ft_dst, self._plan_hook(bool(out.ft)),
                                          before_sample=feed, abort_check=abort_check, vote=vote)
            ev1 = time.perf_counter()
        t_h = self._host("execute", t_h)
        for name, v in zip(("exec_pack_plan", "exec_enqueue", "exec_backward_feed", "exec_sample_wait"),
                           self.runner.last_phases):
            self.host_s[name] = self.host_s.get(name, 0.0) + v
        if self.runner.last_aborted:
            # Partial captures and KV pages of the FT rows are simply released.
            self._rollback_ft(out)
            self.stats["ft_aborts"] = self.stats.get("ft_aborts", 0) + 1
            self.arrival_flag = False
            return []
        if not out.prefill and not out.ft:
            self.stats["decode_steps"] = self.stats.get("decode_steps", 0) + 1
            self.stats["decode_enqueue_s"] = (self.stats.get("decode_enqueue_s", 0.0)
                                              + getattr(self.runner, "last_enqueue_s", 0.0))
        self.stats["h2d_bytes"] += self.runner.last_h2d_bytes
        self.stats["d2h_bytes"] += self.runner.last_d2h_bytes
        self._pending_timing.append(StepRecord(feats, ev0, ev1, pred, "step"))
        now = time.perf_counter()
        done = self.scheduler.update(out, toks, now, eos_id=self.eos_ids())
        if self.tokenizer is not None:
            done.extend(self._check_stop_strings(out, now))
        self.stats["steps"] += 1
        if self.tbt_window is not None:
            self.tbt_window.note_step(now, out.b_d, bool(self.scheduler.running))
        if out.ft and (self.profiling or not record_capture):
            pass  # profiling FT rows: captured at offset 0, never trained
        elif out.ft:
            n = self._ft_rows_in(out)
            self.stats["ft_tokens_forwarded"] += n
            if self.coord.record_capture(n, [s.num_new for s in out.ft]):
                self._start_backward(capture_evt=ev1 if self.cuda else None)
        for r in done:
            self.requests.pop(r.request_id, None)
            for cb in self.request_listeners:
                cb("finish", r)
        self.finished.extend(done)
        self.arrival_flag = False
        t_h = self._host("update", t_h)
        pause = has_inf_prefill and (self.ftcfg.pause_on_arrival or self.ftcfg.pause_until_prefill_done
                                     or self.ftcfg.pause_prefill_always)
        self._advance_backward(idle=False, paused=(pause and bool(self.scheduler.waiting)) or big_step)
        self._host("backward_feed", t_h)
        if self.ftcfg.validate_estimator:
            self._drain_timing(block=True)      # synchronous: every prediction checked at once
        if self.ftcfg.print_engine_batch_done:
            dprint(f"[batch-done] step {self.step_no}: {len(done)} finished")
        return done

    # ------------------------------------------------------------------ backward
    def _start_backward(self, capture_evt=None) -> None:
        if self.trainer is None:
            return
        if self.capture is None:        # save_activations off: retire the samples untrained
            from .trainer import CycleResult
            self._bwd_meta = {"epoch": self.store.current_epoch if self.store else 0}
            self._bwd_result = CycleResult(float("nan"), int(self.coord.fill_count), 0, 0.0, 0.0,
                                           self.trainer.step)
            self._finish_backward(skip_trainer=True)
            return
        n = self.coord.fill_count
        lens = list(self.coord.sample_lens)
        starts = list(np.cumsum([0] + lens[:-1])) if lens else []
        self._bwd_meta = {"n": n, "starts": [int(s) for s in starts], "lens": lens,
                          "epoch": self.store.current_epoch if self.store else 0}
        if self.cuda:
            if capture_evt is not None:
                self.bwd_stream.wait_event(capture_evt)
            else:
                self.bwd_stream.wait_stream(self.fwd_stream)
        if self.ftcfg.print_activation_hash:
            dprint(f"[activations] cycle {self.coord.cycle}: rows {n} hash "
                   f"{float(self.capture.layer_in[:, :n].float().sum()):.6e}")
        gen = self.trainer.cycle(self.capture, n, self._bwd_meta["starts"], lens,
                                 self._bwd_meta["epoch"], sync=False)
        self._bwd_events.clear()
        self._record(("bwd_start", dict(self._bwd_meta)))
        self._bwd_gen = gen
        # head pieces + one step per layer + the optimizer/publish step
        self._bwd_remaining = self.trainer.num_steps()

    @property
    def bwd_active(self) -> bool:
        return self._bwd_gen is not None

    def _advance_backward(self, idle: bool, paused: bool = False) -> None:
        """Enqueue backward steps on the low-priority stream: all remaining when
        the engine is idle, otherwise until ``backward_run_ahead_boundaries``
        steps are outstanding on the GPU. The number of steps is decided first
        and sent to the follower ranks before any of them runs, so every rank
        issues the backward collectives in the same order."""
        if self._bwd_gen is None or (paused and not idle):
            return
        ahead = max(1, self.ftcfg.backward_run_ahead_boundaries)
        if self.cuda:
            while self._bwd_events and self._bwd_events[0].query():
                self._bwd_events.popleft()
            k = self._bwd_remaining if idle else max(0, ahead - len(self._bwd_events))
        else:
            k = self._bwd_remaining if idle else ahead
        k = min(k, self._bwd_remaining)
        if k <= 0:
            return
        for _ in range(k):
            self._record(("bwd_next",))
        self._flush_actions()
        for _ in range(k):
            self._bwd_remaining -= 1
            try:
                if _FAIL_BACKWARD_AT >= 0 and self.stats["bwd_layers"] >= _FAIL_BACKWARD_AT:
                    raise RuntimeError("injected backward failure (DSERVE_TEST_FAIL_BACKWARD)")
                if self.cuda:
                    with torch.cuda.stream(self.bwd_stream):
                        next(self._bwd_gen)
                        ev = torch.cuda.Event()
                        ev.record()
                    self._bwd_events.append(ev)
                else:
                    next(self._bwd_gen)
                self.stats["bwd_layers"] += 1
            except StopIteration as e:
                self._bwd_result = e.value
                self._bwd_gen = None
                if self.cuda:
                    ev = torch.cuda.Event()
                    ev.record(self.bwd_stream)
                    self._bwd_done_evt = ev
                    self._publish_evt = ev
                else:
                    self._finish_backward()
                break
            except Exception as e:
                self._backward_failed(e)
                break

    def _backward_failed(self, err: Exception) -> None:
        """A backward cycle raised (a host-side error, an allocation failure):
        finetuning is switched off for the rest of the run (sticky), the
        cycle's samples are dropped untrained and inference continues — the
        reference's handling of a failed or dead backward child
        (``deltaserve-plugin/deltaserve/coordinator.py:884-919``). Under TP
        the ranks cannot agree on a half-run cycle, so the error propagates."""
        if self.tp_size > 1:
            raise err
        dprint(f"[engine] backward cycle {self.coord.cycle} failed: {err!r}; finetuning disabled")
        self._bwd_gen = None
        self._bwd_result = None
        self._bwd_done_evt = None
        self._publish_evt = None
        self._bwd_events.clear()
        self._bwd_remaining = 0
        c = self.coord
        c.disable(f"backward failed: {err!r}")
        c.pending_backward = False
        c._t_trigger = None
        c.fill_count = 0
        c.sample_lens = []
        c.buffer_samples = []
        self.stats["bwd_failures"] = self.stats.get("bwd_failures", 0) + 1

    def _poll_backward(self) -> None:
        if self._bwd_done_evt is not None and self._bwd_done_evt.query():
            self._finish_backward()

    def _finish_backward(self, skip_trainer: bool = False) -> None:
        res = (self.trainer.finish_cycle(self._bwd_result) if self.trainer and not skip_trainer
               else self._bwd_result)
        self._bwd_done_evt = None
        meta = self._bwd_meta or {}
        trained = self.coord.backward_done(res.n_tokens, res.loss, res.gpu_ms, res.wall_ms,
                                           meta.get("epoch"))
        if self.store is not None:
            self.store.commit_claimed([s for s in trained if s is not None])
            self.coord.min_sample_len = max(1, self.store.min_len() or 1)
            if not self.store.has_next():
                self.store.advance_epoch()
                self._epoch_ended = True
        self.stats["ft_tokens_trained"] += res.n_tokens
        for cb in self.backward_listeners:
            cb(res)
        self._periodic_save()

    def _periodic_save(self) -> None:
        cfg = self.ftcfg
        if not cfg.adapter_save_path or self.trainer is None:
            return
        from ..adapters import peft_io
        st = self.trainer.step
        if cfg.adapter_save_every_backwards > 0 and st % cfg.adapter_save_every_backwards == 0:
            self._save_trainer(os.path.join(cfg.adapter_save_path, f"backward-{st:06d}"), background=True,
                               after=lambda: peft_io.prune_checkpoints(cfg.adapter_save_path,
                                                                       cfg.adapter_save_keep_last))
        if cfg.adapter_save_every_epoch and getattr(self, "_epoch_ended", False):
            ep = self.store.current_epoch if self.store else 0
            self._save_trainer(os.path.join(cfg.adapter_save_path, f"epoch-{ep:04d}"), background=True,
                               after=lambda: peft_io.prune_checkpoints(cfg.adapter_save_path,
                                                                       cfg.adapter_save_keep_last,
                                                                       prefix="epoch-"))
        self._epoch_ended = False

    def _drain_backward(self) -> None:
        while self._bwd_gen is not None:
            self._advance_backward(idle=True)
        self._flush_actions()
        if self._bwd_done_evt is not None:
            self._bwd_done_evt.synchronize()
            self._finish_backward()

    def synchronize(self) -> None:
        if self.cuda:
            torch.cuda.synchronize(self.device)
        self._drain_timing(block=True)

    # ------------------------------------------------------------------ profiling
    def warm_decode_graphs(self) -> None:
        """Capture the decode-step CUDA graphs of every batch bucket now (on
        every rank in lockstep: the graphs hold TP collectives)."""
        if self.runner.graphs is None or getattr(self, "_graphs_warm", False):
            return
        if self.is_driver and self.tp_size > 1:
            self._record(("decode_graphs",))
            self._flush_actions()
        t0 = time.perf_counter()
        with torch.cuda.stream(self.fwd_stream):
            n = self.runner.graphs.capture_all(self.ecfg.max_num_seqs, self.lora is not None)
        torch.cuda.synchronize(self.device)
        self._graphs_warm = True
        dprint(f"[graphs] {n} decode-step graphs captured in {time.perf_counter() - t0:.1f}s")

    def profile_execution_model(self, shapes=None, repeats: int | None = None,
                                max_shapes: int | None = None) -> None:
        """Launch profiling: drive synthetic shapes through real steps, fit the
        estimator (reference: ``deltaserve-plugin/deltaserve/engine_core.py:242-423``).
        A failure here switches the engine to inference-only (finetuning disabled)."""
        from .profiling import ProfilingShapeGenerator
        repeats = self.ftcfg.profile_num_repeats if repeats is None else repeats
        self.warm_decode_graphs()     # profiled decode steps then run as they will in serving
        try:
            if os.environ.get("DSERVE_TEST_FAIL_PROFILING") == "1":
                raise RuntimeError("DSERVE_TEST_FAIL_PROFILING=1")
            gen = ProfilingShapeGenerator(self.ecfg.max_num_batched_tokens,
                                          self.ftcfg.max_saved_finetuning_tokens,
                                          min(self.ecfg.max_model_len, 4096),
                                          self.store.min_len() if self.store else None)
            warm, rec = gen.prepare(with_ft=self.ft_enabled)
            if shapes is not None:
                rec = shapes
            if max_shapes is not None:
                rec = rec[:max_shapes]
            self.profiling = True
            for sh in warm:
                self._profile_shape(sh, record=False)
            for _ in range(max(1, repeats)):
                for sh in rec:
                    self._profile_shape(sh, record=True)
            self.synchronize()
            self.estimator.data_fit(self.tracker)
            self.load_estimator_state()
            if self.ft_enabled and self.trainer is not None and self.capture is not None:
                # One full backward cycle on this thread at the buffer's size:
                # loads every backward kernel before the feeder thread runs.
                cap = self.ftcfg.max_saved_finetuning_tokens
                ln = max(8, min(cap, self.store.min_len() or cap))
                k = max(1, cap // ln)
                self._record(("bwd_warmup", k * ln, [i * ln for i in range(k)], [ln] * k))
                self._flush_actions()
                self.bwd_warmup_ms = self._bwd_call(self.trainer.warmup, self.capture, k * ln,
                                                         [i * ln for i in range(k)], [ln] * k)
                dprint(f"[profile] backward warm-up cycle ({k * ln} tokens): "
                       f"{self.bwd_warmup_ms:.1f} ms")
        except Exception as e:  # profiling failure must not take serving down
            dprint(f"[profile] failed ({e!r}); finetuning disabled, serving continues")
            self.coord.disable(f"profiling failed: {e!r}")
        finally:
            self.profiling = False
            self._forced_ft = None

    def _profile_shape(self, sh, record: bool) -> None:
        rng = np.random.default_rng(self.tracker.size() + 17)
        V = self.arch.vocab
        mk = lambda n: rng.integers(0, V, size=int(n)).tolist()
        n0 = self.tracker.size()
        ids = []
        for i, n in enumerate(sh.inf_lens):
            rid = f"__prof__{self.step_no}_{i}"
            self.add_request(rid, mk(n), SamplingParams(max_tokens=1 + sh.n_decode + (1 if sh.mix_lens else 0)))
            ids.append(rid)
        ft = [Request(f"__proft__{self.step_no}_{j}", mk(n), SamplingParams(max_tokens=1),
                      FT_ADAPTER_NAME, time.perf_counter(), is_ft=True)
              for j, n in enumerate(sh.ft_lens)] if (self.ft_enabled and sh.ft_lens) else []
        if sh.kind in ("coserve", "ft_only"):
            self._forced_ft = ft
            ft = []
        steps = 0
        while self.has_unfinished() and steps < 64:
            if sh.kind == "decode" and ft and all(not r.in_prefill for r in self.scheduler.running):
                self._forced_ft, ft = ft, []
            if sh.kind == "mixed" and sh.mix_lens and all(not r.in_prefill for r in self.scheduler.running):
                for i, n in enumerate(sh.mix_lens):
                    self.add_request(f"__profm__{self.step_no}_{i}", mk(n), SamplingParams(max_tokens=1))
                sh = type(sh)(sh.kind, sh.inf_lens, sh.ft_lens, [], sh.n_decode)
            self.step()
            steps += 1
        if self._forced_ft:
            self._forced_ft_step()
        self.synchronize()
        if not record:
            self.tracker.truncate(n0)
        self.finished = [r for r in self.finished if not r.request_id.startswith("__prof")]

    def _bwd_call(self, fn, *args):
        """Run ``fn`` with the backward stream current (CUDA graphs are captured
        on it; capture is not allowed on the legacy default stream)."""
        if not self.cuda:
            return fn(*args)
        self.bwd_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.bwd_stream):
            return fn(*args)

    def _forced_ft_step(self) -> None:
        out = SchedulerOutput()
        self.scheduler.add_ft(out, self._forced_ft)
        self._forced_ft = None
        if not out.is_empty():
            self._run(out, 0, False, record_capture=False)

    # ------------------------------------------------------------------ TP replay
    @property
    def tp_size(self) -> int:
        return self.comm.size if self.comm is not None else 1

    def eos_ids(self) -> tuple[int, ...]:
        """End-of-sequence token ids: the tokenizer's ``eos_token_id`` plus the
        checkpoint's ``generation_config.json`` ids (Llama-3 instruct models
        end turns with a second id). A request stops on any of them unless
        its ``ignore_eos`` is set."""
        tok = self.tokenizer
        key = id(tok)
        if getattr(self, "_eos_key", None) != key:
            ids = set(self._gen_eos)
            e = getattr(tok, "eos_token_id", None) if tok is not None else None
            if isinstance(e, int):
                ids.add(e)
            elif isinstance(e, (list, tuple)):
                ids.update(int(x) for x in e)
            self._eos_cache, self._eos_key = tuple(sorted(ids)), key
        return self._eos_cache

    def _abort_vote(self):
        """The per-layer pre-emption vote of an interruptible forward (MAX over
        ranks): through the shared-memory channel (one store and a spin per
        layer), else an all-reduce on the process group."""
        if self.plan_chan is not None:
            return self.plan_chan.all_max
        return self.comm.all_reduce_max_int

    def _record(self, action) -> None:
        if self.tp_size > 1 and self.is_driver:
            with self._actions_lock:
                self._actions.append(action)

    def _flush_actions(self) -> None:
        if self.tp_size > 1 and self.is_driver:
            with self._actions_lock:
                acts, self._actions = self._actions, []
            if acts:
                if self.plan_chan is not None:
                    self.plan_chan.send(acts)
                else:
                    self.comm.broadcast_object(acts)

    def _plan_hook(self, has_ft: bool):
        if self.tp_size == 1:
            return None

        def hook(meta, pk):
            arr, spans = pk.freeze()
            self._record(("fwd", arr, spans, meta, has_ft))
            self._flush_actions()
        return hook

    def close(self) -> None:
        """Release GPU resources that hold communicator state. CUDA graphs with
        captured NCCL collectives must be destroyed before the process group,
        or its teardown waits forever. Safe to call on every rank."""
        if self.router is not None:
            self.router.stop()              # indexing thread and encoder processes
        if self.cuda:
            torch.cuda.synchronize(self.device)
        # A cycle cut short by shutdown is a suspended generator whose frame
        # holds the captured backward graphs (NCCL collectives inside): close
        # it first, or releasing the trainer's graph table frees nothing and
        # the process-group teardown waits on those graphs for good.
        if self._bwd_gen is not None:
            self._bwd_gen.close()
            self._bwd_gen = None
        self._bwd_result = None
        if self.trainer is not None:
            self.trainer.release_graphs()
        if self.runner.graphs is not None:
            self.runner.graphs.release()
        if self.cuda:
            torch.cuda.synchronize(self.device)
        if self.embed_peer is not None:
            self.embed_peer.close()
            self.embed_peer = None
        if self.peer_ws is not None:
            self.peer_ws.close()
            self.peer_ws = None
            if self.comm is not None:
                self.comm.peer_ws = None
        if self.bwd_ws is not None:
            if self.trainer is not None:
                self.trainer.bwd.tpws = None
            self.bwd_ws.close()
            self.bwd_ws = None
        if self.opt_ws is not None:
            if self.trainer is not None:
                self.trainer.optws = None
            self.opt_ws.close()
            self.opt_ws = None
        if self.plan_chan is not None:
            self.plan_chan.close()
            self.plan_chan = None

    def _mark_local(self, name: str) -> None:
        """Synchronise every stream of this GPU, then stamp wall time and a CUDA
        event (used to time a region on the device on every rank)."""
        if not hasattr(self, "marks"):
            self.marks = {}
            self._mark_events = {}
        if self.cuda:
            torch.cuda.synchronize(self.device)
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(self.fwd_stream)
            torch.cuda.synchronize(self.device)
            self._mark_events[name] = ev
        self.marks[name] = {"wall": time.perf_counter()}

    def mark(self, name: str) -> None:
        """All ranks stamp ``name`` at the same point of the step stream."""
        self._record(("mark", name))
        self._flush_actions()
        self._mark_local(name)

    def region_ms(self, a: str, b: str) -> tuple[float, float]:
        """(device ms, wall ms) between two marks on this rank."""
        wall = (self.marks[b]["wall"] - self.marks[a]["wall"]) * 1e3
        if self.cuda:
            return self._mark_events[a].elapsed_time(self._mark_events[b]), wall
        return wall, wall

    def gather_region(self, a: str, b: str) -> list[tuple[float, float]]:
        """Every rank's (device ms, wall ms) for a region (driver only)."""
        mine = self.region_ms(a, b)
        if self.tp_size == 1:
            return [mine]
        self._record(("gather", a, b))
        self._flush_actions()
        self.marks["__region__"] = mine
        res = self.comm.gather_objects(self.marks)
        # The followers' host seconds (waiting for step plans / replaying them).
        self.follower_host_s = [r.get("__host__", {}) for r in res[1:]]
        return [mine] + [r["__region__"] for r in res[1:]]

    def shutdown(self) -> None:
        """Stop the follower ranks (driver) after finishing queued work; save
        the estimator state (once, if configured) and close telemetry files."""
        if self.is_driver:
            try:
                self.save_estimator_state()
            except Exception as e:  # best effort at teardown
                dprint(f"[estimator] state save failed: {e!r}")
            self._drain_timing(block=True)
            path = self.ftcfg.batch_prediction_stats_path or (
                self.ftcfg.estimator_validation_path if self.ftcfg.validate_estimator else None)
            if path:
                self.tracker.write_prediction_stats_csv(path, self.estimator.split_mixed)
        self.stop_telemetry()
        if self.trainer is not None:
            self.trainer.wait_saves()
        if self.step_trace is not None:
            self.step_trace.close()
            self.step_trace = None
        if self.tp_size > 1 and self.is_driver:
            self._record(("stop",))
            self._flush_actions()

    def follow(self) -> None:
        """Follower-rank loop: replay rank 0's actions until it stops."""
        assert not self.is_driver
        t_h = time.perf_counter()
        while True:
            actions = self.plan_chan.recv() if self.plan_chan is not None else self.comm.broadcast_object(None)
            t_h = self._host("follower_wait_plan", t_h)
            for a in actions:
                kind = a[0]
                if kind == "stop":
                    self._drain_backward_follower()
                    return
                if kind == "mark":
                    self._mark_local(a[1])
                    continue
                if kind == "bwd_warmup":
                    self._bwd_call(self.trainer.warmup, self.capture, a[1], a[2], a[3])
                    continue
                if kind == "gather":
                    self.marks["__region__"] = self.region_ms(a[1], a[2])
                    self.marks["__host__"] = dict(self.host_s)
                    self.comm.gather_objects(self.marks)
                    continue
                if kind == "save":
                    if self.cuda:
                        torch.cuda.synchronize(self.device)
                    self.trainer.export_full()
                    continue
                if kind == "adapter_load":
                    _, slot, path, rank, alpha, seed, payload = a
                    if payload is not None:
                        tensors = payload
                    elif path is not None:
                        from ..adapters import peft_io
                        tensors, _ = peft_io.read_adapter(path)
                    else:
                        tensors = random_adapter(self.arch, rank, seed)
                    self._write_slot(slot, tensors, rank, alpha)
                    continue
                if kind == "adapter_clear":
                    self._clear_slot(a[1])
                    continue
                if kind == "job":
                    self._apply_job(*a[1:])
                    continue
                if kind == "decode_graphs":
                    self.warm_decode_graphs()
                    continue
                if kind == "fwd":
                    _, arr, spans, meta, has_ft = a
                    from .model_runner import _Packer
                    if self.cuda:
                        # The metadata copy must be ordered before the forward:
                        # both go on the forward stream (as on rank 0).
                        with torch.cuda.stream(self.fwd_stream):
                            if has_ft and self._publish_evt is not None:
                                self.fwd_stream.wait_event(self._publish_evt)
                            self.runner.forward_follower(meta, _Packer.thaw(arr, spans),
                                                         self.capture if has_ft else None,
                                                         vote=self._abort_vote())
                    else:
                        self.runner.forward_follower(meta, _Packer.thaw(arr, spans),
                                                     self.capture if has_ft else None,
                                                     vote=self._abort_vote())
                elif kind == "bwd_start":
                    m = a[1]
                    if self.cuda:
                        self.bwd_stream.wait_stream(self.fwd_stream)
                    self._bwd_gen = self.trainer.cycle(self.capture, m["n"], m["starts"], m["lens"],
                                                       m["epoch"], sync=False)
                elif kind == "bwd_next":
                    if self._bwd_gen is None:
                        continue
                    try:
                        if self.cuda:
                            with torch.cuda.stream(self.bwd_stream):
                                next(self._bwd_gen)
                        else:
                            next(self._bwd_gen)
                    except StopIteration as e:
                        self._bwd_gen = None
                        if self.cuda:
                            ev = torch.cuda.Event()
                            ev.record(self.bwd_stream)
                            self._publish_evt = ev
                        self.trainer.losses.append(0.0)
            t_h = self._host("follower_replay", t_h)

    def _drain_backward_follower(self) -> None:
        if self.cuda:
            torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------ helpers
    def idle_tick(self) -> None:
        """Housekeeping while no step runs: job stages (indexing, admission,
        the next job's init) and routing placement still advance."""
        self._poll_backward()
        if self.ft_enabled:
            self.jobs.tick(self)
        if self.router is not None:
            self.router.tick()

    def has_ft_work(self) -> bool:
        c = self.coord
        if not self.ft_enabled or c.disabled:
            return False
        if self.bwd_active or self._bwd_done_evt is not None or c.pending_backward:
            return True
        return c.ft_started and (c.fill_count > 0 or (self.store is not None and not self.store.finished()))

    def run_until_idle(self, max_steps: int = 100000, finetune: bool = True) -> None:
        for _ in range(max_steps):
            if not self.has_unfinished() and not (finetune and self.has_ft_work()):
                break
            self.step()
        self._drain_backward()


