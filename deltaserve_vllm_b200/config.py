"""Configuration dataclasses.

Three configs describe a launch:

* :class:`FinetuneConfig` — every co-serving knob of the reference plugin's
  ``FinetuneConfig`` (``deltaserve-plugin/deltaserve/config.py:16-699``): same
  field names, same defaults, so a reference YAML loads unchanged.
* :class:`AdapterRoutingConfig` — adapter routing
  (``deltaserve-plugin/deltaserve/config.py:702-948``), same fields and checks.
* :class:`EngineConfig` — the engine itself (model, parallelism, KV cache,
  LoRA slots). The reference hands these keys to vLLM's ``EngineArgs``; this
  engine owns them, and accepts the vLLM key names the reference YAMLs use.

Unknown keys raise ``TypeError`` (dataclass constructor), which mirrors the
reference's ``extra=forbid``.
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
from dataclasses import dataclass, field
from typing import Any


def _check_choice(name: str, value: Any, choices: tuple) -> None:
    if value not in choices:
        raise ValueError(f"{name} must be one of {choices}, got {value!r}")


@dataclass
class FinetuneConfig:
    """Co-serving knobs. Grouped as in the YAML sections of the launcher."""

    # ---- finetune_param: the training job --------------------------------
    enable_finetuning: bool = False
    start_on_launch: bool = True
    finetuning_lora_path: str | None = None
    data_path: str | None = None
    max_prepare: int | None = None
    num_epochs: int = 1
    learning_rate: float = 1e-4
    weight_decay: float = 0.0
    gamma: float = 1.0
    # Tokens per backward cycle: sizes the activation-capture buffers.
    max_saved_finetuning_tokens: int = 256
    adapter_save_path: str | None = None
    adapter_save_every_backwards: int = 0
    adapter_save_every_epoch: bool = False
    adapter_save_keep_last: int = 0
    ft_job: dict | None = None
    # Labels: the first N positions of every sample carry no loss (prompt
    # mask). 0 = the reference's full shift-by-one cross-entropy.
    loss_mask_prefix: int = 0
    # LoRA targets trained by the finetuning adapter. The reference trains
    # q/k/v/o; this engine trains all seven projections by default.
    ft_target_modules: tuple = ("q", "k", "v", "o", "gate", "up", "down")

    # ---- finetune_features: how co-serving runs ---------------------------
    # Kept for YAML compatibility. This engine trains inside the serving
    # process on a low-priority stream, so there is no MPS child to size.
    backward_mps_percentage: int = 0
    backward_fp32: bool = False
    backward_cuda_graph: bool = False
    backward_cuda_graph_attn_bn_max: int = 8
    backward_cuda_graph_attn_l_max: int = 64
    backward_run_ahead_boundaries: int = 2
    save_activations: bool = True
    save_attn_qkv: bool = False
    save_attn_ctx: bool = False
    save_resid_mid: bool = False
    graph_ft_batches: bool = False
    graph_ft_max_tokens: int = 512
    graph_ft_only_batches: bool = False
    forward_interruptible: bool = False
    ft_only_admission_grace_ms: float = 2.0
    pause_on_arrival: bool = False
    pause_prefill_always: bool = False
    pause_until_prefill_done: bool = True

    # ---- throttles ---------------------------------------------------------
    coserving_admission_phase: str = "prefill"
    ft_tokens_admission_constrain_factor: float = -1.0
    match_prefill_workload_factor: float = 0.0
    fwd_token_throttle_enable: bool = False
    fwd_token_throttle: int = 1024
    rps_throttle_enable: bool = False
    rps_throttle_close_rps: float = 50.0
    rps_throttle_open_rps: float = 30.0
    rps_throttle_window_s: float = 1.0
    rps_throttle_close_time: float = 0.0

    # ---- slo + estimator -----------------------------------------------------
    ttft_slo: float = 1.0
    avg_tbt_slo: float = 0.1
    avg_tbt_window_s: float = 0.0
    max_tbt_slo: float = 0.2
    decode_only_ft_safety_margin: float = 0.7
    admission_margin: str = "relative"
    admission_margin_k: float = 1.5
    profile_on_launch: bool = True
    profile_num_repeats: int = 2
    validate_estimator: bool = False
    estimator_validation_path: str | None = None
    estimator_state_save_path: str | None = None
    estimator_state_load_path: str | None = None

    # ---- debug ---------------------------------------------------------------
    print_weight_hash: bool = False
    print_activation_hash: bool = False
    print_step_mode: bool = False
    print_scheduler_add: bool = False
    print_engine_batch_exec: bool = False
    print_engine_batch_done: bool = False
    print_engine_req_recv: bool = False

    # ---- telemetry -------------------------------------------------------------
    metrics_dir: str | None = None
    metrics_interval_s: float = 10.0
    steps_log_max_mb: float = 256.0
    step_trace_path: str | None = None
    bwd_log_path: str | None = None
    batch_prediction_stats_path: str | None = None

    def __post_init__(self) -> None:
        _check_choice("throttles.coserving_admission_phase",
                      self.coserving_admission_phase, ("prefill", "both"))
        _check_choice("slo.admission_margin", self.admission_margin,
                      ("legacy", "relative", "absolute"))
        if self.max_saved_finetuning_tokens < 1:
            raise ValueError("max_saved_finetuning_tokens must be >= 1")
        if self.num_epochs < 1:
            raise ValueError("num_epochs must be >= 1")
        if (self.coserving_admission_phase == "both"
                and self.ft_tokens_admission_constrain_factor != -1):
            # Same rule as the reference (config.py:287-303): the proportional
            # cap is relative to prefill tokens, so decode-only admission
            # cannot use it.
            self.coserving_admission_phase = "prefill"
        self.ft_target_modules = tuple(self.ft_target_modules)
        bad = set(self.ft_target_modules) - set(LORA_PROJS)
        if bad:
            raise ValueError(f"ft_target_modules: unknown projection(s) {sorted(bad)}")

    # Only the fields that change captured graphs or buffer shapes; used as a
    # cache key (reference: ``FinetuneConfig.compute_hash``, config.py:495-511).
    _GRAPH_FIELDS = ("enable_finetuning", "max_saved_finetuning_tokens",
                     "save_activations", "save_attn_qkv", "save_attn_ctx",
                     "save_resid_mid", "graph_ft_batches", "graph_ft_max_tokens",
                     "graph_ft_only_batches", "forward_interruptible",
                     "backward_cuda_graph", "ft_target_modules")

    def compute_hash(self) -> str:
        payload = {k: getattr(self, k) for k in self._GRAPH_FIELDS}
        return hashlib.sha256(json.dumps(payload, sort_keys=True,
                                         default=str).encode()).hexdigest()[:16]


# Projection names, in the order the engine stores them.
LORA_PROJS = ("q", "k", "v", "o", "gate", "up", "down")
# PEFT module names of each projection.
PEFT_MODULE = {"q": "self_attn.q_proj", "k": "self_attn.k_proj",
               "v": "self_attn.v_proj", "o": "self_attn.o_proj",
               "gate": "mlp.gate_proj", "up": "mlp.up_proj",
               "down": "mlp.down_proj"}


# Lower bounds of the numeric routing knobs: counts and sizes need at least
# one; times, shares and slot counts may be zero.
_ROUTING_LOWER_BOUNDS = {
    **dict.fromkeys(("encoder_max_tokens", "max_active_adapters", "route_encode_max_tokens",
                     "indexing_max_samples", "indexing_chunk_samples", "indexing_cpu_max_threads",
                     "indexing_gpu_chunk_samples", "route_min_pool"), 1),
    **dict.fromkeys(("indexing_gpu_after_quiet_s", "pool_protected_slots", "indexing_cpu_busy_threads",
                     "pool_hit_half_life_s", "route_close_band", "route_confidence_slack", "retire_grace_s",
                     "route_reference_samples"), 0),
}


@dataclass
class AdapterRoutingConfig:
    """Adapter routing knobs (``adapter_routing`` YAML section)."""

    enable_adapter_routing: bool = False
    route_model_name: str = "auto"
    router_device: str = "auto"
    router_gpu: int | None = None
    route_encode_max_tokens: int = 1024
    route_encode_async: bool = True
    adapter_copy_ms: float = 4.5
    adapter_read_ms: float = 13.5
    encoder: str = "intfloat/e5-large-v2"
    encoder_query_prefix: str = "query: "
    encoder_max_tokens: int = 512
    route_keep_percent: float = 90.0
    route_confidence_slack: float = 0.0
    route_close_band: float = 0.05
    route_min_pool: int = 4
    route_reference_samples: int = 64
    route_decision_log: bool = False
    fallback_score_threshold: float = 0.0
    max_active_adapters: int = 32
    when_full: str = "retire_least_used"
    retire_grace_s: float = 600.0
    admission_min_self_recall: float = 0.0
    admission_max_stolen: float = 1.0
    pool_protected_slots: int = 1
    pool_hit_half_life_s: float = 300.0
    adapters: list | None = None
    index_path: str | None = None
    indexing_max_samples: int = 2500
    indexing_input_until: str | None = None
    indexing_chunk_samples: int = 16
    indexing_cpu_max_threads: int = 8
    indexing_cpu_busy_threads: int = 2
    indexing_cpus: str | None = None
    indexing_process: bool = True
    indexing_on_gpu: bool = True
    indexing_gpu_chunk_samples: int = 8
    indexing_gpu_after_quiet_s: float = 3.0

    def __post_init__(self) -> None:
        if not self.route_model_name:
            raise ValueError("adapter_routing.route_model_name must not be empty")
        if not self.encoder:
            raise ValueError("adapter_routing.encoder must not be empty")
        _check_choice("adapter_routing.when_full", self.when_full,
                      ("retire_least_used", "admit_retired", "reject"))
        below = [(k, lo) for k, lo in _ROUTING_LOWER_BOUNDS.items() if float(getattr(self, k)) < lo]
        if below:
            raise ValueError(f"adapter_routing.{below[0][0]} must be >= {below[0][1]}")
        if not 0.0 <= float(self.route_keep_percent) <= 100.0:
            raise ValueError("adapter_routing.route_keep_percent is in [0, 100]")
        entries = list(self.adapters or [])
        allowed = {"path", "name", "data_path", "centroid_path", "prewarm"}
        bad = [a for a in entries if not isinstance(a, dict) or not a.get("path")]
        if bad:
            raise ValueError("adapter_routing.adapters: each entry needs a 'path'")
        extra = sorted(set().union(*(set(a) - allowed for a in entries))) if entries else []
        if extra:
            raise ValueError(f"adapter_routing.adapters: unknown key(s) {extra}")
        named = [a["name"] for a in entries if a.get("name")]
        dup = sorted({n for n in named if named.count(n) > 1})
        if dup:
            raise ValueError(f"adapter_routing.adapters: duplicate name '{dup[0]}'")
        if self.router_gpu is not None and int(self.router_gpu) < 0:
            raise ValueError("adapter_routing.router_gpu must be a GPU index >= 0")
        if not -1.0 <= float(self.fallback_score_threshold) <= 1.0:
            raise ValueError("adapter_routing.fallback_score_threshold is a cosine in [-1, 1]")


@dataclass
class EngineConfig:
    """Engine geometry. Field names follow vLLM's ``EngineArgs`` where the
    reference YAMLs use them (``model``, ``tensor_parallel_size``,
    ``max_model_len``, ``gpu_memory_utilization``, ``enable_lora``,
    ``max_loras``, ``max_lora_rank`` ...)."""

    # A preset name (``llama3-8b``, ``qwen3-0.6b`` ...), an HF model id whose
    # architecture is known, or a directory with an HF ``config.json``.
    model: str = "qwen3-tiny"
    # Base weights: "auto" loads the model directory's *.safetensors when it
    # has any and random-initialises otherwise; "safetensors" requires them;
    # "dummy" always random-initialises (vLLM's load_format names).
    load_format: str = "auto"
    tokenizer: str | None = None
    tokenizer_mode: str = "auto"
    trust_remote_code: bool = False
    dtype: str = "auto"
    seed: int = 0
    max_model_len: int = 4096
    tensor_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    # KV cache: page size in tokens and the share of free HBM it may take.
    block_size: int = 64
    gpu_memory_utilization: float = 0.85
    num_gpu_blocks_override: int | None = None
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    enable_chunked_prefill: bool = True
    # Automatic prefix caching of full KV pages (chained token hashes keyed by
    # the LoRA slot version; finetuning rows never share pages).
    enable_prefix_caching: bool = False
    enforce_eager: bool = False
    enable_lora: bool = True
    max_loras: int = 4
    max_lora_rank: int = 16
    served_model_name: str | None = None
    disable_log_stats: bool = True
    async_scheduling: bool = False
    # Accepted for YAML compatibility; CUDA-graph sizes are chosen by the engine.
    compilation_config: dict | None = None
    max_cudagraph_capture_size: int | None = None
    # Collective implementation for tensor parallelism: "fused" = the sm_100a
    # GEMM+collective kernels over NVSwitch peer memory, "nccl" = baseline.
    tp_comm: str = "fused"
    # Device override ("cuda" / "cpu"); None = cuda when available.
    device: str | None = None

    def __post_init__(self) -> None:
        if self.tensor_parallel_size not in (1, 2, 4, 8):
            raise ValueError("tensor_parallel_size must be 1, 2, 4 or 8")
        if self.pipeline_parallel_size != 1:
            raise ValueError("pipeline parallelism is not supported (the reference has none)")
        if self.block_size % 16:
            raise ValueError("block_size must be a multiple of 16")
        _check_choice("tp_comm", self.tp_comm, ("fused", "nccl"))
        if self.max_lora_rank % 8:
            raise ValueError("max_lora_rank must be a multiple of 8")


def engine_config_fields() -> set[str]:
    return {f.name for f in dataclasses.fields(EngineConfig)}
