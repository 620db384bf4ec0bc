"""Sectioned YAML launch config.

Accepts the reference launcher's YAML layout unchanged
(``deltaserve-plugin/deltaserve/config_loader.py:60-131``):

* six finetune sections (``finetune_param``, ``finetune_features``,
  ``throttles``, ``slo``, ``debug``, ``telemetry``) fold into one flat
  :class:`FinetuneConfig`; a key in the "wrong" one of the six still loads
  with a warning; the legacy single ``finetune`` section loads with a note;
* ``adapter_routing`` becomes an :class:`AdapterRoutingConfig`;
* ``ft_job`` sets flat finetune fields (``adapter_path`` → ``finetuning_lora_path``
  ...) plus job metadata;
* ``server`` and ``adapters`` are returned verbatim as extras;
* every other section (``model``, ``engine``, ``lora``, ``parallel`` ...) is
  merged into the :class:`EngineConfig` kwargs; a key in two sections is an
  error, an unknown key is a ``TypeError``.

Relative paths (keys containing ``path`` or ending in ``_dir``) in the
finetune sections, ``adapters``, ``adapter_routing`` and ``ft_job`` resolve
against the YAML file's directory.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import yaml

from . import dprint
from .config import AdapterRoutingConfig, EngineConfig, FinetuneConfig

FINETUNE_SECTIONS: dict[str, tuple[str, ...]] = {
    "finetune_param": (
        "enable_finetuning", "start_on_launch", "finetuning_lora_path",
        "data_path", "max_prepare", "num_epochs", "learning_rate",
        "weight_decay", "gamma", "max_saved_finetuning_tokens",
        "adapter_save_path", "adapter_save_every_backwards",
        "adapter_save_every_epoch", "adapter_save_keep_last",
        "loss_mask_prefix", "ft_target_modules",
    ),
    "finetune_features": (
        "backward_mps_percentage", "backward_fp32", "backward_cuda_graph",
        "backward_cuda_graph_attn_bn_max", "backward_cuda_graph_attn_l_max",
        "backward_run_ahead_boundaries", "save_activations", "save_attn_qkv",
        "save_attn_ctx", "save_resid_mid", "graph_ft_batches",
        "graph_ft_max_tokens", "graph_ft_only_batches", "forward_interruptible",
        "ft_only_admission_grace_ms", "pause_on_arrival", "pause_prefill_always",
        "pause_until_prefill_done",
    ),
    "throttles": (
        "coserving_admission_phase", "ft_tokens_admission_constrain_factor",
        "match_prefill_workload_factor", "fwd_token_throttle_enable",
        "fwd_token_throttle", "rps_throttle_enable", "rps_throttle_close_rps",
        "rps_throttle_open_rps", "rps_throttle_window_s",
        "rps_throttle_close_time",
    ),
    "slo": (
        "ttft_slo", "avg_tbt_slo", "avg_tbt_window_s", "max_tbt_slo",
        "decode_only_ft_safety_margin", "admission_margin", "admission_margin_k",
        "profile_on_launch", "profile_num_repeats", "validate_estimator",
        "estimator_validation_path", "estimator_state_save_path",
        "estimator_state_load_path",
    ),
    "debug": (
        "print_weight_hash", "print_activation_hash", "print_step_mode",
        "print_scheduler_add", "print_engine_batch_exec",
        "print_engine_batch_done", "print_engine_req_recv",
    ),
    "telemetry": (
        "metrics_dir", "metrics_interval_s", "steps_log_max_mb",
        "step_trace_path", "bwd_log_path", "batch_prediction_stats_path",
    ),
}
LEGACY_SECTIONS: tuple[str, ...] = ("finetune",)
ALL_FINETUNE_SECTIONS = (*FINETUNE_SECTIONS, *LEGACY_SECTIONS)
SECTION_OF = {k: s for s, keys in FINETUNE_SECTIONS.items() for k in keys}
RETIRED_KEYS = {"backward_sleep_seconds": "only the removed OPT loss-only service slept"}
PASSTHROUGH_SECTIONS = ("server", "adapters")
ADAPTER_ROUTING_SECTION = "adapter_routing"
FT_JOB_SECTION = "ft_job"
SPECIAL_SECTIONS = (*ALL_FINETUNE_SECTIONS, *PASSTHROUGH_SECTIONS,
                    ADAPTER_ROUTING_SECTION, FT_JOB_SECTION)

# ft_job keys that set a flat FinetuneConfig field, and pure job metadata.
JOB_FLAT_KEYS = {
    "adapter_path": "finetuning_lora_path",
    "data_path": "data_path",
    "num_epochs": "num_epochs",
    "learning_rate": "learning_rate",
    "weight_decay": "weight_decay",
    "gamma": "gamma",
}
JOB_META_KEYS = ("name", "stages", "auto_routing", "adapter_init", "save_path")


def _is_path_key(key: str) -> bool:
    k = key.lower()
    return "path" in k or k.endswith("_dir")


def _absolutize(mapping: dict, base: Path, is_path) -> None:
    """Rewrite, in place, the relative string values of ``mapping`` whose key
    ``is_path`` accepts as absolute paths under ``base``."""
    for key in [k for k, v in mapping.items() if isinstance(v, str) and is_path(k)]:
        p = Path(mapping[key])
        if not p.is_absolute():
            mapping[key] = str((base / p).resolve())


def load_yaml_config(path: str | Path, verbose: bool = False) -> dict[str, Any]:
    """Read a sectioned YAML file into ``{section: {key: value}}`` with
    relative paths made absolute against the file's directory."""
    path = Path(path)
    if not path.is_file():
        raise FileNotFoundError(f"DeltaServe config not found: {path}")
    with path.open() as f:
        raw = yaml.safe_load(f) or {}
    if not isinstance(raw, dict):
        raise ValueError(f"{path}: top level must be a mapping of sections, "
                         f"got {type(raw).__name__}")
    for section, body in raw.items():
        if body is not None and not isinstance(body, dict):
            raise ValueError(f"{path}: section '{section}' must be a mapping "
                             f"(got {type(body).__name__})")
    base = path.resolve().parent
    mappings = [raw.get(s) or {} for s in (*ALL_FINETUNE_SECTIONS, "adapters", ADAPTER_ROUTING_SECTION,
                                           FT_JOB_SECTION)]
    listed = (raw.get(ADAPTER_ROUTING_SECTION) or {}).get("adapters") or []
    for m in mappings:
        _absolutize(m, base, _is_path_key)
    for m in listed:                      # routing's adapter list: {name, path, data_path, ...}
        if isinstance(m, dict):
            _absolutize(m, base, lambda k: "path" in k.lower())
    if verbose:
        dprint(f"loaded config ({path}):")
        for section, body in raw.items():
            kvs = "  ".join(f"{k}={v}" for k, v in (body or {}).items()) or "(empty)"
            dprint(f"  [{section}] {kvs}")
    return raw


def _finetune_settings(config: dict[str, Any]):
    """Every finetune setting of a loaded YAML as ``(where, field, value)``:
    the keys of the finetune sections (legacy one included), then the
    ``ft_job`` keys that stand for a flat field."""
    for section in ALL_FINETUNE_SECTIONS:
        for key, value in (config.get(section) or {}).items():
            yield section, key, value
    for key, value in (config.get(FT_JOB_SECTION) or {}).items():
        if key in JOB_FLAT_KEYS:
            yield f"{FT_JOB_SECTION}.{key}", JOB_FLAT_KEYS[key], value


def finetune_kwargs(config: dict[str, Any]) -> dict[str, Any]:
    """Flat :class:`FinetuneConfig` kwargs from the finetune sections and
    ``ft_job``, checked against the dataclass: a field set from two places is
    an error, a retired key is dropped with a warning, a key outside its
    usual section is accepted with a warning, and ``ft_job``'s metadata keys
    land in ``ft_job``."""
    import dataclasses
    known = {f.name for f in dataclasses.fields(FinetuneConfig)}
    for section in LEGACY_SECTIONS:
        if config.get(section):
            dprint(f"[config] section '{section}' uses the single-section layout; its keys are read as they are")
    values: dict[str, Any] = {}
    source: dict[str, str] = {}
    for where, field_name, value in _finetune_settings(config):
        if field_name in RETIRED_KEYS:
            dprint(f"[config] WARNING: {where}.{field_name} has no effect any more "
                   f"({RETIRED_KEYS[field_name]}) and is dropped")
            continue
        home = SECTION_OF.get(field_name)
        if where in FINETUNE_SECTIONS and home is not None and home != where:
            dprint(f"[config] WARNING: {where}.{field_name} is normally under '{home}'; accepted")
        if field_name in values:
            raise ValueError(f"finetune setting '{field_name}' is given twice ({source[field_name]} and {where})")
        if field_name not in known:
            raise ValueError(f"{where}.{field_name} is not a finetune setting")
        values[field_name], source[field_name] = value, where
    job = config.get(FT_JOB_SECTION)
    if job:
        extra = sorted(k for k in job if k not in JOB_FLAT_KEYS and k not in JOB_META_KEYS)
        if extra:
            raise ValueError(f"{FT_JOB_SECTION}: unsupported key(s) {extra}; allowed: "
                             f"{sorted((*JOB_META_KEYS, *JOB_FLAT_KEYS))}")
        values["ft_job"] = {k: v for k, v in job.items() if k in JOB_META_KEYS}
    return values


def finetune_value(config: dict[str, Any], key: str, default: Any = None) -> Any:
    """``key`` from whichever finetune section sets it (first one wins)."""
    found = (config[s][key] for s in ALL_FINETUNE_SECTIONS if key in (config.get(s) or {}))
    return next(found, default)


def adapter_routing_config(config: dict[str, Any]) -> AdapterRoutingConfig:
    return AdapterRoutingConfig(**dict(config.get(ADAPTER_ROUTING_SECTION) or {}))


def engine_kwargs(config: dict[str, Any]) -> dict[str, Any]:
    """Every non-special section merged into one flat dict; duplicates are errors."""
    out: dict[str, Any] = {}
    for section, body in config.items():
        if section in SPECIAL_SECTIONS:
            continue
        for key, value in (body or {}).items():
            if key in out:
                raise ValueError(f"duplicate engine key '{key}' (appears in section "
                                 f"'{section}' and another section)")
            out[key] = value
    return out


def split_config(config: dict[str, Any]
                 ) -> tuple[EngineConfig, FinetuneConfig, AdapterRoutingConfig, dict]:
    """Split a loaded YAML into (engine, finetune, routing, extras)."""
    from .engine.ft_job import FinetuneJobSpec

    extras = {name: dict(config.get(name) or {}) for name in PASSTHROUGH_SECTIONS}
    # vLLM keys the reference YAMLs carry that have no meaning here.
    ekw = engine_kwargs(config)
    for ignored in ("disable_log_stats",):
        ekw.pop(ignored, None)
    engine = EngineConfig(**ekw)
    ft = FinetuneConfig(**finetune_kwargs(config))
    routing = adapter_routing_config(config)
    if ft.enable_finetuning:
        FinetuneJobSpec.from_finetune_config(ft).validate(routing.enable_adapter_routing)
    return engine, ft, routing, extras


def load_launch_config(path: str | Path, verbose: bool = False):
    return split_config(load_yaml_config(path, verbose=verbose))


def additional_config(config: dict[str, Any], **overrides: Any) -> dict:
    """The finetune sections as one JSON-able dict (the reference passed this to
    ``vllm serve --additional-config``; here it round-trips a config between
    processes)."""
    def given(d: dict) -> dict:
        return dict(filter(lambda kv: kv[1] is not None, d.items()))

    settings = finetune_kwargs(config)
    settings.update(given(overrides))
    doc = {"deltaserve": given(settings)}
    routing = given(config.get(ADAPTER_ROUTING_SECTION) or {})
    if routing:
        doc["deltaserve_adapter_routing"] = routing
    return doc


def finetune_cli_args(config: dict[str, Any], **overrides: Any) -> list[str]:
    return ["--additional-config", json.dumps(additional_config(config, **overrides))]
