"""PEFT LoRA checkpoints: read, write (atomic), merge across TP ranks, prune.

A checkpoint directory holds ``adapter_model.safetensors`` (fp32 factors, PEFT
key names, B unscaled — PEFT applies ``lora_alpha / r`` itself),
``adapter_config.json`` and ``trainer_state.json``. Every file is written to a
temporary name and renamed; ``trainer_state.json`` goes last and is the
completion marker a waiting ``POST /save_adapter`` polls for (same handshake
as the reference, ``deltaserve-plugin/deltaserve/adapter_io.py:95-142``).
"""

from __future__ import annotations

import json
import os
import re
import shutil
import time

import torch
from safetensors.torch import load_file, save_file

from ..models.lora import COLUMN_PARALLEL

STATE_FILE = "trainer_state.json"
ERROR_FILE = "save_error.json"
WEIGHTS_FILE = "adapter_model.safetensors"
CONFIG_FILE = "adapter_config.json"
_KEY = re.compile(r"layers\.(\d+)\.(?:self_attn|mlp)\.(\w+)_proj\.lora_([AB])\.weight$")


def parse_key(key: str) -> tuple[int, str, str] | None:
    m = _KEY.search(key)
    return (int(m.group(1)), m.group(2), m.group(3)) if m else None


def read_adapter(path: str) -> tuple[dict[str, torch.Tensor], dict]:
    """(tensors, adapter_config) of a PEFT LoRA directory."""
    cfg_path = os.path.join(path, CONFIG_FILE)
    with open(cfg_path) as f:
        cfg = json.load(f)
    wpath = os.path.join(path, WEIGHTS_FILE)
    if os.path.isfile(wpath):
        tensors = load_file(wpath)
    elif os.path.isfile(os.path.join(path, "adapter_model.bin")):
        tensors = torch.load(os.path.join(path, "adapter_model.bin"), map_location="cpu")
    else:
        tensors = {}
    # PEFT names the module with the adapter name inside some versions
    # ("lora_A.default.weight"); normalise.
    tensors = {k.replace(".default.weight", ".weight"): v for k, v in tensors.items()}
    return tensors, cfg


def adapter_rank_alpha(cfg: dict) -> tuple[int, float]:
    r = int(cfg.get("r", 8))
    return r, float(cfg.get("lora_alpha", r))


def merge_tp_shards(shards: list[dict[str, torch.Tensor]]) -> dict[str, torch.Tensor]:
    """Inverse of the TP shard slice: column-parallel B (q/k/v/gate/up) concat
    on dim 0, row-parallel A (o/down) concat on dim 1, replicated factors from
    rank 0."""
    if len(shards) == 1:
        return dict(shards[0])
    out = {}
    for key, t0 in shards[0].items():
        pk = parse_key(key)
        if pk is None:
            out[key] = t0
            continue
        _, proj, ab = pk
        if proj in COLUMN_PARALLEL and ab == "B":
            out[key] = torch.cat([s[key] for s in shards], 0)
        elif proj in ("o", "down") and ab == "A":
            out[key] = torch.cat([s[key] for s in shards], 1)
        else:
            out[key] = t0
    return out


def write_json_atomic(path: str, obj, indent: int | None = 2) -> None:
    """``obj`` as JSON at ``path`` (folders made), through a sibling file and
    one rename, so a reader sees the old document or the new one."""
    folder = os.path.dirname(os.path.abspath(path))
    os.makedirs(folder, exist_ok=True)
    part = os.path.join(folder, f".{os.path.basename(path)}.{os.getpid()}.part")
    with open(part, "w") as f:
        json.dump(obj, f, indent=indent)
    os.replace(part, path)



def write_peft_adapter(path: str, tensors: dict[str, torch.Tensor], adapter_config: dict,
                       state: dict) -> None:
    os.makedirs(path, exist_ok=True)
    tmp = os.path.join(path, WEIGHTS_FILE + ".tmp")
    save_file({k: v.detach().float().contiguous().cpu() for k, v in tensors.items()}, tmp,
              metadata={"format": "pt"})
    os.replace(tmp, os.path.join(path, WEIGHTS_FILE))
    write_json_atomic(os.path.join(path, CONFIG_FILE), adapter_config)
    err = os.path.join(path, ERROR_FILE)
    if os.path.exists(err):
        os.remove(err)
    write_json_atomic(os.path.join(path, STATE_FILE), state)


def write_save_error(path: str, save_id: str, error: str) -> None:
    os.makedirs(path, exist_ok=True)
    write_json_atomic(os.path.join(path, ERROR_FILE), {"save_id": save_id, "error": error})


def read_save_result(path: str, save_id: str) -> dict | None:
    """The finished save's state (or {'error': ...}) once ``save_id`` landed, else None."""
    for name, is_err in ((STATE_FILE, False), (ERROR_FILE, True)):
        p = os.path.join(path, name)
        if os.path.isfile(p):
            try:
                with open(p) as f:
                    d = json.load(f)
            except (OSError, json.JSONDecodeError):
                continue
            if d.get("save_id") == save_id:
                return d
    return None


def wait_save_result(path: str, save_id: str, timeout_s: float = 60.0) -> dict | None:
    t0 = time.time()
    while time.time() - t0 < timeout_s:
        r = read_save_result(path, save_id)
        if r is not None:
            return r
        time.sleep(0.02)
    return None


def prune_checkpoints(root: str, keep_last: int, prefix: str = "backward-") -> list[str]:
    """Delete all but the newest ``keep_last`` ``<prefix>NNNNNN`` directories."""
    if keep_last <= 0 or not os.path.isdir(root):
        return []
    dirs = sorted(d for d in os.listdir(root) if d.startswith(prefix)
                  and os.path.isdir(os.path.join(root, d)))
    removed = []
    for d in dirs[:-keep_last]:
        shutil.rmtree(os.path.join(root, d), ignore_errors=True)
        removed.append(d)
    return removed


def default_adapter_config(rank: int, alpha: float, targets, base_model: str = "") -> dict:
    names = {"q": "q_proj", "k": "k_proj", "v": "v_proj", "o": "o_proj", "gate": "gate_proj",
             "up": "up_proj", "down": "down_proj"}
    return {"peft_type": "LORA", "task_type": "CAUSAL_LM", "r": int(rank),
            "lora_alpha": float(alpha), "lora_dropout": 0.0, "bias": "none",
            "target_modules": [names[t] for t in targets], "base_model_name_or_path": base_model,
            "fan_in_fan_out": False, "inference_mode": True}
