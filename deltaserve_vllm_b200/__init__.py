"""DeltaServe-B200: a Blackwell-native engine that serves LLM inference and
trains LoRA adapters on the same GPUs.

Package layout:

* ``config`` / ``config_loader`` — dataclass configs and the sectioned YAML
  launch file (same sections and keys as the reference plugin's loader,
  ``deltaserve-plugin/deltaserve/config_loader.py:60-107``).
* ``models`` — decoder architectures (Llama-3, Qwen3), weight layout, and the
  hand-written LoRA backward.
* ``ops`` — the hot ops; CUDA tensors go to the sm_100a extension, CPU tensors
  to the fp32 PyTorch oracle used by the tests.
* ``parallel`` — tensor parallelism: process groups, shard geometry, NCCL
  baseline collectives and the fused compute+collective kernels.
* ``engine`` — paged KV cache, continuous-batching scheduler, finetuning
  admission (store, coordinator, estimator), trainer and the step loop.
* ``server`` — the OpenAI-compatible HTTP API plus the finetuning routes.
* ``adapters`` — PEFT checkpoint I/O and adapter routing.
* ``utils`` — metrics, step trace, live feed.
"""

import os
import sys

__version__ = "0.1.0"

_GREEN = "\033[32m"
_PURPLE = "\033[35m"
_RESET = "\033[0m"


def dprint(*args, **kwargs) -> None:
    """Print with a ``[deltaserve]`` prefix. Rank-worker processes other than
    rank 0 use a different colour so interleaved logs stay readable
    (the reference colours its backward child the same way,
    ``deltaserve-plugin/deltaserve/__init__.py:28-44``)."""
    if os.environ.get("DSERVE_QUIET") == "1":
        return
    rank = os.environ.get("RANK", "0")
    colour = _GREEN if rank in ("0", "") else _PURPLE
    tty = sys.stdout.isatty()
    prefix = f"{colour}[deltaserve]{_RESET}" if tty else "[deltaserve]"
    if rank not in ("0", ""):
        prefix += f"[r{rank}]"
    kwargs.setdefault("flush", True)
    print(prefix, *args, **kwargs)
