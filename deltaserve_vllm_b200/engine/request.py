"""Request state for the continuous-batching scheduler."""

from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field


class Status(enum.Enum):
    WAITING = 0
    RUNNING = 1
    FINISHED = 2
    ABORTED = 3


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0
    seed: int | None = None
    ignore_eos: bool = True
    stop_token_ids: tuple[int, ...] = ()
    top_k: int = 0                   # 0 = off
    top_p: float = 1.0               # 1 = off
    logprobs: bool = False           # record the chosen token's log-probability
    top_logprobs: int = 0            # and this many most likely alternatives per position
    stop: tuple[str, ...] = ()       # stop strings (checked on the decoded output)
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0  # 1 = off
    min_tokens: int = 0              # no EOS / stop token / stop string before this many
    logit_bias: tuple[tuple[int, float], ...] = ()

    @property
    def has_penalties(self) -> bool:
        return bool(self.presence_penalty or self.frequency_penalty or self.repetition_penalty != 1.0
                    or self.min_tokens > 0 or self.logit_bias)

    @property
    def needs_full_sampler(self) -> bool:
        return self.top_k > 0 or self.top_p < 1.0 or self.logprobs or self.has_penalties


_counter = itertools.count()


@dataclass(eq=False)
class Request:
    """One inference or finetuning request. Compared by identity: the
    scheduler's queues test membership on every step, and a field-by-field
    comparison (prompt token lists included) made that O(fields) per test."""
    request_id: str
    prompt_ids: list[int]
    params: SamplingParams = field(default_factory=SamplingParams)
    adapter: str | None = None       # LoRA adapter name (None = base model)
    arrival_time: float = field(default_factory=time.perf_counter)
    # Finetuning sample: prefill-only, produces no output token, never shares
    # KV pages with anything (so a cached prefix can never skip its activations).
    is_ft: bool = False
    ft_sample: object = None
    # -- runtime state --------------------------------------------------
    status: Status = Status.WAITING
    output_ids: list[int] = field(default_factory=list)
    output_logprobs: list[float] = field(default_factory=list)
    output_top_logprobs: list[list[tuple[int, float]]] = field(default_factory=list)
    stop_reason: str | None = None   # the stop string that ended the request
    num_computed: int = 0            # tokens whose KV is in the cache
    block_ids: list[int] = field(default_factory=list)
    lora_slot: int = -1
    first_token_time: float | None = None
    token_times: list[float] = field(default_factory=list)
    finish_time: float | None = None
    seq_no: int = field(default_factory=lambda: next(_counter))
    # Route decision headers, filled by adapter routing.
    trace: dict = field(default_factory=dict)
    # Prefix caching: hashes of the request's full pages (chained), how many
    # of its pages are registered, and prompt tokens served from the cache.
    block_hashes: list = field(default_factory=list)
    num_registered: int = 0
    num_cached_tokens: int = 0

    @property
    def all_ids(self) -> list[int]:
        return self.prompt_ids + self.output_ids

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)

    @property
    def num_prompt(self) -> int:
        return len(self.prompt_ids)

    @property
    def in_prefill(self) -> bool:
        """True while more than the newest token lacks KV: a fresh prompt, a
        chunked prompt, or a request pre-empted by recompute (which must
        recompute its prompt AND the tokens it already produced before
        decoding continues)."""
        pending = self.num_tokens - self.num_computed
        return pending > 1 or (not self.output_ids and pending > 0)

    @property
    def remaining_prefill(self) -> int:
        """Tokens the prefill still has to process (the last one's logits give
        the next token)."""
        return self.num_tokens - self.num_computed if self.in_prefill else 0

    def finished(self) -> bool:
        return self.status in (Status.FINISHED, Status.ABORTED)

    def ttft(self) -> float | None:
        return None if self.first_token_time is None else self.first_token_time - self.arrival_time

    def tbts(self) -> list[float]:
        t = ([self.first_token_time] if self.first_token_time is not None else []) + self.token_times
        return [b - a for a, b in zip(t, t[1:])]
