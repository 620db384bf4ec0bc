"""Finetuning coordinator: capture-buffer accounting, backward trigger and
acknowledgement, admission flags, throttles and failure detection.

Lifecycle of one buffer (reference: ``deltaserve-plugin/deltaserve/coordinator.py:484-962``):

* ``reserve(n)`` at scheduling time returns the row offset the step's FT rows
  are captured at; ``record_capture(n)`` after the forward commits them;
* the buffer triggers a backward when the next sample no longer fits
  (``space_remaining() < min_sample_len``) or at an epoch boundary / end of
  corpus ("flush"); admission closes while the backward is pending, so the next
  FT forward always sees the weights of the previous step;
* ``backward_done`` (the trainer finished and published) commits the trained
  samples, logs the cycle and reopens admission.

Failure handling: a backward that raises, or that has not finished after
``stuck_disable_s`` (warning after ``stuck_warn_s``), disables finetuning for
the rest of the run (sticky); inference continues.
"""

from __future__ import annotations

import csv
import os
import time
from collections import deque
from dataclasses import dataclass, field

from ... import dprint


class RpsTracker:
    def __init__(self, window_s: float = 1.0):
        self.window_s = float(window_s)
        self._t: deque = deque()

    def note(self, now: float) -> None:
        self._t.append(now)

    def rps(self, now: float) -> float:
        while self._t and self._t[0] < now - self.window_s:
            self._t.popleft()
        return len(self._t) / self.window_s if self.window_s > 0 else 0.0


@dataclass
class _FillBuffer:
    """The activation buffer's row accounting. ``reserved`` rows belong to
    finetuning rows admitted into a step that has not run yet; they become
    ``committed`` when the step's forward captured them (or go back when the
    step is rolled back). ``lens`` are the committed samples' lengths and
    ``samples`` the store items the next backward will train."""
    committed: int = 0
    reserved: int = 0
    lens: list = field(default_factory=list)
    samples: list = field(default_factory=list)

    def used(self) -> int:
        return self.committed + self.reserved

    def take(self, n: int, samples) -> int:
        """Reserve ``n`` rows; returns their first row."""
        first = self.used()
        self.reserved += int(n)
        self.samples.extend(samples or ())
        return first

    def give_back(self, n: int, samples) -> None:
        self.reserved = max(0, self.reserved - int(n))
        if samples:
            gone = {id(x) for x in samples}
            self.samples = [x for x in self.samples if id(x) not in gone]

    def commit(self, n: int, lens) -> None:
        self.committed += n
        self.reserved = max(0, self.reserved - n)
        self.lens.extend(int(x) for x in (lens or ()))

    def drain(self) -> list:
        """Empty the buffer after a backward; returns the trained samples."""
        out, self.samples = self.samples, []
        self.committed, self.lens = 0, []
        return out


class FinetuneCoordinator:
    def __init__(self, capacity: int, ft_started: bool = True, per_step_budget: int | None = None,
                 bwd_log_path: str | None = None, stuck_warn_s: float = 5.0,
                 stuck_disable_s: float = 60.0):
        self.capacity = int(capacity)
        self.per_step_budget = int(per_step_budget or capacity)
        self.ft_started = ft_started
        self.admission_open = True
        self.pending_backward = False
        self.disabled = False
        self.disabled_reason: str | None = None
        self.buf = _FillBuffer()
        self.min_sample_len = 1
        self.epoch_flush_pending = False
        self.current_epoch = 0
        self.cycle = 0
        self.completed_cycles = 0
        self.total_trained_tokens = 0
        self.last_loss: float | None = None
        self._t_trigger: float | None = None
        # When the buffer last became free to fill (the previous cycle's end):
        # the fill time of a cycle is the gap from there to its trigger.
        self._t_free: float | None = None
        self._fill_ms: float | None = None
        self._warned = False
        self.stuck_warn_s, self.stuck_disable_s = stuck_warn_s, stuck_disable_s
        self.rps = RpsTracker()
        self.rps_throttle_active = False
        self.rps_engaged_at: float | None = None
        self.fwd_throttle_active = False
        self.bwd_log_path = bwd_log_path
        self.history: list[dict] = []

    # Views of the buffer under the names the engine and the status use.
    @property
    def fill_count(self) -> int:
        return self.buf.committed

    @fill_count.setter
    def fill_count(self, v: int) -> None:
        self.buf.committed = int(v)

    @property
    def reserved_fill(self) -> int:
        return self.buf.reserved

    @property
    def sample_lens(self) -> list:
        return self.buf.lens

    @sample_lens.setter
    def sample_lens(self, v) -> None:
        self.buf.lens = list(v)

    @property
    def buffer_samples(self) -> list:
        return self.buf.samples

    @buffer_samples.setter
    def buffer_samples(self, v) -> None:
        self.buf.samples = list(v)

    # ------------------------------------------------------------ flags
    def space_remaining(self) -> int:
        return max(0, self.capacity - self.buf.used())

    def next_ft_budget(self) -> int:
        if self.disabled or not self.ft_started or not self.admission_open or self.pending_backward:
            return 0
        return min(self.per_step_budget, self.space_remaining())

    def start(self) -> None:
        if not self.disabled:
            self.ft_started = True
            self.admission_open = True

    def stop(self) -> None:
        self.ft_started = False

    def disable(self, reason: str) -> None:
        """Sticky: finetuning stays off for the rest of the run."""
        if not self.disabled:
            dprint(f"[coord] finetuning DISABLED: {reason}")
        self.disabled = True
        self.disabled_reason = reason
        self.ft_started = False
        self.admission_open = False

    # ------------------------------------------------------------ buffer
    def reserve(self, n: int, samples: list | None = None) -> int:
        return self.buf.take(n, samples)

    def unreserve(self, n: int, samples: list | None = None) -> None:
        """Roll back a reservation whose step did not run (or was pre-empted).
        The admission that made it may have closed the buffer for a flush;
        with its rows gone that decision is re-made at the next admission."""
        self.buf.give_back(n, samples)
        if not self.pending_backward and not self.disabled and self.ft_started:
            self.epoch_flush_pending = False
            self.admission_open = True

    def note_injection(self, next_sample_len: int | None, admitted_now: int = 0) -> None:
        """After an admission: close the buffer (flush pending) when the
        smallest remaining sample can no longer fit, or the corpus/epoch is done."""
        if self.pending_backward or self.buf.used() + admitted_now <= 0:
            return
        space = self.space_remaining() - admitted_now
        if next_sample_len is None or next_sample_len > space:
            self.epoch_flush_pending = True
            self.admission_open = False

    def record_capture(self, n: int, sample_lens: list[int] | None = None) -> bool:
        """Commit ``n`` captured rows; returns True when a backward should start."""
        if n <= 0:
            return False
        self.buf.commit(n, sample_lens)
        # A backward starts once nothing is in flight and either no sample
        # fits any more or a flush was asked for.
        full = self.space_remaining() < self.min_sample_len
        if not self.pending_backward and self.buf.reserved == 0 and (full or self.epoch_flush_pending):
            return self._trigger()
        return False

    def try_flush(self) -> bool:
        """Train a partial buffer that no further FT forward will fill."""
        idle = not self.pending_backward and not self.disabled and self.buf.reserved == 0
        if idle and self.epoch_flush_pending and self.buf.committed > 0:
            return self._trigger()
        return False

    def _trigger(self) -> bool:
        self.admission_open = False
        self.pending_backward = True
        self.epoch_flush_pending = False
        self.cycle += 1
        self._t_trigger = time.monotonic()
        self._fill_ms = (self._t_trigger - self._t_free) * 1e3 if self._t_free is not None else None
        self._warned = False
        return True

    def backward_done(self, n: int, loss: float, gpu_ms: float, wall_ms: float,
                      epoch: int | None = None) -> list:
        """A cycle finished: returns the samples it trained (to commit)."""
        trained = self.buf.drain()
        self.total_trained_tokens += int(n)
        self.completed_cycles += 1
        self.last_loss = loss
        rec = {"time": time.time(), "cycle": self.cycle, "epoch": self.current_epoch if epoch is None else epoch,
               "batch_tokens": int(n), "loss": float(loss), "gpu_ms": float(gpu_ms),
               "wall_ms": float(wall_ms), "total_tokens": self.total_trained_tokens,
               "fill_ms": self._fill_ms}
        self._t_free = time.monotonic()
        self.history.append(rec)
        self._log(rec)
        self.pending_backward = False
        self._t_trigger = None
        if not self.disabled and not self.rps_throttle_active:
            self.admission_open = True
        return trained

    def _log(self, rec: dict) -> None:
        if not self.bwd_log_path:
            return
        new = not os.path.exists(self.bwd_log_path)
        if os.path.dirname(self.bwd_log_path):
            os.makedirs(os.path.dirname(self.bwd_log_path), exist_ok=True)
        with open(self.bwd_log_path, "a", newline="") as f:
            w = csv.writer(f)
            if new:
                w.writerow(["timestamp", "epoch", "batch_idx", "batch_tokens", "batch_loss",
                            "total_processed_tokens"])
            w.writerow([rec["time"], rec["epoch"], rec["cycle"], rec["batch_tokens"], rec["loss"],
                        rec["total_tokens"]])

    # ------------------------------------------------------------ health
    def check_stuck(self, backward_alive: bool = True) -> None:
        """Warn after ``stuck_warn_s``; disable after ``stuck_disable_s`` or when
        the backward is gone."""
        if not self.pending_backward or self._t_trigger is None:
            return
        el = time.monotonic() - self._t_trigger
        if not backward_alive:
            self.disable("backward worker died")
        elif el > self.stuck_disable_s:
            self.disable(f"backward stuck for {el:.0f}s")
        elif el > self.stuck_warn_s and not self._warned:
            self._warned = True
            dprint(f"[coord] WARNING: backward cycle {self.cycle} running for {el:.1f}s")

    # ------------------------------------------------------------ throttles
    def note_arrival(self, now: float) -> None:
        self.rps.note(now)

    def check_rps_throttle(self, now: float, close_rps: float, open_rps: float, window_s: float,
                           close_time: float = 0.0) -> None:
        """Close admission while the arrival rate is above ``close_rps``; reopen
        below ``open_rps`` (held at least ``close_time`` s unless the rate is 0)."""
        if close_rps <= 0:
            return
        self.rps.window_s = float(window_s)
        cur = self.rps.rps(now)
        if self.rps_throttle_active:
            held = now - (self.rps_engaged_at or now)
            if cur < open_rps and (close_time <= 0 or held >= close_time or cur == 0.0):
                self.rps_throttle_active = False
                self.rps_engaged_at = None
                if not self.pending_backward and not self.disabled:
                    self.admission_open = True
            else:
                self.admission_open = False
        elif cur > close_rps:
            self.rps_throttle_active = True
            self.rps_engaged_at = now
            self.admission_open = False

    def status(self) -> dict:
        return {"ft_started": self.ft_started, "disabled": self.disabled,
                "disabled_reason": self.disabled_reason, "admission_open": self.admission_open,
                "pending_backward": self.pending_backward, "fill": self.fill_count,
                "reserved": self.reserved_fill, "capacity": self.capacity, "cycle": self.cycle,
                "completed_cycles": self.completed_cycles,
                "total_trained_tokens": self.total_trained_tokens, "last_loss": self.last_loss,
                "epoch": self.current_epoch, "rps_throttle_active": self.rps_throttle_active}
