"""Finetuning jobs: a job is an ordered list of *stages* (``init`` ->
``training`` -> optional ``ready``; with adapter routing also ``indexing`` and
``admission``), run by :class:`FtJobManager` one job at a time from a queue
(reference: ``deltaserve-plugin/deltaserve/ft_job.py:66-429``)."""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any

DEFAULT_STAGES = ("init", "training")
GATED_STAGES = {"indexing": "adapter_routing.enable_adapter_routing",
                "admission": "adapter_routing.enable_adapter_routing"}
JOB_META_KEYS = ("name", "stages", "auto_routing", "adapter_init", "save_path")


class Stage:
    """One step of a finetuning job. A subclass declares itself with
    ``class Foo(Stage, key="foo")`` and job specs can then list ``foo``.
    ``begin`` runs once, when every prerequisite stage of the job is done;
    ``settled`` is asked on every engine tick after that until it is True.
    Stage objects hold no state of their own (they are made afresh each
    tick); a stage keeps its working state in ``job.data``."""

    key: str = ""
    _kinds: dict[str, type["Stage"]] = {}

    def __init_subclass__(cls, key: str = "", **kw):
        super().__init_subclass__(**kw)
        if not key:
            raise TypeError(f"{cls.__name__}: a stage needs a key (class {cls.__name__}(Stage, key=...))")
        cls.key = key
        Stage._kinds[key] = cls

    def prerequisites(self, listed: tuple[str, ...]) -> tuple[str, ...]:
        """The stages of this job (``listed``) that must be done first."""
        return ()

    def begin(self, job: "FinetuneJob", ctx: Any) -> None:
        pass

    def settled(self, job: "FinetuneJob", ctx: Any) -> bool:
        return True


def stage_keys() -> tuple[str, ...]:
    return tuple(Stage._kinds)


def load_gated_stages(adapter_routing: bool) -> None:
    if adapter_routing and "indexing" not in Stage._kinds:
        from ..adapters.routing import stages  # noqa: F401  (declares them)


class InitStage(Stage, key="init"):
    """The job's adapter weights and dataset are in place. The launch job's
    were loaded at engine start; a later job switches the trainer (adapter
    init, optimiser settings) and the corpus once the previous job's samples
    have all been trained (``ctx.begin_job`` returns False until then)."""

    def settled(self, job, ctx) -> bool:
        switch = getattr(ctx, "begin_job", None)
        if switch is not None and not switch(job):
            return False
        store = getattr(ctx, "store", None)
        return store is None or len(store) > 0


class TrainingStage(Stage, key="training"):
    """Done once the corpus finished every epoch and the last backward landed."""

    def prerequisites(self, listed):
        return tuple(k for k in ("init",) if k in listed)

    def begin(self, job, ctx) -> None:
        # Admission opens now unless the launch config keeps it closed until
        # POST /start_finetuning.
        coord, cfg = getattr(ctx, "coord", None), getattr(ctx, "ftcfg", None)
        if coord is not None and getattr(cfg, "start_on_launch", True):
            coord.start()

    def settled(self, job, ctx) -> bool:
        store, coord = getattr(ctx, "store", None), getattr(ctx, "coord", None)
        if store is None or coord is None:
            return True
        drained = not coord.pending_backward and coord.fill_count == 0
        return drained and store.finished()


class ReadyStage(Stage, key="ready"):
    """The trained adapter is saved (when the job names a save path)."""

    def prerequisites(self, listed):
        return ("training",)

    def begin(self, job, ctx) -> None:
        save = getattr(ctx, "save_job_adapter", None)
        if save is not None and job.spec.save_path:
            save(job)


@dataclass
class FinetuneJobSpec:
    name: str = "default"
    stages: tuple[str, ...] = DEFAULT_STAGES
    adapter_path: str | None = None
    data_path: str | None = None
    num_epochs: int = 1
    learning_rate: float = 1e-4
    weight_decay: float = 0.0
    gamma: float = 1.0
    auto_routing: bool = False
    adapter_init: str | None = None
    save_path: str | None = None

    @classmethod
    def from_finetune_config(cls, cfg) -> "FinetuneJobSpec":
        meta = dict(cfg.ft_job or {})
        unknown = sorted(set(meta) - set(JOB_META_KEYS))
        if unknown:
            raise ValueError(f"unknown ft_job key(s) {unknown}")
        stages = meta.get("stages", DEFAULT_STAGES)
        if isinstance(stages, str) or not all(isinstance(s, str) for s in stages):
            raise ValueError("ft_job.stages must be a list of stage names")
        return cls(name=meta.get("name", "default"), stages=tuple(stages),
                   adapter_path=cfg.finetuning_lora_path, data_path=cfg.data_path,
                   num_epochs=cfg.num_epochs, learning_rate=cfg.learning_rate,
                   weight_decay=cfg.weight_decay, gamma=cfg.gamma,
                   auto_routing=bool(meta.get("auto_routing", False)),
                   adapter_init=meta.get("adapter_init"), save_path=meta.get("save_path"))

    def validate(self, adapter_routing: bool = False) -> None:
        load_gated_stages(adapter_routing)
        for s in self.stages:
            if s in GATED_STAGES and not adapter_routing:
                raise ValueError(f"ft_job stage '{s}' needs {GATED_STAGES[s]}: true")
            if s not in Stage._kinds:
                raise ValueError(f"unknown ft_job stage '{s}' (known: {sorted(Stage._kinds)})")
        if len(set(self.stages)) != len(self.stages):
            raise ValueError("ft_job.stages lists a stage twice")
        for s in self.stages:
            missing = [k for k in Stage._kinds[s]().prerequisites(self.stages) if k not in self.stages]
            if missing:
                raise ValueError(f"stage '{s}' needs stage '{missing[0]}'")
        if self.adapter_init not in (None, "from_path", "random"):
            raise ValueError(f"ft_job.adapter_init '{self.adapter_init}' is not supported; "
                             "available: ['from_path', 'random']")


@dataclass
class FinetuneJob:
    spec: FinetuneJobSpec
    job_id: int = 0
    state: str = "queued"          # queued | running | done | failed | cancelled
    stage_state: dict = field(default_factory=dict)
    created: float = field(default_factory=time.time)
    started: float | None = None
    finished: float | None = None
    error: str | None = None
    # Per-stage working state (stage objects are re-created every tick).
    data: dict = field(default_factory=dict)
    report: dict | None = None

    def status(self) -> dict:
        return {"job_id": self.job_id, "name": self.spec.name, "state": self.state,
                "stages": dict(self.stage_state), "error": self.error,
                "created": self.created, "started": self.started, "finished": self.finished}


class FtJobManager:
    """Runs queued jobs one at a time; ``tick(ctx)`` advances stages."""

    def __init__(self):
        self.jobs: list[FinetuneJob] = []
        self._next_id = 1

    def submit(self, spec: FinetuneJobSpec, adapter_routing: bool = False) -> FinetuneJob:
        spec.validate(adapter_routing)
        job = FinetuneJob(spec, self._next_id)
        self._next_id += 1
        job.stage_state = {s: "pending" for s in spec.stages}
        self.jobs.append(job)
        return job

    def current(self) -> FinetuneJob | None:
        for j in self.jobs:
            if j.state in ("queued", "running"):
                return j
        return None

    def cancel(self, job_id: int) -> bool:
        for j in self.jobs:
            if j.job_id == job_id and j.state in ("queued", "running"):
                j.state = "cancelled"
                j.finished = time.time()
                return True
        return False

    def tick(self, ctx: Any) -> None:
        job = self.current()
        if job is None:
            return
        if job.state == "queued":
            job.state = "running"
            job.started = time.time()
        listed = job.spec.stages
        for key in listed:
            phase = job.stage_state[key]
            if phase == "done":
                continue
            stage = Stage._kinds[key]()
            if not all(job.stage_state.get(k) == "done" for k in stage.prerequisites(listed)):
                continue
            try:
                if phase == "pending":
                    stage.begin(job, ctx)
                    job.stage_state[key] = "running"
                if stage.settled(job, ctx):
                    job.stage_state[key] = "done"
            except Exception as e:  # a failing stage fails the job, not the engine
                job.state = "failed"
                job.error = f"{key}: {e!r}"
                job.finished = time.time()
                return
        if all(v == "done" for v in job.stage_state.values()):
            job.state = "done"
            job.finished = time.time()

    def status(self) -> list[dict]:
        return [j.status() for j in self.jobs]
