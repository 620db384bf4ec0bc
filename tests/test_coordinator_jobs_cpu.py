"""The coordinator's buffer accounting (reservations, roll-back, capture,
the backward trigger when no sample fits or a flush is due) and the
finetuning-job stage declarations (subclass keys, prerequisites, spec
validation, a failing stage failing only its job)."""
import pytest

from deltaserve_vllm_b200.engine.ft.coordinator import FinetuneCoordinator
from deltaserve_vllm_b200.engine.ft_job import FinetuneJobSpec, FtJobManager, Stage, stage_keys


def test_reserve_rollback_capture_and_trigger():
    c = FinetuneCoordinator(capacity=100)
    c.min_sample_len = 20
    assert c.next_ft_budget() == 100
    s1, s2 = object(), object()
    assert c.reserve(30, [s1]) == 0 and c.reserve(40, [s2]) == 30
    assert c.space_remaining() == 30 and c.reserved_fill == 70
    c.unreserve(40, [s2])                                    # the step carrying s2 was rolled back
    assert c.reserved_fill == 30 and c.buffer_samples == [s1]
    assert not c.record_capture(30, [30])                   # 70 rows still free: no backward yet
    assert c.fill_count == 30 and c.reserved_fill == 0 and c.sample_lens == [30]
    assert c.reserve(55, [s2]) == 30
    assert not c.record_capture(25, [25])                   # rows of the step still in flight
    assert c.record_capture(30, [30])                       # 15 free < the smallest sample: train
    assert c.pending_backward and not c.admission_open and c.next_ft_budget() == 0
    trained = c.backward_done(85, 1.5, 10.0, 12.0)
    assert trained == [s1, s2] and c.fill_count == 0 and c.sample_lens == [] and c.admission_open
    assert c.total_trained_tokens == 85 and c.completed_cycles == 1


def test_flush_trains_a_partial_buffer():
    c = FinetuneCoordinator(capacity=100)
    c.reserve(10)
    c.note_injection(next_sample_len=None)                  # the corpus has no sample left
    assert c.epoch_flush_pending and not c.admission_open
    assert not c.try_flush()                                # rows still in flight
    assert c.record_capture(10)                             # the capture completes the flush
    c.backward_done(10, 1.0, 1.0, 1.0)
    c.disable("test")
    assert c.next_ft_budget() == 0 and not c.ft_started
    c.start()
    assert not c.ft_started                                 # disabling is sticky


def test_stage_declarations_and_validation():
    assert {"init", "training", "ready"} <= set(stage_keys())
    with pytest.raises(TypeError, match="needs a key"):
        class Nameless(Stage):                              # noqa: F841
            pass
    FinetuneJobSpec(stages=("init", "training", "ready")).validate()
    with pytest.raises(ValueError, match="needs stage 'training'"):
        FinetuneJobSpec(stages=("init", "ready")).validate()
    with pytest.raises(ValueError, match="unknown ft_job stage"):
        FinetuneJobSpec(stages=("init", "bake")).validate()
    with pytest.raises(ValueError, match="needs adapter_routing"):
        FinetuneJobSpec(stages=("init", "indexing")).validate(adapter_routing=False)
    with pytest.raises(ValueError, match="twice"):
        FinetuneJobSpec(stages=("init", "init")).validate()


def test_manager_runs_stages_in_prerequisite_order_and_contains_failures():
    seen = []

    class First(Stage, key="t-first"):
        def begin(self, job, ctx):
            seen.append("first")

        def settled(self, job, ctx):
            return ctx["ready"]

    class Second(Stage, key="t-second"):
        def prerequisites(self, listed):
            return ("t-first",)

        def begin(self, job, ctx):
            seen.append("second")

    class Broken(Stage, key="t-broken"):
        def begin(self, job, ctx):
            raise RuntimeError("boom")

    m = FtJobManager()
    job = m.submit(FinetuneJobSpec(name="j", stages=("t-second", "t-first")))
    m.tick({"ready": False})
    assert seen == ["first"] and job.stage_state == {"t-second": "pending", "t-first": "running"}
    m.tick({"ready": True})                                 # first settles; second waits for the next tick
    assert seen == ["first"] and job.stage_state["t-first"] == "done"
    m.tick({"ready": True})
    assert seen == ["first", "second"] and job.state == "done"
    bad = m.submit(FinetuneJobSpec(name="b", stages=("t-broken",)))
    m.tick({})
    assert bad.state == "failed" and "boom" in bad.error and job.state == "done"
