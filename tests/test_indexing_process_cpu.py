"""Indexing off the serving process: the CPU encoder process (low scheduling
priority, same embeddings as in-process), the weight-sharing encoder process
(built around the parent's tensors, gated per layer by the grant byte), the
busy/idle placement, and the indexing service moving chunks between the
executors (a preempted GPU chunk is redone on the CPU; the centroid is the
one a plain CPU pass gives). Behaviour follows the reference's
``tests/test_adapter_indexing.py`` and ``adapter_routing/runner.py:40-230``."""
import os
import tempfile
import time

import numpy as np
import pytest

from deltaserve_vllm_b200.adapters.routing.encoder import HashingEncoder, SentenceEncoder
from deltaserve_vllm_b200.adapters.routing.index import Indexer, l2_normalize
from deltaserve_vllm_b200.adapters.routing.index_process import (EncoderProcess, IndexGrant, InlineExecutor,
                                                                 Preempted, _install_grant_checks, parse_cpus)
from deltaserve_vllm_b200.adapters.routing.indexing import BUSY, IDLE, IndexingPlacement, IndexingService

TEXTS = [f"sample {i} about topic {i % 5} with words {' '.join(str(j) for j in range(i % 7))}"
         for i in range(53)]


def tiny_bert_dir(d: str, layers: int = 3) -> str:
    """A random 3-layer BERT and its tokenizer, saved where SentenceEncoder reads them."""
    import torch
    from transformers import BertConfig, BertModel, BertTokenizerFast
    words = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]", "query", ":", "sample", "about", "topic",
             "with", "words"] + [str(i) for i in range(60)]
    BertTokenizerFast(vocab={w: i for i, w in enumerate(words)}).save_pretrained(d)
    torch.manual_seed(0)
    cfg = BertConfig(vocab_size=len(words), hidden_size=32, num_hidden_layers=layers, num_attention_heads=2,
                     intermediate_size=64, max_position_embeddings=64)
    BertModel(cfg).save_pretrained(d)
    return d


def test_parse_cpus():
    assert parse_cpus("0-2,5, 7-8") == [0, 1, 2, 5, 7, 8]
    assert parse_cpus(None) is None and parse_cpus("") is None
    assert parse_cpus([3, 1, 3]) == [1, 3]
    with pytest.raises(ValueError):
        parse_cpus("4-2")


def test_cpu_process_matches_in_process_and_runs_at_idle_priority():
    enc = HashingEncoder(dim=256, prefix="query: ")
    ex = EncoderProcess(enc, "cpu", cpus=[0], name="cpu").start()
    try:
        assert ex.info["priority"] in ("SCHED_IDLE", "nice 19")
        if ex.info["priority"] == "SCHED_IDLE":
            assert os.sched_getscheduler(ex.pid) == os.SCHED_IDLE
        assert os.sched_getaffinity(ex.pid) == {0}
        got = ex.encode(TEXTS[:20], threads=1)
        np.testing.assert_allclose(got, enc.encode(TEXTS[:20]), rtol=0, atol=1e-6)
        # a cancelled chunk's late answer is dropped, the next one is returned
        ex.submit(TEXTS[:5])
        ex.cancel()
        got = ex.encode(TEXTS[5:9])
        np.testing.assert_allclose(got, enc.encode(TEXTS[5:9]), atol=1e-6)
        with pytest.raises(RuntimeError):
            ex.submit(TEXTS[:1]); ex.submit(TEXTS[:1])   # noqa: E702 -- one chunk in flight
    finally:
        ex.stop()
    assert not ex.ready


def test_shared_weight_process_uses_parent_tensors_and_obeys_grant():
    with tempfile.TemporaryDirectory() as d:
        tiny_bert_dir(d)
        parent = SentenceEncoder(d, "query: ", 32, "cpu")
        want = parent.encode(TEXTS[:12])
        grant = IndexGrant()
        grant.set(True)
        desc = SentenceEncoder(d, "query: ", 32, "cpu")
        ex = EncoderProcess(desc, "cpu", shared=parent.shared_state(), grant=grant, low_priority=False,
                            name="gpu").start()
        try:
            assert ex.info["layers_checked"] == 3
            np.testing.assert_allclose(ex.encode(TEXTS[:12]), want, rtol=1e-5, atol=1e-6)
            # the same storage: a change in the parent's weights shows in the child
            import torch
            with torch.no_grad():
                parent._model.embeddings.word_embeddings.weight.mul_(2.0)
            changed = parent.encode(TEXTS[:4])
            np.testing.assert_allclose(ex.encode(TEXTS[:4]), changed, rtol=1e-5, atol=1e-6)
            grant.set(False)
            with pytest.raises(Preempted):
                ex.encode(TEXTS[:4])
            grant.set(True)
            assert ex.encode(TEXTS[:2]).shape == (2, 32)
        finally:
            ex.stop()


def test_grant_check_stops_the_forward_between_layers():
    with tempfile.TemporaryDirectory() as d:
        tiny_bert_dir(d, layers=4)
        enc = SentenceEncoder(d, "query: ", 32, "cpu")
        grant = IndexGrant()
        grant.set(True)
        assert _install_grant_checks(enc, grant) == 4
        seen = []
        layers = enc.layers()
        # clear the grant from inside layer 1: layers 2 and 3 must not run
        layers[1].register_forward_hook(lambda *_: grant.set(False))
        for i, layer in enumerate(layers):
            layer.register_forward_pre_hook(lambda _m, _a, i=i: seen.append(i))
        with pytest.raises(Preempted):
            enc.encode(TEXTS[:3])
        assert seen == [0, 1]


def test_placement_levels_and_grant():
    now = [100.0]
    grant = IndexGrant()
    p = IndexingPlacement(gpu_after_quiet_s=3.0, grant=grant, idle_threads=8, busy_threads=2,
                          clock=lambda: now[0])
    assert not grant.granted                      # nothing granted before the first look
    assert p.level() == IDLE and grant.granted and p.cpu_threads() == 8 and p.use_gpu(True)
    assert not p.use_gpu(False)
    p.note_inference()
    assert not grant.granted                      # cleared in the same call
    assert p.level() == BUSY and p.cpu_threads() == 2 and not p.use_gpu(True)
    now[0] += 2.9
    assert p.level() == BUSY
    now[0] += 0.2
    assert p.level() == IDLE and grant.granted
    assert p.changes == 2


class _FakeGpu:
    """A GPU executor stand-in: encodes in-thread, answers Preempted when the
    grant is cleared at submit time (what the real child does at its next layer)."""

    device, ready, info = "gpu", True, {}

    def __init__(self, enc, grant, fail=False):
        self.enc, self.grant, self.fail = enc, grant, fail
        self.job = None
        self.submitted = 0

    def submit(self, texts, threads=0):
        self.submitted += 1
        self.job = ("pre",) if not self.grant.granted else ("err",) if self.fail \
            else ("ok", self.enc.encode(texts))

    def poll(self, timeout=0.0):
        job, self.job = self.job, None
        if job is None:
            return None
        if job[0] == "pre":
            raise Preempted()
        if job[0] == "err":
            raise RuntimeError("device out of memory")
        return job[1]

    def cancel(self):
        self.job = None

    def stop(self):
        pass

    def describe(self):
        return {"name": "gpu"}


def _wait(job, s=30.0):
    t0 = time.time()
    while not job.finished and time.time() - t0 < s:
        time.sleep(0.01)
    assert job.finished, job.describe()


def _want(enc, texts):
    return l2_normalize(l2_normalize(enc.encode(texts).astype(np.float64)).mean(0))


def test_service_idle_uses_gpu_busy_uses_cpu_and_centroid_is_exact():
    enc = HashingEncoder(dim=64)
    grant = IndexGrant()
    p = IndexingPlacement(gpu_after_quiet_s=1000.0, grant=grant)
    gpu = _FakeGpu(enc, grant)
    svc = IndexingService({"cpu": InlineExecutor(enc), "gpu": gpu}, p, chunk={"cpu": 4, "gpu": 8}, poll_s=0.001)
    try:
        a = svc.submit("idle", Indexer(TEXTS, "fp"))          # never any inference: all on the GPU
        _wait(a)
        assert a.done and a.chunks["gpu"] == 7 and a.chunks["cpu"] == 0
        np.testing.assert_allclose(a.indexer.centroid(), _want(enc, TEXTS), rtol=1e-5, atol=1e-6)
        p.note_inference()                                    # busy for the quiet period
        b = svc.submit("busy", Indexer(TEXTS[:20], "fp"))
        _wait(b)
        assert b.done and b.chunks == {"cpu": 5, "gpu": 0}
        np.testing.assert_allclose(b.indexer.centroid(), _want(enc, TEXTS[:20]), rtol=1e-5, atol=1e-6)
    finally:
        svc.stop()


def test_service_redoes_preempted_and_failed_gpu_chunks_on_cpu():
    enc = HashingEncoder(dim=64)
    grant = IndexGrant()
    p = IndexingPlacement(gpu_after_quiet_s=0.0, grant=grant)

    class Racy(_FakeGpu):
        # an arrival lands while every other GPU chunk is in flight
        def submit(self, texts, threads=0):
            super().submit(texts, threads)
            if self.submitted % 2 == 1:
                self.job = ("pre",)

    svc = IndexingService({"cpu": InlineExecutor(enc), "gpu": Racy(enc, grant)}, p, chunk=4, poll_s=0.001)
    try:
        j = svc.submit("racy", Indexer(TEXTS, "fp"))
        _wait(j)
        assert j.done and j.preempted > 0 and j.discarded >= j.preempted
        np.testing.assert_allclose(j.indexer.centroid(), _want(enc, TEXTS), rtol=1e-5, atol=1e-6)
    finally:
        svc.stop()
    svc = IndexingService({"cpu": InlineExecutor(enc), "gpu": _FakeGpu(enc, grant, fail=True)}, p, chunk=4,
                          poll_s=0.001)
    try:
        j = svc.submit("oom", Indexer(TEXTS[:16], "fp"))
        _wait(j)
        # one GPU failure, then the CPU for the back-off period
        assert j.done and j.chunks == {"cpu": 4, "gpu": 0} and j.discarded == 1
    finally:
        svc.stop()


def test_service_failure_and_stop_and_cpu_pause():
    class Broken:
        def encode(self, texts):
            raise ValueError("bad sample")

    p = IndexingPlacement(gpu_after_quiet_s=0.0)
    svc = IndexingService({"cpu": InlineExecutor(Broken())}, p, chunk=4, poll_s=0.001)
    try:
        j = svc.submit("x", Indexer(TEXTS[:8], "fp"))
        _wait(j)
        assert j.state == "failed" and "bad sample" in j.error
    finally:
        svc.stop()
    # busy_threads = 0: CPU indexing pauses while inference runs
    p = IndexingPlacement(gpu_after_quiet_s=1000.0, busy_threads=0)
    p.note_inference()
    svc = IndexingService({"cpu": InlineExecutor(HashingEncoder(dim=16))}, p, chunk=4, poll_s=0.001,
                          recheck_s=0.01)
    try:
        j = svc.submit("paused", Indexer(TEXTS[:8], "fp"))
        time.sleep(0.2)
        assert j.state == "paused" and j.indexer.progress[0] == 0
        p.gpu_after_quiet_s = 0.0                    # quiet: CPU at full width
        _wait(j)
        assert j.done
        k = svc.submit("stopped", Indexer(TEXTS, "fp"))
        k.stop()
        _wait(k)
        assert k.state == "stopped"
    finally:
        svc.stop()


def test_service_with_real_cpu_process_end_to_end():
    enc = HashingEncoder(dim=128)
    p = IndexingPlacement(gpu_after_quiet_s=0.0)
    svc = IndexingService({"cpu": EncoderProcess(enc, "cpu").start()}, p, chunk=8)
    try:
        jobs = [svc.submit(f"j{i}", Indexer(TEXTS[i * 10:], "fp")) for i in range(3)]
        for j in jobs:
            _wait(j, 120)
        for i, j in enumerate(jobs):
            assert j.done
            np.testing.assert_allclose(j.indexer.centroid(), _want(enc, TEXTS[i * 10:]), rtol=1e-5, atol=1e-6)
        assert svc.describe()["executors"]["cpu"]["running"]
    finally:
        svc.stop()
