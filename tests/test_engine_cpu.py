"""End-to-end co-serving on CPU (fp32 oracle ops): inference requests and
finetuning samples share steps, backward cycles run, the adapter is published
and saved, and FT rows never produce outputs."""
import os
import tempfile

import torch

from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine, FT_ADAPTER_NAME
from deltaserve_vllm_b200.engine.request import SamplingParams
from deltaserve_vllm_b200.adapters import peft_io


def make_engine(tmp, **ft):
    ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=512, block_size=16,
                        max_num_batched_tokens=256, max_loras=3, max_lora_rank=8)
    fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=96,
                          learning_rate=1e-3, adapter_save_path=os.path.join(tmp, "ckpt"),
                          bwd_log_path=os.path.join(tmp, "bwd.csv"), **ft)
    store = FinetuningStore.synthetic(1024, 12, 16, 40, seed=0, max_saved_finetuning_tokens=96,
                                      total_epochs=2)
    eng = CoServingEngine(ecfg, fcfg, ft_store=store)
    eng.load_inference_adapter("toy", rank=8, alpha=16)
    return eng


def test_coserving_cpu_end_to_end():
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)
        g = torch.Generator().manual_seed(0)
        for i in range(6):
            eng.add_request(f"r{i}", torch.randint(0, 1024, (20 + 7 * i,), generator=g).tolist(),
                            SamplingParams(max_tokens=5), adapter="toy" if i % 2 else None)
        eng.run_until_idle(max_steps=2000)
        st = eng.finetuning_status()
        assert st["completed_cycles"] >= 2, st
        assert all(l == l for l in eng.trainer.losses)  # finite
        assert len(eng.finished) == 6 and all(len(r.output_ids) == 5 for r in eng.finished)
        assert not any(r.is_ft for r in eng.finished)
        assert eng.store.finished()
        assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks
        path = eng.save_adapter(save_id="x1")
        tensors, cfg = peft_io.read_adapter(path)
        assert len(tensors) == 2 * 7 * eng.arch.num_layers
        assert os.path.exists(os.path.join(tmp, "bwd.csv"))


def test_launch_profiling_fits_estimator_cpu():
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)
        eng.profile_execution_model(repeats=1)
        assert eng.estimator.is_ready
        assert not eng.coord.disabled
        assert not eng.has_unfinished()
        assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks
        assert eng.stats["ft_tokens_forwarded"] == 0


def test_profiling_failure_disables_finetuning(monkeypatch):
    monkeypatch.setenv("DSERVE_TEST_FAIL_PROFILING", "1")
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)
        eng.profile_execution_model(repeats=1)
        assert eng.coord.disabled and "profiling" in eng.coord.disabled_reason
        eng.add_request("x", list(range(10)), SamplingParams(max_tokens=2))
        eng.run_until_idle(max_steps=100)
        assert len(eng.finished) == 1 and eng.stats["ft_tokens_forwarded"] == 0


def test_recompute_matches_saved_activations_cpu():
    """save_attn_qkv / save_attn_ctx / save_resid_mid off: the backward
    recomputes those activations; losses and trained adapters match the run
    that captured them."""
    import tempfile as _tf
    outs = []
    for flags in ({}, {"save_attn_qkv": False, "save_attn_ctx": False, "save_resid_mid": False}):
        with _tf.TemporaryDirectory() as tmp:
            eng = make_engine(tmp, **flags)
            eng.run_until_idle(max_steps=2000)
            outs.append((list(eng.trainer.losses), eng.trainer.export_full()))
    (l0, a0), (l1, a1) = outs
    assert len(l0) == len(l1) >= 2
    for x, y in zip(l0, l1):
        assert abs(x - y) < 1e-3 * max(1.0, abs(x)), (l0, l1)
    for k in a0:
        torch.testing.assert_close(a0[k], a1[k], rtol=1e-3, atol=1e-5)


def test_save_activations_off_trains_nothing_cpu():
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp, save_activations=False)
        eng.run_until_idle(max_steps=2000)
        assert eng.capture is None
        assert eng.trainer.step == 0
        assert eng.store.finished()            # samples were forwarded and retired
        assert eng.coord.completed_cycles >= 1


def test_tier_c_abort_ft_only_step_cpu():
    """An FT-only forward pre-empted between layers (tier C) releases its
    rows (KV pages, capture reservation, claimed samples); training then
    proceeds normally."""
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp, forward_interruptible=True, ft_only_admission_grace_ms=0)
        orig = eng.runner.abort_hook
        state = {"n": 0}

        def patched(should_abort, vote=None, ahead=2):
            def sa():
                state["n"] += 1
                return state["n"] == 2          # a request "arrives" before layer 1
            return orig(sa, vote, ahead)
        eng.runner.abort_hook = patched
        eng.step()
        assert eng.stats.get("ft_aborts") == 1
        assert eng.coord.reserved_fill == 0 and eng.coord.fill_count == 0
        assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks
        eng.runner.abort_hook = orig
        eng.run_until_idle(max_steps=2000)
        assert eng.coord.completed_cycles >= 2
        assert eng.store.finished()


def test_backward_failure_disables_finetuning_sticky(monkeypatch):
    """A backward cycle that raises (injected on the host) switches
    finetuning off for the rest of the run; inference keeps serving and a
    later start request does not re-enable it."""
    from deltaserve_vllm_b200.engine import llm_engine
    monkeypatch.setattr(llm_engine, "_FAIL_BACKWARD_AT", 1)
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)
        g = torch.Generator().manual_seed(1)
        for i in range(4):
            eng.add_request(f"r{i}", torch.randint(0, 1024, (30,), generator=g).tolist(),
                            SamplingParams(max_tokens=6))
        eng.run_until_idle(max_steps=2000)
        assert eng.stats.get("bwd_failures") == 1
        assert eng.coord.disabled and "backward failed" in eng.coord.disabled_reason
        assert not eng.bwd_active and eng.trainer.step == 0
        assert len(eng.finished) == 4 and all(len(r.output_ids) == 6 for r in eng.finished)
        eng.start_finetuning()
        assert eng.coord.disabled and not eng.coord.admission_open
        eng.add_request("late", list(range(40)), SamplingParams(max_tokens=3))
        fwd = eng.stats["ft_tokens_forwarded"]
        eng.run_until_idle(max_steps=200)
        assert eng.finished[-1].request_id == "late" and eng.stats["ft_tokens_forwarded"] == fwd
        assert eng.finetuning_status()["disabled"]
        assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks


def test_lora_slot_limit_with_pinned_ft_slot():
    """max_loras counts the pinned finetuning slot: with max_loras=3 two
    inference adapters fit, a third is refused, and requests of every loaded
    adapter are co-batched with FT rows (the reference's scheduler edge case
    ``tests/test_ft_lora_limit.py``: FT rows must not be starved by the slot
    limit)."""
    import pytest
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)                  # loads "toy" (max_loras=3: toy + FT + one more)
        eng.load_inference_adapter("second", rank=8, alpha=16, seed=3)
        with pytest.raises(RuntimeError, match="no free LoRA slot"):
            eng.load_inference_adapter("third", rank=8, alpha=16, seed=4)
        g = torch.Generator().manual_seed(5)
        for i, ad in enumerate(["toy", "second", None, "toy"]):
            eng.add_request(f"r{i}", torch.randint(0, 1024, (25,), generator=g).tolist(),
                            SamplingParams(max_tokens=4), adapter=ad)
        eng.run_until_idle(max_steps=2000)
        assert len(eng.finished) == 4
        assert eng.stats["ft_tokens_forwarded"] > 0 and eng.coord.completed_cycles >= 1
        eng.unload_inference_adapter("second")
        eng.load_inference_adapter("third", rank=8, alpha=16, seed=4)   # the freed slot is reusable


def test_tp_diag_recompute_matches_capture(monkeypatch):
    """DSERVE_TP_DIAG: the backward's recompute of every captured activation
    agrees with what the serving forward captured."""
    monkeypatch.setenv("DSERVE_TP_DIAG", "2")
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)
        eng.run_until_idle(max_steps=2000)
        log = eng.trainer.diag_log
        assert len(log) == 2 * eng.arch.num_layers
        for rec in log:
            assert rec["qkv"] < 1e-4 and rec["ctx"] < 1e-4 and rec["resid_mid"] < 1e-4, rec


def test_prefix_caching_engine_adapters_versions_and_ft():
    """Engine with prefix caching and co-served finetuning: pages are shared
    only between requests of the same adapter version, requests on the
    adapter being trained and FT rows never use or feed the cache."""
    with tempfile.TemporaryDirectory() as tmp:
        ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=512, block_size=16,
                            max_num_batched_tokens=256, max_loras=3, max_lora_rank=8,
                            enable_prefix_caching=True)
        fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=96, learning_rate=1e-3)
        store = FinetuningStore.synthetic(1024, 12, 16, 40, seed=0, max_saved_finetuning_tokens=96)
        eng = CoServingEngine(ecfg, fcfg, ft_store=store)
        eng.load_inference_adapter("toy", rank=8, alpha=16)
        prefix = list(range(100, 180))                           # 5 full pages
        sched = eng.scheduler

        def run(rid, adapter, tail):
            eng.add_request(rid, prefix + tail, SamplingParams(max_tokens=3), adapter=adapter)
            eng.run_until_idle(max_steps=500)
            return next(r for r in eng.finished if r.request_id == rid)

        assert run("a0", None, [1, 2]).num_cached_tokens == 0
        assert run("a1", None, [3]).num_cached_tokens == 80        # same (base) prefix
        assert run("b0", "toy", [4]).num_cached_tokens == 0        # other adapter: other K/V
        assert run("b1", "toy", [5]).num_cached_tokens == 80
        eng.unload_inference_adapter("toy")
        eng.load_inference_adapter("toy", rank=8, alpha=16, seed=77)   # new weights, same slot
        assert run("b2", "toy", [6]).num_cached_tokens == 0
        assert run("f0", FT_ADAPTER_NAME, [7]).num_cached_tokens == 0
        assert run("f1", FT_ADAPTER_NAME, [8]).num_cached_tokens == 0  # never shared
        assert eng.coord.completed_cycles >= 1                     # FT rows ran alongside
        ft_reqs = [r for r in eng.finished if r.is_ft]
        assert all(r.num_cached_tokens == 0 for r in ft_reqs)
        assert sched.cache_stats()["hit_pages"] >= 10
        assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks


def test_stop_strings_end_requests():
    class LetterTok:
        def encode(self, text, add_special_tokens=False):
            return [ord(c) % 1024 for c in text]

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr(65 + int(i) % 26) for i in ids)

    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp, start_on_launch=False)
        eng.tokenizer = LetterTok()
        eng.add_request("full", [5, 6, 7, 8], SamplingParams(max_tokens=10))
        eng.run_until_idle(max_steps=200)
        full = eng.finished[-1]
        text = eng.tokenizer.decode(full.output_ids)
        stop = text[3:5]
        eng.add_request("cut", [5, 6, 7, 8], SamplingParams(max_tokens=10, stop=(stop,)))
        eng.run_until_idle(max_steps=200)
        cut = eng.finished[-1]
        assert cut.stop_reason == stop
        k = text.find(stop)
        assert cut.output_ids == full.output_ids[:k + len(stop)]   # ended on the token completing the match
        assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks


def test_eos_ends_requests_unless_ignored(tmp_path):
    """A request stops on the tokenizer's end-of-sequence id (or one listed in
    the model directory's generation_config.json) unless ignore_eos is set."""
    import json as _json
    from deltaserve_vllm_b200.engine.llm_engine import _generation_eos_ids

    class Tok:
        eos_token_id = None

    eng = make_engine(str(tmp_path), start_on_launch=False)
    eng.tokenizer = Tok()
    eng.add_request("full", [5, 6, 7, 8], SamplingParams(max_tokens=8, ignore_eos=True))
    eng.run_until_idle(max_steps=200)
    full = eng.finished[-1].output_ids
    assert len(full) == 8
    k = 3
    eos = full[k]
    first = full.index(eos)
    tok2 = Tok()
    tok2.eos_token_id = eos
    eng.tokenizer = tok2
    eng.add_request("eos", [5, 6, 7, 8], SamplingParams(max_tokens=8, ignore_eos=False))
    eng.add_request("ign", [5, 6, 7, 8], SamplingParams(max_tokens=8, ignore_eos=True))
    eng.run_until_idle(max_steps=200)
    got = {r.request_id: r.output_ids for r in eng.finished[-2:]}
    assert got["eos"] == full[:first + 1]                  # the EOS token is the last output
    assert got["ign"] == full
    assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks
    # generation_config.json: an int or a list
    d = tmp_path / "m"
    d.mkdir()
    (d / "generation_config.json").write_text(_json.dumps({"eos_token_id": [128001, 128009]}))
    assert _generation_eos_ids(str(d)) == (128001, 128009)
    (d / "generation_config.json").write_text(_json.dumps({"eos_token_id": 7}))
    assert _generation_eos_ids(str(d)) == (7,)
    assert _generation_eos_ids("qwen3-tiny") == ()
