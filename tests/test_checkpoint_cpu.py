"""Adapter checkpoints on CPU: periodic, epoch and manual saves, pruning,
the save handshake (state / error files), and resume from a saved adapter.

The periodic save taken after the last backward and a manual save taken at
the same point must be bit-identical to each other and to the trainer's fp32
masters (the reference's ``tests/test_adapter_save.py``: "periodic / epoch /
manual saves bit-exact", "error files")."""

import json
import os
import tempfile

import torch

from deltaserve_vllm_b200.adapters import peft_io
from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
from deltaserve_vllm_b200.engine.llm_engine import FT_ADAPTER_NAME, CoServingEngine
from deltaserve_vllm_b200.engine.request import SamplingParams


def _engine(tmp, store_epochs=2, **ft):
    ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=512, block_size=16,
                        max_num_batched_tokens=256, max_loras=3, max_lora_rank=8)
    fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=96, learning_rate=1e-3,
                          adapter_save_path=os.path.join(tmp, "ckpt"), **ft)
    store = FinetuningStore.synthetic(1024, 12, 16, 40, seed=0, max_saved_finetuning_tokens=96,
                                      total_epochs=store_epochs)
    return CoServingEngine(ecfg, fcfg, ft_store=store)


def _dirs(root, prefix):
    return sorted(d for d in os.listdir(root) if d.startswith(prefix))


def _same(a, b):
    assert set(a) == set(b)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_periodic_epoch_and_manual_saves_bit_exact():
    with tempfile.TemporaryDirectory() as tmp:
        eng = _engine(tmp, adapter_save_every_backwards=1, adapter_save_keep_last=2,
                      adapter_save_every_epoch=True)
        eng.run_until_idle(max_steps=4000)
        eng.trainer.wait_saves()
        root = os.path.join(tmp, "ckpt")
        steps = eng.trainer.step
        assert steps >= 3
        back = _dirs(root, "backward-")
        assert back == [f"backward-{s:06d}" for s in (steps - 1, steps)]   # keep-last-2 pruning
        epochs = _dirs(root, "epoch-")
        assert 1 <= len(epochs) <= 2
        for d in back + epochs:
            files = set(os.listdir(os.path.join(root, d)))
            assert {peft_io.WEIGHTS_FILE, peft_io.CONFIG_FILE, peft_io.STATE_FILE} <= files
            assert not any(f.endswith(".tmp") for f in files)
        with open(os.path.join(root, back[-1], peft_io.STATE_FILE)) as f:
            state = json.load(f)
        assert state["step"] == steps and state["last_loss"] == eng.trainer.losses[-1]

        periodic, cfg = peft_io.read_adapter(os.path.join(root, back[-1]))
        masters = eng.trainer.export_full()
        _same(periodic, masters)
        manual = eng.save_adapter(os.path.join(tmp, "manual"), save_id="m1")
        got, cfg2 = peft_io.read_adapter(manual)
        _same(got, periodic)
        assert cfg2 == cfg and cfg["peft_type"] == "LORA" and cfg["r"] == eng.trainer.rank_r
        assert peft_io.read_save_result(manual, "m1")["step"] == steps
        assert peft_io.read_save_result(manual, "other-id") is None
        # the last epoch snapshot was taken after the final backward too
        last_epoch, _ = peft_io.read_adapter(os.path.join(root, epochs[-1]))
        _same(last_epoch, masters)
        # B is stored unscaled, A/B as fp32 in PEFT orientation
        k = next(k for k in got if k.endswith("q_proj.lora_B.weight"))
        assert got[k].dtype == torch.float32 and got[k].shape[1] == eng.trainer.rank_r


def test_background_save_handshake_and_error_file(monkeypatch):
    with tempfile.TemporaryDirectory() as tmp:
        eng = _engine(tmp, store_epochs=1)
        eng.run_until_idle(max_steps=2000)
        path = os.path.join(tmp, "bg")
        assert eng.save_adapter(path, save_id="b1", background=True) == path
        res = peft_io.wait_save_result(path, "b1", timeout_s=30)
        assert res is not None and "error" not in res and res["save_id"] == "b1"

        def boom(*a, **k):
            raise OSError("disk full")
        monkeypatch.setattr(peft_io, "write_peft_adapter", boom)
        bad = os.path.join(tmp, "bad")
        eng.save_adapter(bad, save_id="b2", background=True)
        eng.trainer.wait_saves()
        res = peft_io.read_save_result(bad, "b2")
        assert res is not None and "disk full" in res["error"]
        monkeypatch.undo()
        # a later good save into the same directory clears the error file
        eng.save_adapter(bad, save_id="b3")
        assert not os.path.exists(os.path.join(bad, peft_io.ERROR_FILE))
        assert peft_io.read_save_result(bad, "b3")["save_id"] == "b3"


def test_resume_from_saved_adapter():
    """``finetuning_lora_path`` pointing at a saved checkpoint restores the
    masters exactly (the optimizer starts fresh), and the served slot holds
    the same adapter: greedy outputs of the resumed engine equal the
    original's."""
    with tempfile.TemporaryDirectory() as tmp:
        eng = _engine(tmp, store_epochs=1)
        eng.run_until_idle(max_steps=2000)
        path = eng.save_adapter(os.path.join(tmp, "saved"), save_id="s")
        masters = eng.trainer.export_full()
        prompt = list(range(3, 40))
        eng.add_request("a", prompt, SamplingParams(max_tokens=6), adapter=FT_ADAPTER_NAME)
        eng.run_until_idle(max_steps=200)
        ref_out = eng.finished[-1].output_ids

        eng2 = _engine(tmp, store_epochs=1, finetuning_lora_path=path, start_on_launch=False)
        assert eng2.trainer.step == 0
        _same(eng2.trainer.export_full(), masters)
        eng2.add_request("a", prompt, SamplingParams(max_tokens=6), adapter=FT_ADAPTER_NAME)
        eng2.run_until_idle(max_steps=200)
        assert eng2.finished[-1].output_ids == ref_out
