"""Inference-correctness gate: finetuning rows must not leak into inference.

The trained adapter is amplified 10x (so any leak through shared GEMM tiles,
LoRA slot masks, KV pages or captured activations would move the other rows'
logits by far more than rounding), inference requests arrive staggered so they
are co-batched with FT rows and with backward cycles, and their greedy
outputs must equal a run of the same engine with finetuning off. A request
served with the FT adapter is the positive control: it must differ from the
base model (the reference's gates ``tests/test_phase1_m1.py`` and
``tests/test_tp_inference_leak.py``)."""

import torch

from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
from deltaserve_vllm_b200.engine.llm_engine import FT_ADAPTER_NAME, CoServingEngine
from deltaserve_vllm_b200.engine.request import SamplingParams
from deltaserve_vllm_b200.models.configs import PRESETS
from deltaserve_vllm_b200.models.lora import random_adapter


def _run(with_ft: bool):
    arch = PRESETS["qwen3-tiny"]
    ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=512, block_size=16,
                        max_num_batched_tokens=192, max_loras=3, max_lora_rank=8)
    ad = random_adapter(arch, 8, seed=21, b_std=0.05)
    ad = {k: v * 10.0 if ".lora_B." in k else v for k, v in ad.items()}   # amplified FT adapter
    if with_ft:
        fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=96, learning_rate=1e-3)
        store = FinetuningStore.synthetic(1024, 24, 16, 48, seed=1, max_saved_finetuning_tokens=96,
                                          total_epochs=2)
        eng = CoServingEngine(ecfg, fcfg, ft_store=store, ft_adapter=(ad, 8, 16.0))
    else:
        eng = CoServingEngine(ecfg, FinetuneConfig(enable_finetuning=False))
    eng.load_inference_adapter("toy", rank=8, alpha=16, seed=7)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 1024, (12 + 9 * i,), generator=g).tolist() for i in range(9)]
    for wave in range(3):                    # staggered arrivals: co-batched with FT rows
        for i in range(3):
            j = 3 * wave + i
            eng.add_request(f"r{j}", prompts[j], SamplingParams(max_tokens=8),
                            adapter="toy" if j % 3 == 1 else None)
        for _ in range(4):
            eng.step()
    ctrl = None
    if with_ft:
        eng.add_request("ctrl", prompts[0], SamplingParams(max_tokens=8), adapter=FT_ADAPTER_NAME)
    eng.run_until_idle(max_steps=3000)
    outs = {r.request_id: list(r.output_ids) for r in eng.finished}
    if with_ft:
        ctrl = outs.pop("ctrl")
        assert eng.coord.completed_cycles >= 1 and eng.stats["ft_tokens_forwarded"] > 0
    return outs, ctrl


def test_ft_rows_do_not_leak_into_inference():
    base, _ = _run(False)
    co, ctrl = _run(True)
    assert set(base) == set(co) and len(base) == 9
    for rid in base:
        assert co[rid] == base[rid], rid
    assert ctrl != base["r0"]          # positive control: the amplified adapter matters
