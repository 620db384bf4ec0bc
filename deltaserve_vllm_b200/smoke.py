"""One tiny co-serving run on cuda:0 (used by ``__graft_entry__.smoke``): a
2-layer model with Llama-3-8B layer geometry serves LoRA requests (prefill +
decode) while one finetuning cycle (capture -> hand-written LoRA backward ->
AdamW -> publish) runs, all through the sm_100a kernels."""

from __future__ import annotations

import torch


def run_smoke() -> None:
    from . import ops
    from .config import EngineConfig, FinetuneConfig
    from .engine.ft.store import FinetuningStore
    from .engine.llm_engine import CoServingEngine
    from .engine.request import SamplingParams

    assert torch.cuda.is_available(), "smoke needs a GPU"
    assert ops.native_available(), f"extension not loaded: {ops._C_ERR!r}"
    ecfg = EngineConfig(model="llama3-8b-2l", max_model_len=2048, block_size=64,
                        max_num_batched_tokens=2048, max_loras=2, max_lora_rank=16,
                        num_gpu_blocks_override=128)
    fcfg = FinetuneConfig(enable_finetuning=True, backward_cuda_graph=True, max_saved_finetuning_tokens=512, learning_rate=1e-4)
    store = FinetuningStore.synthetic(8192, 2, 256, 256, seed=0, max_saved_finetuning_tokens=512)
    eng = CoServingEngine(ecfg, fcfg, ft_store=store)
    eng.load_inference_adapter("inf", rank=16, alpha=32)
    for i, n in enumerate((300, 17)):
        eng.add_request(f"smoke-{i}", list(range(1, n + 1)), SamplingParams(max_tokens=3),
                        adapter="inf" if i == 0 else None)
    eng.run_until_idle(max_steps=200)
    eng.synchronize()
    err = ops.check_device_error()
    assert err == 0, f"device error {err}"
    assert eng.coord.completed_cycles >= 1, eng.finetuning_status()
    loss = eng.trainer.losses[-1]
    assert loss == loss and loss > 0, loss
    print(f"smoke ok: {eng.stats['steps']} steps, {eng.coord.completed_cycles} backward cycle(s), "
          f"loss {loss:.4f}, outputs {[r.output_ids for r in eng.finished]}")
