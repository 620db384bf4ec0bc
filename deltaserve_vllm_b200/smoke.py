"""One tiny co-serving step on cuda:0 (used by ``__graft_entry__.smoke``):
a 2-layer model with Llama-3-8B layer geometry serves two LoRA requests
(prefill + decode) through the sm_100a kernels."""

from __future__ import annotations

import torch


def run_smoke() -> None:
    from . import ops
    from .engine.kv_cache import KVCache
    from .engine.model_runner import ModelRunner
    from .engine.request import Request, SamplingParams
    from .engine.scheduler import Scheduler
    from .models.configs import PRESETS
    from .models.decoder import DecoderModel
    from .models.lora import LoraServeBuffers, random_adapter
    from .models.weights import init_weights

    assert torch.cuda.is_available(), "smoke needs a GPU"
    assert ops.native_available(), f"extension not loaded: {ops._C_ERR!r}"
    arch = PRESETS["llama3-8b-2l"]
    dev = "cuda:0"
    w = init_weights(arch, seed=0, device=dev)
    kv = KVCache(arch.num_layers, 64, arch.num_kv_heads, 64, 128, dev)
    lora = LoraServeBuffers(arch, w.tp, slots=2, max_rank=16, device=dev)
    lora.load_slot(0, random_adapter(arch, 16, seed=1), 16, 32)
    model = DecoderModel(w, kv.k, kv.v, lora)
    sched = Scheduler(kv.allocator, 64, max_num_batched_tokens=1024, max_model_len=2048)
    runner = ModelRunner(model, 64, dev)
    for i, n in enumerate((300, 17)):
        r = Request(f"smoke-{i}", list(range(1, n + 1)), SamplingParams(max_tokens=3))
        r.lora_slot = 0 if i == 0 else -1
        sched.add(r)
    steps = 0
    while sched.has_unfinished() and steps < 16:
        out = sched.schedule()
        toks, logits = runner.execute(out)
        assert logits is None or torch.isfinite(logits).all()
        sched.update(out, toks)
        steps += 1
    torch.cuda.synchronize()
    err = ops.check_device_error()
    assert err == 0, f"device error {err}"
    assert not sched.has_unfinished()
    print(f"smoke ok: {steps} steps, outputs "
          f"{[r.output_ids for r in sched.finished]}")
