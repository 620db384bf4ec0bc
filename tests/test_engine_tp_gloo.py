"""The rank-0-driven step protocol under tensor parallelism, on CPU ranks
(gloo): rank 0 schedules, admits finetuning, triggers and advances backward
cycles and broadcasts each step's plan; rank 1 replays it. Both ranks must
issue the same collectives in the same order (a mismatch hangs or fails the
gloo collectives, bounded by the process-group timeout)."""
import os
import socket
import tempfile
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir, model="qwen3-tiny"):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
    from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
    from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
    from deltaserve_vllm_b200.engine.request import SamplingParams
    from deltaserve_vllm_b200.parallel.comm import TPComm
    comm = TPComm()
    ecfg = EngineConfig(model=model, device="cpu", tensor_parallel_size=world, max_model_len=512,
                        block_size=16, max_num_batched_tokens=256, max_loras=2, max_lora_rank=8)
    fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=96, learning_rate=1e-3)
    store = FinetuningStore.synthetic(1024, 10, 16, 40, seed=0, max_saved_finetuning_tokens=96)
    eng = CoServingEngine(ecfg, fcfg, comm=comm, ft_store=store)
    try:
        if rank != 0:
            eng.follow()
            return
        eng.load_inference_adapter("inf", rank=8, alpha=16)     # replayed on rank 1
        eng.profile_execution_model(repeats=1, max_shapes=6)
        g = torch.Generator().manual_seed(0)
        for i in range(5):
            eng.add_request(f"r{i}", torch.randint(0, 1024, (20 + 9 * i,), generator=g).tolist(),
                            SamplingParams(max_tokens=4), adapter="inf" if i % 2 else None)
        eng.run_until_idle(max_steps=3000)
        eng.mark("a")
        eng.mark("b")
        regions = eng.gather_region("a", "b")
        # TP-merged PEFT save (both ranks join the gather), then serve the
        # saved adapter from disk in a freshly loaded slot on both ranks.
        ck = eng.save_adapter(os.path.join(outdir, "ck"), save_id="s1")
        eng.unload_inference_adapter("inf")
        eng.load_inference_adapter("trained", path=ck)
        eng.add_request("t0", list(range(5, 40)), SamplingParams(max_tokens=3), adapter="trained")
        eng.run_until_idle(max_steps=200, finetune=False)
        eng.shutdown()
        torch.save({"cycles": eng.coord.completed_cycles, "losses": eng.trainer.losses,
                    "outs": sorted(len(r.output_ids) for r in eng.finished if r.request_id.startswith("r")),
                    "t0": [len(r.output_ids) for r in eng.finished if r.request_id == "t0"],
                    "ck": ck, "regions": regions}, os.path.join(outdir, "res.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("model,world", [("qwen3-tiny", 2), ("llama3-tiny-kv4", 4)])
def test_tp_engine_protocol_gloo(model, world):
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _port(), d, model), nprocs=world, join=True, start_method="spawn")
        r = torch.load(os.path.join(d, "res.pt"))
        assert r["cycles"] >= 2
        assert all(l == l for l in r["losses"])
        assert r["outs"] == [4] * 5
        assert len(r["regions"]) == world
        assert r["t0"] == [3]
        from deltaserve_vllm_b200.adapters import peft_io
        tensors, cfg = peft_io.read_adapter(r["ck"])
        from deltaserve_vllm_b200.models.configs import resolve_arch
        arch = resolve_arch(model)
        assert len(tensors) == 2 * 7 * arch.num_layers
        q_b = [v for k, v in tensors.items() if "q_proj.lora_B" in k][0]
        assert q_b.shape[0] == arch.num_heads * arch.head_dim      # merged across ranks
