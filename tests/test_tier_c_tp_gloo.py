"""Tier-C pre-emption under tensor parallelism, on two CPU ranks (gloo).

Each rank observes "a request arrived" at a different point: in the first
pre-emptible FT-only forward only rank 0 sees it (before layer 1); in the
second only rank 1 does (before layer 0). The per-layer MAX vote must make
both ranks abandon the same forward at the same layer, both times, and the
ranks must then keep issuing the same collectives (training finishes; a
mismatch would fail the gloo collectives at the process-group timeout). This
is the reference's asymmetric-arrival check (``tests/test_ft_abort_tp.py``)."""

import os
import tempfile
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_engine_tp_gloo import _port


def _worker(rank, world, port, outdir):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
    from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
    from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
    from deltaserve_vllm_b200.parallel.comm import TPComm
    comm = TPComm()
    ecfg = EngineConfig(model="qwen3-tiny", device="cpu", tensor_parallel_size=world, max_model_len=512,
                        block_size=16, max_num_batched_tokens=256, max_loras=2, max_lora_rank=8)
    fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=96, learning_rate=1e-3,
                          forward_interruptible=True, ft_only_admission_grace_ms=0)
    store = FinetuningStore.synthetic(1024, 10, 16, 40, seed=0, max_saved_finetuning_tokens=96)
    eng = CoServingEngine(ecfg, fcfg, comm=comm, ft_store=store)
    orig = eng.runner.abort_hook
    seen = {"hooks": 0, "aborted": []}
    # (hook index, layer) at which THIS rank alone observes an arrival
    mine = {0: (1, 1), 1: (2, 0)}[rank]

    def patched(should_abort, vote=None, ahead=2):
        seen["hooks"] += 1
        idx = seen["hooks"]
        checks = {"n": 0}

        def sa():
            l = checks["n"]
            checks["n"] += 1
            return (idx, l) == mine or should_abort()
        inner = orig(sa, vote, ahead)

        def hook(l):
            r = inner(l)
            if r:
                seen["aborted"].append((idx, l))
            return r
        return hook
    eng.runner.abort_hook = patched
    try:
        if rank != 0:
            eng.follow()
        else:
            eng.run_until_idle(max_steps=3000)
            eng.shutdown()
        res = {"aborted": seen["aborted"], "hooks": seen["hooks"]}
        if rank == 0:
            res.update(cycles=eng.coord.completed_cycles, aborts=eng.stats.get("ft_aborts", 0),
                       finished=eng.store.finished(), free=eng.kv.allocator.num_free,
                       blocks=eng.kv.allocator.num_blocks, losses=list(eng.trainer.losses))
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_tier_c_asymmetric_arrival_tp2_gloo():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _port(), d), nprocs=2, join=True, start_method="spawn")
        r0, r1 = torch.load(os.path.join(d, "r0.pt")), torch.load(os.path.join(d, "r1.pt"))
        assert r0["aborted"] == [(1, 1), (2, 0)], r0["aborted"]
        assert r1["aborted"] == r0["aborted"]
        assert r0["hooks"] == r1["hooks"] >= 3
        assert r0["aborts"] == 2
        assert r0["cycles"] >= 2 and r0["finished"]
        assert r0["free"] == r0["blocks"]
        assert all(l == l for l in r0["losses"])
