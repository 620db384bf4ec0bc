"""CPU/gloo TP=2 plumbing check of the tiny Qwen3-style decoder. Two ranks run the sharded
serving forward (with its all-reduces) + the hand-written backward (per-layer
residual all-reduces, bucketed replicated-factor all-reduce, rank-symmetric
clip). The TP-merged gradients and loss equal torch autograd on the unsharded
model to 1e-5, and the PEFT save merged across both ranks round-trips."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from deltaserve_vllm_b200.adapters import peft_io
from deltaserve_vllm_b200.models.configs import PRESETS
from deltaserve_vllm_b200.models.lora import random_adapter
from deltaserve_vllm_b200.models.weights import TPInfo
from deltaserve_vllm_b200.parallel.comm import TPComm


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, name, outdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from lora_harness import config1_data, manual_backward
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        arch = PRESETS[name]
        comm = TPComm()
        seqs = config1_data(arch)
        ad = random_adapter(arch, 8, seed=7, b_std=0.01)
        trainer, res = manual_backward(arch, seqs, ad, 8, 16, tp=TPInfo(rank, world), comm=comm,
                                       lr=0.0)
        grads = trainer.masters.export_peft(8, grads=True)
        shards = comm.gather_objects(grads)
        path = os.path.join(outdir, "ckpt")
        trainer.save_adapter(path, save_id="s1")
        if rank == 0:
            torch.save({"loss": res[0].loss, "grads": peft_io.merge_tp_shards(shards),
                        "collectives": comm.num_collectives}, os.path.join(outdir, "r0.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,world", [("qwen3-tiny", 2), ("llama3-tiny", 2), ("llama3-tiny-kv4", 4)])
def test_tp_gloo_matches_autograd_and_peft_roundtrip(name, world):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from lora_harness import autograd_reference, config1_data
    arch = PRESETS[name]
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _port(), name, d), nprocs=world, join=True,
                           start_method="spawn")
        r0 = torch.load(os.path.join(d, "r0.pt"))
        ad = random_adapter(arch, 8, seed=7, b_std=0.01)
        ref_loss, ref_grads = autograd_reference(arch, config1_data(arch), ad, 8, 16)
        assert abs(r0["loss"] - ref_loss) <= 1e-5 * max(1.0, abs(ref_loss))
        scale = max(g.abs().max().item() for g in ref_grads.values())
        for k, g in ref_grads.items():
            torch.testing.assert_close(r0["grads"][k], g, rtol=1e-5, atol=1e-5 * scale, msg=k)
        # lr=0: the saved, merged adapter is the adapter we started from.
        saved, cfg = peft_io.read_adapter(os.path.join(d, "ckpt"))
        assert set(saved) == set(ad)
        for k, t in ad.items():
            torch.testing.assert_close(saved[k], t, rtol=0, atol=0, msg=k)
        assert cfg["r"] == 8 and cfg["lora_alpha"] == 16
        assert peft_io.read_save_result(os.path.join(d, "ckpt"), "s1") is not None
