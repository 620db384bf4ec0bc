"""Shared helpers for the LoRA-backward tests: run the serving forward with
activation capture over FT samples, then the trainer's manual backward; and the
autograd reference over the independent dense forward."""
import torch
import torch.nn.functional as F

from deltaserve_vllm_b200.engine.kv_cache import KVCache
from deltaserve_vllm_b200.engine.model_runner import ModelRunner
from deltaserve_vllm_b200.engine.request import Request, SamplingParams
from deltaserve_vllm_b200.engine.scheduler import Scheduler, SchedulerOutput
from deltaserve_vllm_b200.engine.trainer import LoraTrainer
from deltaserve_vllm_b200.models.decoder import CaptureBuffers, DecoderModel
from deltaserve_vllm_b200.models.lora import LoraServeBuffers, peft_key, random_adapter
from deltaserve_vllm_b200.models.lora_backward import make_labels
from deltaserve_vllm_b200.models.weights import full_layer_tensors, init_weights, TPInfo

from dense_ref import dense_forward


def config1_data(arch, n_seq=4, seq_len=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, arch.vocab, (seq_len,), generator=g).tolist() for _ in range(n_seq)]


def manual_backward(arch, seqs, adapter, rank, alpha, tp=None, comm=None, mask_prefix=16,
                    device="cpu", dtype=torch.float32, seed=3, steps=1, lr=1e-3):
    tp = tp or TPInfo()
    w = init_weights(arch, tp=tp, seed=seed, device=device, dtype=dtype)
    kv = KVCache(arch.num_layers, 64, arch.num_kv_heads // tp.size, 16, arch.head_dim, device, dtype)
    served = LoraServeBuffers(arch, tp, slots=1, max_rank=rank, device=device, dtype=dtype)
    served.load_slot(0, adapter, rank, alpha)
    model = DecoderModel(w, kv.k, kv.v, served, comm)
    n = sum(len(s) for s in seqs)
    cap = CaptureBuffers.allocate(w, n + 8, device, dtype)
    trainer = LoraTrainer(w, served, 0, rank, alpha, lr=lr, comm=comm, mask_prefix=mask_prefix,
                          cos_sin_table=model.cos_sin)
    trainer.load_adapter(adapter, rank, alpha)
    runner = ModelRunner(model, 16, device, ft_slot=0)
    sched = Scheduler(kv.allocator, 16, max_num_batched_tokens=4096, max_model_len=1024)
    results = []
    for _ in range(steps):
        out = SchedulerOutput()
        reqs = [Request(f"ft{i}", s, SamplingParams(max_tokens=1), is_ft=True) for i, s in enumerate(seqs)]
        assert not sched.add_ft(out, reqs)
        runner.execute(out, cap, ft_dst=0)
        sched.update(out, {})
        starts, lens, st = [], [], 0
        for s in seqs:
            starts.append(st)
            lens.append(len(s))
            st += len(s)
        results.append(trainer.run_cycle(cap, n, starts, lens))
    return trainer, results


def autograd_reference(arch, seqs, adapter, rank, alpha, mask_prefix=16, seed=3):
    w = init_weights(arch, seed=seed, dtype=torch.float32)
    full = [full_layer_tensors(arch, i, seed, "cpu", torch.float32) for i in range(arch.num_layers)]
    params = {k: v.clone().float().requires_grad_(True) for k, v in adapter.items()}
    total, n_valid = 0.0, 0
    for s in seqs:
        ids = torch.tensor(s)
        logits = dense_forward(arch, full, w.embed, w.lm_head_full, w.final_norm, ids,
                               lora=params, scaling=alpha / rank)
        lab = make_labels(ids, [0], [len(s)], len(s), mask_prefix)
        ok = lab >= 0
        total = total + F.cross_entropy(logits[ok], lab[ok], reduction="sum")
        n_valid += int(ok.sum())
    loss = total / n_valid
    loss.backward()
    return float(loss.detach()), {k: p.grad for k, p in params.items()}
