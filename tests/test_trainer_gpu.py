"""The LoRA backward on the GPU (tcgen05 GEMMs, bf16 operands) == the fp32 CPU
oracle run of the same trainer, within bf16 tolerance, on head_dim-128 models."""
import pytest
import torch

from deltaserve_vllm_b200 import ops
from deltaserve_vllm_b200.engine.kv_cache import KVCache
from deltaserve_vllm_b200.engine.model_runner import ModelRunner
from deltaserve_vllm_b200.engine.request import Request, SamplingParams
from deltaserve_vllm_b200.engine.scheduler import Scheduler, SchedulerOutput
from deltaserve_vllm_b200.engine.trainer import LoraTrainer
from deltaserve_vllm_b200.models.configs import PRESETS
from deltaserve_vllm_b200.models.decoder import CaptureBuffers, DecoderModel
from deltaserve_vllm_b200.models.lora import LoraServeBuffers, random_adapter
from deltaserve_vllm_b200.models.weights import init_weights

pytestmark = pytest.mark.gpu


def run(arch, seqs, ad, device, dtype, steps=1, lr=0.0, tp=None, comm=None, fused_tp=False):
    """Forward the FT rows through the serving model (capturing activations)
    and run ``steps`` backward cycles. ``fused_tp``: the residual-gradient
    reductions and the replicated factors' optimizer over peer memory (the
    caller closes ``tr.bwd.tpws`` and ``tr.optws``)."""
    from deltaserve_vllm_b200.models.weights import TPInfo
    tp = tp or TPInfo()
    w = init_weights(arch, tp=tp, seed=5, device="cpu", dtype=torch.float32).to(device, dtype)
    kv = KVCache(arch.num_layers, 64, arch.num_kv_heads // tp.size, 64, 128, device, dtype)
    served = LoraServeBuffers(arch, w.tp, slots=2, max_rank=16, device=device, dtype=dtype)
    model = DecoderModel(w, kv.k, kv.v, served, comm)
    n = sum(len(s) for s in seqs)
    cap = CaptureBuffers.allocate(w, n + 8, device, dtype)
    tr = LoraTrainer(w, served, 1, 16, 32, lr=lr, mask_prefix=16, cos_sin_table=model.cos_sin, comm=comm)
    tr.load_adapter(ad, 16, 32)
    tr.publish()
    if fused_tp:
        from deltaserve_vllm_b200.parallel.peer import BwdPeerWorkspace, OptPeerWorkspace
        tr.bwd.tpws = BwdPeerWorkspace(comm, n + 8, arch.hidden)
        tr.optws = OptPeerWorkspace(comm, tr.masters.rep_total, arch.num_layers)
    runner = ModelRunner(model, 64, device, ft_slot=1)
    sched = Scheduler(kv.allocator, 64, max_num_batched_tokens=8192, max_model_len=4096)
    res = []
    for _ in range(steps):
        out = SchedulerOutput()
        reqs = [Request(f"f{i}", s, SamplingParams(max_tokens=1), is_ft=True) for i, s in enumerate(seqs)]
        assert not sched.add_ft(out, reqs)
        runner.execute(out, cap, 0)
        sched.update(out, {})
        starts = [sum(len(x) for x in seqs[:i]) for i in range(len(seqs))]
        res.append(tr.run_cycle(cap, n, starts, [len(s) for s in seqs]))
    return tr, res


def cos(a, b):
    a, b = a.flatten().double(), b.flatten().double()
    return float((a @ b) / (a.norm() * b.norm() + 1e-30))


@pytest.mark.parametrize("name", ["qwen3-test", "llama3-test"])
def test_gpu_backward_matches_cpu_oracle(name):
    arch = PRESETS[name]
    g = torch.Generator().manual_seed(1)
    seqs = [torch.randint(0, arch.vocab, (n,), generator=g).tolist() for n in (64, 200, 33, 130)]
    ad = random_adapter(arch, 16, seed=3, b_std=0.02)
    gt, gres = run(arch, seqs, ad, "cuda", torch.bfloat16)
    ct, cres = run(arch, seqs, ad, "cpu", torch.float32)
    assert ops.check_device_error() == 0
    assert abs(gres[0].loss - cres[0].loss) < 0.02 * abs(cres[0].loss)
    gg = gt.masters.export_peft(16, grads=True)
    cg = ct.masters.export_peft(16, grads=True)
    # Elementwise per tensor (bf16 operands against the fp32 oracle; measured
    # worst: 2.6 % relative L2, 3.5 % of the tensor's max): a wrong scale on a
    # projection's slice or a missing row block moves either far more.
    for k in cg:
        x, y = gg[k].double(), cg[k].double()
        rel_l2 = float((x - y).norm() / (y.norm() + 1e-30))
        rel_max = float((x - y).abs().max() / (y.abs().max() + 1e-30))
        assert rel_l2 < 0.05 and rel_max < 0.08, (k, rel_l2, rel_max)


def test_gpu_training_reduces_loss():
    arch = PRESETS["llama3-test"]
    g = torch.Generator().manual_seed(2)
    seqs = [torch.randint(0, arch.vocab, (96,), generator=g).tolist() for _ in range(4)]
    ad = random_adapter(arch, 16, seed=3, b_std=0.0)
    tr, res = run(arch, seqs, ad, "cuda", torch.bfloat16, steps=10, lr=2e-3)
    assert res[-1].loss < res[0].loss - 0.05, [r.loss for r in res]


def test_graph_replay_after_a_shape_change_matches_eager():
    """Cycles of two batch shapes alternate (A, B, A, B, A): shape A's graphs
    are captured on its second cycle and replayed on the third, after shape B
    ran in between; with lr = 0 the replayed cycle's gradients equal an eager
    cycle's (the cycle scratch is shared by every shape's graphs, so a replay
    never touches memory freed by another shape)."""
    arch = PRESETS["qwen3-test"]
    g = torch.Generator().manual_seed(9)
    shapes = {"A": [torch.randint(0, arch.vocab, (n,), generator=g).tolist() for n in (130, 64, 200)],
              "B": [torch.randint(0, arch.vocab, (n,), generator=g).tolist() for n in (300, 33)]}
    ad = random_adapter(arch, 16, seed=4, b_std=0.02)
    dev, dt = "cuda", torch.bfloat16
    w = init_weights(arch, seed=5, device="cpu", dtype=torch.float32).to(dev, dt)
    kv = KVCache(arch.num_layers, 64, arch.num_kv_heads, 64, 128, dev, dt)
    served = LoraServeBuffers(arch, w.tp, slots=2, max_rank=16, device=dev, dtype=dt)
    model = DecoderModel(w, kv.k, kv.v, served, None)
    cap = CaptureBuffers.allocate(w, 512, dev, dt)
    runner = ModelRunner(model, 64, dev, ft_slot=1)
    sched = Scheduler(kv.allocator, 64, max_num_batched_tokens=8192, max_model_len=4096)

    def trainer():
        tr = LoraTrainer(w, served, 1, 16, 32, lr=0.0, mask_prefix=0, cos_sin_table=model.cos_sin)
        tr.load_adapter(ad, 16, 32)
        tr.publish()
        return tr

    def cycle(tr, name):
        seqs = shapes[name]
        out = SchedulerOutput()
        reqs = [Request(f"{name}{i}", s, SamplingParams(max_tokens=1), is_ft=True) for i, s in enumerate(seqs)]
        assert not sched.add_ft(out, reqs)
        runner.execute(out, cap, 0)
        sched.update(out, {})
        lens = [len(s) for s in seqs]
        starts = [sum(lens[:i]) for i in range(len(lens))]
        return tr.run_cycle(cap, sum(lens), starts, lens)

    tr = trainer()
    for name in ("A", "B", "A", "B", "A"):
        res = cycle(tr, name)
    assert len(tr._graphs) == 2
    graphed = tr.masters.export_peft(16, grads=True)
    eager_tr = trainer()
    eager_tr.use_graphs = False
    res_e = cycle(eager_tr, "A")
    eager = eager_tr.masters.export_peft(16, grads=True)
    assert ops.check_device_error() == 0
    assert abs(res.loss - res_e.loss) < 1e-4 * abs(res_e.loss)
    for k, y in eager.items():
        torch.testing.assert_close(graphed[k], y, rtol=1e-3, atol=1e-6)
