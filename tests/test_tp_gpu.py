"""Tensor parallelism on real GPUs (NCCL over NVLink): TP=2 serving forward
logits and LoRA-backward gradients equal the TP=1 run on the same model.
Needs 2 GPUs (skipped otherwise)."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(rank, world, port, outdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    torch.cuda.set_device(rank)
    if world > 1:
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, device_id=torch.device("cuda", rank))
    from deltaserve_vllm_b200.models.configs import PRESETS
    from deltaserve_vllm_b200.models.lora import random_adapter
    from deltaserve_vllm_b200.models.weights import TPInfo
    from deltaserve_vllm_b200.parallel.comm import TPComm
    from test_trainer_gpu import run as run_trainer
    arch = PRESETS["llama3-test"]
    g = torch.Generator().manual_seed(1)
    seqs = [torch.randint(0, arch.vocab, (n,), generator=g).tolist() for n in (64, 200, 33, 130)]
    ad = random_adapter(arch, 16, seed=3, b_std=0.02)
    comm = TPComm() if world > 1 else None
    tr, res = run_trainer(arch, seqs, ad, "cuda", torch.bfloat16, tp=TPInfo(rank, world), comm=comm)
    grads = tr.masters.export_peft(16, grads=True)
    if comm is not None:
        shards = comm.gather_objects(grads)
        if rank == 0:
            from deltaserve_vllm_b200.adapters.peft_io import merge_tp_shards
            grads = merge_tp_shards(shards)
    if rank == 0:
        torch.save({"loss": res[0].loss, "grads": grads}, os.path.join(outdir, f"tp{world}.pt"))
    if world > 1:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_backward_matches_tp1_on_gpu():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_run, args=(2, _port(), d), nprocs=2, join=True, start_method="spawn")
        mp.start_processes(_run, args=(1, _port(), d), nprocs=1, join=True, start_method="spawn")
        a, b = torch.load(os.path.join(d, "tp2.pt")), torch.load(os.path.join(d, "tp1.pt"))
        assert abs(a["loss"] - b["loss"]) < 0.01 * abs(b["loss"])
        for k, g in b["grads"].items():
            x, y = a["grads"][k].double(), g.double()
            rel_l2 = float((x - y).norm() / (y.norm() + 1e-30))
            rel_max = float((x - y).abs().max() / (y.abs().max() + 1e-30))
            assert rel_l2 < 0.05 and rel_max < 0.08, (k, rel_l2, rel_max)


def _run_gemm_ar(rank, world, port, outdir):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=torch.device("cuda", rank))
    from deltaserve_vllm_b200 import ops
    from deltaserve_vllm_b200.parallel.comm import TPComm
    from deltaserve_vllm_b200.parallel.peer import PeerWorkspace
    comm = TPComm(None, dist.new_group(backend="gloo"))
    ws = PeerWorkspace(comm, 2048, 4096)
    errs = []
    try:
        for it, (M, K) in enumerate([(1, 2048), (16, 896), (300, 512), (2048, 1024), (5, 7168)]):
            g = torch.Generator(device="cuda").manual_seed(100 * it + rank)
            a = (torch.randn(M, K, generator=g, device="cuda")).bfloat16()
            b = (torch.randn(4096, K, generator=g, device="cuda") * 0.05).bfloat16()
            fused = ops.gemm_ar(a, b, ws).clone()
            ref = (a.float() @ b.float().t())
            dist.all_reduce(ref)
            errs.append(float((fused.float() - ref).abs().max() / (ref.abs().max() + 1e-6)))
        torch.cuda.synchronize()
        err_code = ops.check_device_error()
    finally:
        ws.close()
    torch.save({"errs": errs, "code": err_code}, os.path.join(outdir, f"ar{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_gemm_allreduce_tp2():
    """The fused GEMM + all-reduce over peer memory equals GEMM + NCCL all-reduce."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_run_gemm_ar, args=(2, _port(), d), nprocs=2, join=True, start_method="spawn")
        for r in range(2):
            res = torch.load(os.path.join(d, f"ar{r}.pt"))
            assert res["code"] == 0
            assert max(res["errs"]) < 2e-2, res["errs"]


def _run_fused_vs_nccl(rank, world, port, outdir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=torch.device("cuda", rank))
    from deltaserve_vllm_b200 import ops
    from deltaserve_vllm_b200.adapters.peft_io import merge_tp_shards
    from deltaserve_vllm_b200.models.configs import PRESETS
    from deltaserve_vllm_b200.models.lora import random_adapter
    from deltaserve_vllm_b200.models.weights import TPInfo
    from deltaserve_vllm_b200.parallel.comm import TPComm
    from test_trainer_gpu import run as run_trainer
    arch = PRESETS["llama3-8b-2l"]
    g = torch.Generator().manual_seed(7)
    seqs = [torch.randint(0, arch.vocab, (n,), generator=g).tolist() for n in (512, 200, 333, 130)]
    ad = random_adapter(arch, 16, seed=3, b_std=0.02)
    comm = TPComm(None, dist.new_group(backend="gloo"))
    out = {}
    for mode in ("nccl", "fused"):
        # lr = 0: the gradients are compared. The unreplicated factors' ones
        # (column-parallel B, row-parallel A) are final on every rank on both
        # paths; the replicated ones end up summed only in each slice owner on
        # the fused path (their optimizer has its own test below).
        tr, res = run_trainer(arch, seqs, ad, "cuda", torch.bfloat16, tp=TPInfo(rank, world), comm=comm,
                              fused_tp=mode == "fused")
        shards = comm.gather_objects(tr.masters.export_peft(16, grads=True))
        if rank == 0:
            full = merge_tp_shards(shards)
            out[mode] = {"loss": res[0].loss,
                         "grads": {k: v for k, v in full.items()
                                   if any(f".{p}_proj.lora_B" in k for p in ("q", "k", "v", "gate", "up"))
                                   or any(f".{p}_proj.lora_A" in k for p in ("o", "down"))}}
        if tr.bwd.tpws is not None:
            tr.bwd.tpws.close()
            tr.bwd.tpws = None
        if tr.optws is not None:
            tr.optws.close()
            tr.optws = None
    torch.cuda.synchronize()
    out["code"] = ops.check_device_error()
    if rank == 0:
        torch.save(out, os.path.join(outdir, "fused_vs_nccl.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_tp_backward_matches_nccl(world):
    """The tensor-parallel backward with its residual-gradient reductions
    fused over peer memory (dX GEMM pushes bf16 partial rows to the row
    owner, owner reduce + RMSNorm backward + all-gather) gives the same loss
    and, elementwise, the same LoRA gradients as the NCCL all-reduce path
    on the same ranks (Llama-3-8B layer geometry, 2 layers)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_run_fused_vs_nccl, args=(world, _port(), d), nprocs=world, join=True,
                           start_method="spawn")
        r = torch.load(os.path.join(d, "fused_vs_nccl.pt"))
        assert r["code"] == 0
        a, b = r["fused"], r["nccl"]
        assert abs(a["loss"] - b["loss"]) < 1e-3 * abs(b["loss"])
        assert b["grads"]
        for k, y in b["grads"].items():
            x = a["grads"][k].float()
            y = y.float()
            scale = float(y.abs().max()) + 1e-12
            assert float((x - y).abs().max()) < 3e-2 * scale, (k, float((x - y).abs().max()) / scale)
            assert float((x - y).norm()) < 1e-2 * (float(y.norm()) + 1e-12), k


def _run_fused_optimizer(rank, world, port, outdir):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=torch.device("cuda", rank))
    from deltaserve_vllm_b200 import ops
    from deltaserve_vllm_b200.parallel.comm import TPComm
    from deltaserve_vllm_b200.parallel.peer import OptPeerWorkspace
    comm = TPComm(None, dist.new_group(backend="gloo"))
    L, seg = 5, 3000 + 17                    # layers x elements per layer (odd sizes on purpose)
    T = L * seg
    ws = OptPeerWorkspace(comm, T, L)
    g0 = torch.Generator().manual_seed(0)
    p0 = torch.randn(T, generator=g0)
    m0 = torch.randn(T, generator=g0) * 0.01
    v0 = torch.rand(T, generator=g0) * 0.01
    gr = torch.Generator().manual_seed(100 + rank)
    g_in = (torch.randn(T, generator=gr) * 0.3).cuda()
    g = torch.empty_like(g_in)
    shard_sq = (torch.rand(L, generator=gr) * 2.0).cuda()
    p, m, v = p0.cuda(), m0.cuda(), v0.cuda()
    for step in (1, 2):                     # twice: the counters and buffers reset themselves
        g.copy_(g_in)                       # (the owner's slice of g is overwritten by the sum)
        ops.push_slices(g, 3 * seg, T, ws)
        ops.push_slices(g, 0, 3 * seg, ws)
        total = ops.fused_replicated_adamw(ws, p, g, m, v, seg, shard_sq, max_norm=1.0, lr=1e-2, wd=0.01, step=step)
        ops.fused_replicated_finish(ws, p)
    torch.cuda.synchronize()
    gs = comm.all_gather_object(g_in.cpu())
    sqs = comm.all_gather_object(shard_sq.cpu())
    ps = comm.all_gather_object(p.cpu())
    code = ops.check_device_error()
    ws.close()
    if rank == 0:
        torch.save({"gs": gs, "sqs": sqs, "ps": ps, "total": total.cpu(), "p0": p0, "m0": m0, "v0": v0,
                    "code": code, "L": L, "seg": seg}, os.path.join(outdir, "opt.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_replicated_optimizer(world):
    """The replicated factors' optimizer over peer memory: after two steps
    every rank holds the same parameters, equal to AdamW with per-layer
    clipping applied on the host to the sum of the ranks' gradients (the
    per-layer norms including every rank's shard part)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_run_fused_optimizer, args=(world, _port(), d), nprocs=world, join=True,
                           start_method="spawn")
        r = torch.load(os.path.join(d, "opt.pt"))
        assert r["code"] == 0
        L, seg = r["L"], r["seg"]
        # every step pushes the rank's same gradients (the test does not rerun a backward)
        G = sum(r["gs"])
        sq = (G.view(L, seg) ** 2).sum(1) + sum(r["sqs"])
        coef = torch.clamp(1.0 / (sq.sqrt() + 1e-6), max=1.0).repeat_interleave(seg)
        p, m, v = r["p0"].clone(), r["m0"].clone(), r["v0"].clone()
        for step in (1, 2):
            gi = G * coef
            p = p - 1e-2 * 0.01 * p
            m = 0.9 * m + 0.1 * gi
            v = 0.999 * v + 0.001 * gi * gi
            p = p - 1e-2 * (m / (1 - 0.9 ** step)) / ((v / (1 - 0.999 ** step)).sqrt() + 1e-8)
        torch.testing.assert_close(r["total"], sq, rtol=1e-4, atol=1e-4)
        for got in r["ps"]:
            torch.testing.assert_close(got, p, rtol=1e-4, atol=1e-5)


def _run_embedding_peer(rank, world, port, outdir):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=torch.device("cuda", rank))
    from deltaserve_vllm_b200 import ops
    from deltaserve_vllm_b200.parallel.comm import TPComm
    from deltaserve_vllm_b200.parallel.peer import PeerTable
    comm = TPComm(None, dist.new_group(backend="gloo"))
    V, D = 1000 * world, 256
    vl = V // world
    full = torch.randn(V, D, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).cuda()
    shard = full[rank * vl:(rank + 1) * vl].clone()
    pt = PeerTable(comm, shard, V)
    ids = torch.randint(-2, V + 2, (777,), generator=torch.Generator().manual_seed(6)).cuda()
    got = torch.empty(ids.numel(), D, dtype=torch.bfloat16, device="cuda")
    ops.embedding_peer(ids, pt, got)
    ref = torch.empty_like(got)
    ops.embedding(ids, pt.local, ref, rank * vl)
    dist.all_reduce(ref)
    torch.cuda.synchronize()
    ok = torch.equal(got, ref) and torch.equal(pt.local, shard) and ops.check_device_error() == 0
    oks = comm.all_gather_object(bool(ok))
    pt.close()
    if rank == 0:
        torch.save({"oks": oks}, os.path.join(outdir, "emb.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_embedding_from_peer_shards(world):
    """The vocabulary-parallel embedding read over peer memory equals the
    sharded embedding + NCCL all-reduce of the partial rows on every rank,
    including ids outside the vocabulary (zero rows)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_run_embedding_peer, args=(world, _port(), d), nprocs=world, join=True,
                           start_method="spawn")
        assert all(torch.load(os.path.join(d, "emb.pt"))["oks"])


def _run_gemm_ag(rank, world, port, outdir):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=torch.device("cuda", rank))
    from deltaserve_vllm_b200 import ops
    from deltaserve_vllm_b200.parallel.comm import TPComm
    from deltaserve_vllm_b200.parallel.peer import AGPeerWorkspace
    comm = TPComm(None, dist.new_group(backend="gloo"))
    K, rows = 1024, 256                       # rows per rank (multiple of 128)
    M = rows * world
    ws = AGPeerWorkspace(comm, 384, K)
    g = torch.Generator(device="cuda").manual_seed(10 + rank)
    x = torch.randn(rows, K, generator=g, device="cuda").to(torch.bfloat16)
    ws.local[:rows].copy_(x)
    torch.cuda.synchronize()
    comm.barrier()                            # every shard written before any rank reads it
    gw = torch.Generator(device="cuda").manual_seed(99)
    N = 768
    w = (torch.randn(N, K, generator=gw, device="cuda") * 0.05).to(torch.bfloat16)
    full = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    dist.all_gather_into_tensor(full, x)
    res = {}
    # plain bf16
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.gemm_ag(ws, rows, w, out)
    ref = torch.empty_like(out)
    ops.gemm(full, w, ref)
    res["bf16"] = float((out.float() - ref.float()).abs().max() / ref.float().abs().max())
    remote = torch.ones(M, dtype=torch.bool, device="cuda")
    remote[rank * rows:(rank + 1) * rows] = False
    res["gathered"] = float((ws.gathered[:M][remote].float() - full[remote].float()).abs().max())
    out_d = torch.empty_like(out)
    ops.gemm_ag(ws, rows, w, out_d, copy_once=False)          # every tile read from its owner
    res["bf16_direct"] = float((out_d.float() - ref.float()).abs().max() / ref.float().abs().max())
    # SwiGLU + LoRA expand, with the shrink of the gathered rows (the GEMM
    # reuses the rows the shrink gathered: fresh=False)
    slots, pr, seg = 2, 32, 64
    A = (torch.randn(slots, pr, K, generator=gw, device="cuda") * 0.05).to(torch.bfloat16)
    B2 = (torch.randn(N, slots * seg, generator=gw, device="cuda") * 0.05).to(torch.bfloat16)
    sid = (torch.arange(M, device="cuda", dtype=torch.int32) // 100) % slots
    mask = torch.full(((M + 127) // 128,), 3, dtype=torch.int32, device="cuda")
    Z = torch.empty(M, slots * seg, dtype=torch.bfloat16, device="cuda")
    ops.lora_shrink_ag(ws, rows, A, sid, Z, seg)
    Zr = torch.empty_like(Z)
    ops.lora_shrink(full, A, sid, Zr, seg)
    res["shrink"] = float((Z.float() - Zr.float()).abs().max() / Zr.float().abs().max())
    o2 = torch.empty(M, N // 2, dtype=torch.bfloat16, device="cuda")
    ops.gemm_ag(ws, rows, w, o2, epi=ops.EPI_SWIGLU, z=Z, b2=B2, tile_slots=mask, lora_seg=seg, fresh=False)
    r2 = torch.empty_like(o2)
    ops.gemm(full, w, r2, epi=ops.EPI_SWIGLU, z=Zr, b2=B2, tile_slots=mask, lora_seg=seg)
    res["swiglu_lora"] = float((o2.float() - r2.float()).abs().max() / r2.float().abs().max())
    torch.cuda.synchronize()
    res["code"] = ops.check_device_error()
    allres = comm.all_gather_object(res)
    comm.barrier()
    ws.close()
    if rank == 0:
        torch.save({"res": allres}, os.path.join(outdir, "ag.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gemm_all_gather(world):
    """All-gather -> GEMM with the remote row blocks copied once into the
    gathered buffer (bf16 and SwiGLU + LoRA expand epilogues, the shrink of
    the gathered rows, a second call reusing them) or read by every tile from
    their owners' memory == NCCL all-gather then the local GEMM (which may
    split K: equal to bf16 rounding); the gathered rows equal the shards."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_run_gemm_ag, args=(world, _port(), d), nprocs=world, join=True, start_method="spawn")
        for r in torch.load(os.path.join(d, "ag.pt"))["res"]:
            assert r["code"] == 0
            assert r["bf16"] < 1e-2 and r["shrink"] < 1e-2 and r["swiglu_lora"] < 1e-2, r
            assert r["gathered"] == 0.0 and r["bf16_direct"] < 1e-2, r
