"""The shared-memory step-plan channel between TP ranks (gloo ranks on CPU):
messages arrive in order on every follower, payloads larger than the slot
travel through the process-group fallback, the per-layer MAX vote agrees
with the process group's, and a wait ends with an error
(not a hang) when the peer process has exited."""
import os
import socket
import tempfile

import torch.distributed as dist
import torch.multiprocessing as mp

from deltaserve_vllm_b200.parallel.comm import TPComm
from deltaserve_vllm_b200.parallel.shm_channel import ShmChannel


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _order_worker(rank, world, port, outdir):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        comm = TPComm()
        ch = ShmChannel(comm, capacity=4096, timeout_s=60)
        msgs = [[("fwd", i, list(range(i % 7)))] for i in range(200)]
        msgs[50] = [("big", bytes(20000))]               # larger than the slot: fallback path
        msgs[51] = [("after_big", 51)]
        got = []
        for m in msgs:
            if rank == 0:
                ch.send(m)
            else:
                got.append(ch.recv())
        # votes: MAX over ranks, every rank sees the same sequence
        import random
        rng = random.Random(rank)
        flags = [1 if rng.random() < 0.1 else 0 for _ in range(300)]
        votes = [ch.all_max(f) for f in flags]
        all_flags = comm.all_gather_object(flags)
        votes_ok = votes == [max(col) for col in zip(*all_flags)]
        # the process group still works in step with the channel
        total = comm.all_reduce_max_int(rank)
        if rank != 0:
            ok = got == msgs and total == world - 1 and votes_ok
            with open(os.path.join(outdir, f"r{rank}"), "w") as f:
                f.write("ok" if ok else "bad")
        ch.close()
    finally:
        dist.destroy_process_group()


def test_shm_channel_order_and_fallback():
    world = 3
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_order_worker, args=(world, _port(), d), nprocs=world, join=True,
                           start_method="spawn")
        for r in range(1, world):
            assert open(os.path.join(d, f"r{r}")).read() == "ok"


def _dead_peer_worker(rank, world, port, outdir):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    comm = TPComm()
    ch = ShmChannel(comm, capacity=4096, timeout_s=60)
    if rank == 0:
        ch.send(["first"])
        # rank 1 exits without acknowledging: the next send must raise, not hang
        try:
            ch.send(["second"])
            res = "no error"
        except RuntimeError as e:
            res = "raised: " + str(e)
        with open(os.path.join(outdir, "r0"), "w") as f:
            f.write(res)
    else:
        os._exit(0)                                      # leaves before reading anything


def test_shm_channel_detects_exited_rank():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _port()
        procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive
        res = open(os.path.join(d, "r0")).read()
        assert res.startswith("raised:") and "rank 1 exited" in res, res


def _fallback_worker(rank, world, port, outdir):
    import deltaserve_vllm_b200.parallel.shm_channel as sc
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        if rank == 1:
            sc._SHM_DIR = os.path.join(outdir, "missing")   # this rank cannot open the segment
        comm = TPComm()
        try:
            sc.ShmChannel(comm, capacity=4096, timeout_s=60)
            res = "built"
        except sc.ChannelUnavailable:
            res = "unavailable"
        # the process group is still in step on every rank
        res += f" {comm.all_reduce_max_int(rank)}"
        with open(os.path.join(outdir, f"r{rank}"), "w") as f:
            f.write(res)
    finally:
        dist.destroy_process_group()


def test_shm_channel_setup_failure_is_agreed():
    world = 3
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_fallback_worker, args=(world, _port(), d), nprocs=world, join=True,
                           start_method="spawn")
        for r in range(world):
            assert open(os.path.join(d, f"r{r}")).read() == f"unavailable {world - 1}"
        if os.path.isdir("/dev/shm"):                   # rank 0 removed its segment
            assert not [f for f in os.listdir("/dev/shm") if f.startswith("dsv_tp_")]


def _idle_worker(rank, world, port, outdir):
    import time
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ch = ShmChannel(TPComm(), capacity=4096, timeout_s=0.5)
        if rank == 0:
            time.sleep(2.0)                  # an idle server: no plan for longer than timeout_s
            ch.send(["late"])
        else:
            with open(os.path.join(outdir, "r1"), "w") as f:
                f.write(repr(ch.recv()))
        ch.close()
    finally:
        dist.destroy_process_group()


def test_shm_channel_follower_waits_through_idle_periods():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_idle_worker, args=(2, _port(), d), nprocs=2, join=True, start_method="spawn")
        assert open(os.path.join(d, "r1")).read() == "['late']"
