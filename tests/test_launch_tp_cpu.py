"""The launcher end to end on CPU ranks: ``--tp 2`` re-runs itself under
torchrun (two gloo ranks), serves HTTP on rank 0, answers a completion with
both ranks stepping in lockstep, shuts down cleanly on ``POST /shutdown``,
and leaves no orphan when rank 0 is killed (the reference's process-hygiene
check, ``tests/test_tp_no_orphans.py``: SIGKILL the engine process, every
worker is gone within 20 s)."""

import json
import os
import signal
import socket
import subprocess
import sys
import textwrap
import time
import urllib.request

import pytest

psutil = pytest.importorskip("psutil")

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _config(tmp, port) -> str:
    path = os.path.join(tmp, "tiny.yaml")
    with open(path, "w") as f:
        f.write(textwrap.dedent(f"""
            model:
              model: qwen3-tiny
              max_model_len: 256
              device: cpu
            engine:
              block_size: 16
              max_num_batched_tokens: 128
              max_loras: 2
              max_lora_rank: 8
            finetune_param:
              enable_finetuning: false
            server:
              host: 127.0.0.1
              port: {port}
        """))
    return path


def _get(url, timeout=2.0):
    with urllib.request.urlopen(url, timeout=timeout) as r:
        return json.loads(r.read())


def _post(url, body, timeout=60.0):
    req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read())


def _start(tmp):
    port = _port()
    cfg = _config(tmp, port)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=REPO)
    proc = subprocess.Popen([sys.executable, "-m", "deltaserve_vllm_b200.launch", "--config", cfg, "--tp", "2",
                             "--no-profile"], cwd=tmp, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                            start_new_session=True)
    base = f"http://127.0.0.1:{port}"
    t0 = time.time()
    while time.time() - t0 < 150:
        if proc.poll() is not None:
            raise AssertionError(proc.stdout.read().decode()[-3000:])
        try:
            if _get(base + "/health").get("ok"):
                return proc, base
        except Exception:
            time.sleep(0.5)
    proc.kill()
    raise AssertionError("server did not come up")


def _family(proc):
    try:
        p = psutil.Process(proc.pid)
        return [p] + p.children(recursive=True)
    except psutil.NoSuchProcess:
        return []


def _all_gone(procs, timeout):
    t0 = time.time()
    while time.time() - t0 < timeout:
        alive = [p for p in procs if p.is_running() and p.status() != psutil.STATUS_ZOMBIE]
        if not alive:
            return True
        time.sleep(0.25)
    return False


def test_launch_tp2_serves_and_shuts_down(tmp_path):
    proc, base = _start(str(tmp_path))
    try:
        ranks = [p for p in psutil.Process(proc.pid).children(recursive=True) if "deltaserve_vllm_b200.launch" in
                 " ".join(p.cmdline())]
        assert len(ranks) >= 2, [p.cmdline() for p in ranks]
        out = _post(base + "/v1/completions", {"prompt": "hello there", "max_tokens": 5})
        assert out["usage"]["completion_tokens"] == 5
        fam = _family(proc)
        _post(base + "/shutdown", {})
        assert proc.wait(timeout=60) == 0
        assert _all_gone(fam, 30)
    finally:
        if proc.poll() is None:
            os.killpg(proc.pid, signal.SIGKILL)


def test_launch_tp2_no_orphans_after_rank0_kill(tmp_path):
    proc, base = _start(str(tmp_path))
    try:
        fam = _family(proc)
        rank0 = None
        for p in fam:
            try:
                if p.environ().get("RANK") == "0" and "deltaserve_vllm_b200.launch" in " ".join(p.cmdline()):
                    rank0 = p
            except (psutil.AccessDenied, psutil.NoSuchProcess):
                pass
        assert rank0 is not None
        rank0.send_signal(signal.SIGKILL)
        assert _all_gone(fam, 30), [(p.pid, p.cmdline()) for p in fam if p.is_running()]
    finally:
        if proc.poll() is None:
            os.killpg(proc.pid, signal.SIGKILL)
