"""Eval harness and dashboard against a live HTTP server on CPU: a trace is
generated, replayed with streaming requests (TTFT/TBT per request), summarized;
dserve-top polls the same server and exports its history."""
import json
import os
import socket
import tempfile
import threading
import time

import uvicorn

from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
from deltaserve_vllm_b200.eval import report
from deltaserve_vllm_b200.eval.replay import replay
from deltaserve_vllm_b200.eval.trace import make_trace
from deltaserve_vllm_b200.server.api import create_app
from deltaserve_vllm_b200.utils import top


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_replay_report_and_top():
    import asyncio
    with tempfile.TemporaryDirectory() as tmp:
        ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=512, block_size=16,
                            max_num_batched_tokens=256, max_loras=2, max_lora_rank=8)
        fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=96,
                              metrics_dir=os.path.join(tmp, "m"), metrics_interval_s=0.2)
        store = FinetuningStore.synthetic(1024, 8, 16, 40, seed=0, max_saved_finetuning_tokens=96,
                                          total_epochs=100)
        eng = CoServingEngine(ecfg, fcfg, ft_store=store)
        app = create_app(eng)
        port = _port()
        srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
        th = threading.Thread(target=srv.run, daemon=True)
        th.start()
        url = f"http://127.0.0.1:{port}"
        for _ in range(200):
            if srv.started:
                break
            time.sleep(0.05)
        rec = top.Recorder(url, poll_s=0.1)
        rec.start_telemetry()
        trace = make_trace(20.0, 0.5, 1024, seed=1, prompt_median=24, prompt_min=4, prompt_max=64,
                           out_min=2, out_max=6)
        res = asyncio.run(replay(url, trace))
        s = report.summarize(res, ttft_slo=30.0, tbt_slo=30.0)
        assert s["completed"] == len(trace) and s["errors"] == 0
        assert s["slo_attainment"] == 1.0 and s["ttft_p99_s"] is not None
        assert all(r["output_tokens"] == t["max_tokens"] for r, t in zip(res, trace))
        rec.poll_once()
        snap = rec.export()
        assert snap["steps"] and snap["metrics"]
        with open(os.path.join(tmp, "top.json"), "w") as f:
            json.dump(snap, f)
        r2 = top.Recorder(None)
        r2.load(os.path.join(tmp, "top.json"))
        assert len(r2.steps) == len(snap["steps"])
        srv.should_exit = True
        th.join(timeout=30)
        eng.shutdown()
        rep = report.metrics_dir_report(os.path.join(tmp, "m"), 30.0, 30.0)
        assert rep["requests"]["completed"] == len(trace)
        cmp_ = report.compare(s, s)
        assert cmp_["completed"]["delta"] == 0


def test_pure_ft_throughput_cpu():
    from deltaserve_vllm_b200.eval import pure_ft
    r = pure_ft.run("qwen3-tiny", seq=32, batch=2, cycles=3, warmup=1, device="cpu", rank=8)
    assert r["cycles"] == 3 and r["ft_tokens"] == 3 * 2 * 32
    assert r["ft_tok_s"] > 0 and r["wall_s"] > 0
