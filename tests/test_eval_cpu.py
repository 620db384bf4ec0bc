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


def test_estimator_report_from_a_step_trace(tmp_path):
    """The estimator report reads a trace written by the engine's step-trace
    writer: per-regime accuracy of the raw model (a regime predicted 20 %
    low shows ratio 1.25 and negative bias), the backward-in-flight split,
    margin coverage, admission fidelity, the worst miss and the steps during
    a request's TTFT violation."""
    from deltaserve_vllm_b200.eval.estimator_report import load_trace, report
    from deltaserve_vllm_b200.utils.step_trace import StepTraceWriter

    path = str(tmp_path / "trace.csv")
    w = StepTraceWriter(path)
    t0 = 1_000_000.0
    for i in range(40):
        dec = i % 2 == 0
        actual = 0.010 if dec else 0.025
        pred_raw = actual if dec else actual / 1.25          # the prefill regime under-predicts
        w.put_row(kind="decode" if dec else "prefill", t_done=t0 + 0.05 * i,
                  regime="decode_only" if dec else "inf_prefill",
                  regime_used="decode_only" if dec else "inf_prefill",
                  t_in=0 if dec else 512, p=0 if dec else 1, t_ft=0 if dec else 128, b_d=8, k=1024, s=0,
                  pred_raw=pred_raw, pred=pred_raw * 1.1, actual=actual,
                  admit_code="A" if not dec else None, t_baseline=None,
                  t_admit=0.02 if not dec else None, bwd_in_flight=not dec)
    # one outlier step
    w.put_row(kind="decode", t_done=t0 + 2.5, regime="decode_only", regime_used="decode_only", t_in=0, p=0,
              t_ft=0, b_d=8, k=1024, s=0, pred_raw=0.010, pred=0.011, actual=0.050, bwd_in_flight=True)
    w.close()
    rows = load_trace(path)
    assert len(rows) == 41
    results = [{"t": 0.0, "ttft_s": 0.8, "sent_unix": t0 + 0.02},     # waits through steps 1..16
               {"t": 1.0, "ttft_s": 0.1, "sent_unix": t0 + 1.0}]      # within the SLO
    rep = report(rows, results, ttft_slo=0.5, top=3, max_tbt_slo=0.02)
    acc = rep["accuracy"]
    pre = acc["by_regime"]["inf_prefill"]
    assert pre["n"] == 20 and abs(pre["ratio_p50"] - 1.25) < 1e-3 and pre["bias_ms"] < 0
    dec = acc["by_regime"]["decode_only"]
    assert dec["n"] == 21 and abs(dec["ratio_p50"] - 1.0) < 1e-3 and dec["over_2x"] > 0
    assert acc["margin_coverage"]["decode_only"] == round(20 / 21, 4)
    assert acc["margin_coverage"]["inf_prefill"] == 0.0              # 1.1 x margin < 1.25 x miss
    assert acc["by_backward_in_flight"]["True"]["n"] == 21
    adm = rep["admission"]
    assert adm["n"] == 20 and adm["actual_over_admit"] == 1.0 and adm["admit_codes"] == {"A": 20}
    assert rep["worst_misses"][0]["ratio"] == 5.0 and rep["worst_misses"][0]["step"]["seq"] == 41
    (v,) = rep["ttft_violations"]
    assert v["steps_while_waiting"] == 16 and v["steps_by_kind"] == {"decode": 8, "prefill": 8}
    ol = rep["over_limit"]
    assert ol["ft_steps_with_decodes"] == 20 and ol["ft_over_limit"] == 1.0
    assert ol["inference_steps_with_decodes"] == 21 and ol["inference_over_limit"] == round(1 / 21, 4)
    assert ol["ft_actual_over_admit_p50"] == 1.25
    from deltaserve_vllm_b200.eval.estimator_report import compare_row
    row = compare_row("arm", rows, 0.02)
    assert row["ft_over_limit"] == 1.0 and row["ft_tokens"] == 20 * 128
    assert row["margin_coverage"] == round(20 / 41, 4)


def test_prefill_probe_against_an_idle_server():
    """The prefill probe reports TTFT per prompt length (sequential, idle
    server) and the concurrent phase's aggregate rate, with no errors."""
    import asyncio
    from deltaserve_vllm_b200.eval.prefill_probe import probe
    ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=256, block_size=16,
                        max_num_batched_tokens=256, max_loras=1, max_lora_rank=8, enable_prefix_caching=True)
    eng = CoServingEngine(ecfg, FinetuneConfig(enable_finetuning=False))
    app = create_app(eng)
    port = _port()
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    for _ in range(200):
        if srv.started:
            break
        time.sleep(0.05)
    try:
        out = asyncio.run(probe(f"http://127.0.0.1:{port}", [32, 96], reps=2, conc=3, conc_len=64,
                                vocab=1024, max_tokens=2))
    finally:
        srv.should_exit = True
        th.join(timeout=30)
        eng.shutdown()
    s = out["summary"]
    assert s["errors"] == 0
    assert set(s["sequential"]) == {"32", "96"} and s["sequential"]["96"]["n"] == 2
    assert s["sequential"]["32"]["ms_per_token"] > 0
    assert s["concurrent"]["n"] == 3 and s["concurrent"]["aggregate_prefill_tok_s"] > 0
    assert len(out["rows"]) == 7


def test_trace_schedule_scale_slice_and_csv(tmp_path):
    """Trace generation with a rate schedule (peaks, valleys, an idle
    stretch) and log-uniform prompts; scale keeps the arrival pattern at a
    new rate; slice rebases a window; a timeline CSV becomes a trace."""
    import numpy as np
    from deltaserve_vllm_b200.eval.trace import from_timeline_csv, main, scale_trace, slice_trace
    tr = make_trace(0.0, 120.0, 1000, seed=3, rates=[2.0, 8.0, 0.0], period_s=10.0, prompt_dist="loguniform",
                    prompt_min=16, prompt_max=160, out_min=4, out_max=8)
    ts = np.array([r["t"] for r in tr])
    assert np.all(np.diff(ts) > 0)
    phase = (ts // 10).astype(int) % 3
    assert not np.any(phase == 2)                                # idle stretches stay empty
    lo, hi = np.sum(phase == 0), np.sum(phase == 1)
    assert 2.5 < hi / lo < 6.5                                   # 8 vs 2 req/s
    lens = np.array([len(r["prompt"]) for r in tr])
    assert lens.min() >= 16 and lens.max() <= 160 and np.median(lens) < 70   # log-uniform: median ~ 51
    # the single-rate stream is unchanged by the schedule support
    a = make_trace(5.0, 10.0, 1000, seed=1)
    b = make_trace(5.0, 10.0, 1000, seed=1, rates=[5.0])
    assert a == b
    half = scale_trace(tr, 0.5, seed=0)
    assert abs(len(half) - len(tr) / 2) <= 1 and set(r["t"] for r in half) <= set(ts.tolist())
    dbl = scale_trace(tr, 2.0, seed=0)
    assert len(dbl) == 2 * len(tr) and all(x["t"] <= y["t"] for x, y in zip(dbl, dbl[1:]))
    assert not any(int(r["t"] // 10) % 3 == 2 and r["t"] % 10 > 1.0 for r in dbl)   # pattern kept
    cut = slice_trace(tr, 30.0, 50.0)
    assert cut and all(0 <= r["t"] < 20.0 for r in cut)
    assert len(cut) == int(np.sum((ts >= 30.0) & (ts < 50.0)))
    csv_path = tmp_path / "timeline.csv"
    csv_path.write_text("timestamp_s,prompt_length,max_new_tokens,second,index_in_second\n"
                        "0.5,12,7,0,0\n1.25,40,3,1,0\n")
    got = from_timeline_csv(str(csv_path), vocab=500)
    assert [(r["t"], len(r["prompt"]), r["max_tokens"]) for r in got] == [(0.5, 12, 7), (1.25, 40, 3)]
    assert all(3 <= x < 500 for r in got for x in r["prompt"])
    import contextlib
    import io
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        main(["from-csv", "--input", str(csv_path), "--vocab", "500"])
    assert len(buf.getvalue().splitlines()) == 2


def test_auto_bench_launches_replays_and_shuts_down(tmp_path):
    """The one-command timeline benchmark on CPU: the launcher serves a
    derived YAML (finetuning on, step trace on), the trace is replayed with a
    warm-up slice first, finetuning tokens are trained during the recorded
    window, the server exits 0 on /shutdown and every output file exists."""
    from deltaserve_vllm_b200.eval.auto_bench import parse, run
    lines = [f"sample {i} " + "the quick brown fox jumps over the lazy dog " * (1 + i % 4) for i in range(200)]
    (tmp_path / "data.txt").write_text("\n".join(lines) + "\n")
    (tmp_path / "co.yaml").write_text(
        "model:\n  model: qwen3-tiny\n  max_model_len: 256\n  device: cpu\n"
        "engine:\n  block_size: 16\n  max_num_batched_tokens: 128\n  max_loras: 2\n  max_lora_rank: 8\n"
        "finetune_param:\n  enable_finetuning: true\n  data_path: data.txt\n  max_saved_finetuning_tokens: 64\n"
        "slo:\n  ttft_slo: 30.0\n  avg_tbt_slo: 30.0\n  max_tbt_slo: 30.0\n  profile_on_launch: false\n")
    out = tmp_path / "out"
    s = run(parse(["--config", str(tmp_path / "co.yaml"), "--co", "--rate", "10", "--duration", "3",
                   "--prompt-median", "24", "--prompt-min", "4", "--prompt-max", "64", "--out-min", "2",
                   "--out-max", "6", "--warmup-s", "0.5", "--out-dir", str(out), "--tag", "t",
                   "--step-trace", "--ttft-slo", "30", "--tbt-slo", "30", "--ready-timeout", "300"]))
    assert s["errors"] == 0 and s["completed"] == s["requests"] > 0
    assert s["server_exit_code"] == 0 and s["warmup_requests"] > 0
    assert s["ft_tokens_trained"] > 0 and s["estimator"]["steps"] > 0
    for name in ("config_t.yaml", "results_t.jsonl", "summary_t.json", "meta_t.json", "server_t.log",
                 "step_trace_t.csv"):
        assert (out / name).exists(), name
    res = [json.loads(x) for x in (out / "results_t.jsonl").read_text().splitlines()]
    assert len(res) == s["requests"] and all("sent_unix" in r for r in res)


def test_gpu_util_sampler_with_a_fake_nvml(tmp_path):
    """The utilisation sampler reads NVML only (a fake here): rows per GPU
    with timestamps, a per-GPU mean, and a clean summary without NVML."""
    import types
    from deltaserve_vllm_b200.eval.auto_bench import GpuUtilSampler
    calls = {"n": 0}

    def util(h):
        calls["n"] += 1
        return types.SimpleNamespace(gpu=50 + 10 * h)

    fake = types.SimpleNamespace(nvmlInit=lambda: None, nvmlDeviceGetCount=lambda: 2,
                                 nvmlDeviceGetHandleByIndex=lambda i: i,
                                 nvmlDeviceGetUtilizationRates=util,
                                 nvmlDeviceGetMemoryInfo=lambda h: types.SimpleNamespace(used=(1000 + h) << 20))
    path = tmp_path / "u.csv"
    with GpuUtilSampler(str(path), period_s=0.01, nvml=fake) as smp:
        for _ in range(200):
            if calls["n"] >= 6:
                break
            time.sleep(0.01)
    s = smp.summary()
    assert s["samples"] >= 6 and s["util_mean_pct"] == {"0": 50.0, "1": 60.0} and s["mem_used_max_mb"] == 1001
    lines = path.read_text().splitlines()
    assert lines[0] == "timestamp,gpu,util_pct,mem_used_mb" and len(lines) == s["samples"] + 1

    def broken():
        raise RuntimeError("no NVML")

    with GpuUtilSampler(str(tmp_path / "v.csv"), nvml=types.SimpleNamespace(nvmlInit=broken)) as smp2:
        time.sleep(0.05)
    assert smp2.summary()["samples"] == 0 and "no NVML" in smp2.summary()["error"]
