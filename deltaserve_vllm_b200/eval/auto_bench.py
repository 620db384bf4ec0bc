"""The timeline benchmark in one command: launch the server from a YAML
config, replay a request trace against it, collect the results, shut down.

    python -m deltaserve_vllm_b200.eval.auto_bench --config configs/llama3_8b.yaml --co \\
        --rate 8 --duration 120 [--warmup-s 10] [--tp 2] [--step-trace] [--out-dir bench_out] [--tag run1]
    python -m deltaserve_vllm_b200.eval.auto_bench --config configs/qwen3_14b_tp2.yaml --co \\
        --timeline-csv timeline_tight.csv
    python -m deltaserve_vllm_b200.eval.auto_bench --config configs/llama3_8b.yaml --trace trace.jsonl   # inference only

Steps: the YAML is resolved (relative paths made absolute) and written to the
output directory with this run's overrides (port, finetuning on or off, the
step trace and metrics paths); ``deltaserve_vllm_b200.launch`` serves it (as
its own process group, re-running itself under torchrun for TP), its output in
``server_<tag>.log``; once ``/health`` answers, ``--co`` opens finetuning
admission, the first ``--warmup-s`` seconds of the trace are replayed without
being recorded, then the whole trace is replayed as streaming requests. Output:

    results_<tag>.jsonl    per request: TTFT, TBT, tokens, routing headers, send wall time
    summary_<tag>.json     SLO attainment, TTFT / TBT percentiles, FT tokens trained per second
                           over the recorded window, the estimator report with --step-trace
    meta_<tag>.json        wall-clock anchor of the recorded window, command, config path
    step_trace_<tag>.csv   with --step-trace (see eval.estimator_report)
    gpu_util_<tag>.csv     with --gpu-util: NVML utilisation and memory per GPU every 0.2 s

The reference's counterpart is ``eval-tp/auto_benchmark_tp.py`` (its timeline
CSVs load with ``--timeline-csv``).
"""

from __future__ import annotations

import argparse
import asyncio
import json
import os
import signal
import socket
import subprocess
import sys
import time
import urllib.request

import yaml


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _get(url: str, timeout: float = 5.0) -> dict:
    with urllib.request.urlopen(url, timeout=timeout) as r:
        return json.loads(r.read().decode())


def _post(url: str, body: dict | None = None, timeout: float = 60.0) -> dict:
    req = urllib.request.Request(url, data=json.dumps(body or {}).encode(),
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read().decode() or "{}")


def derive_config(config: str, out_dir: str, tag: str, port: int, co: bool, step_trace: bool,
                  tp: int | None = None) -> tuple[str, dict]:
    """This run's YAML: the given one with paths resolved and the overrides
    applied. Returns (path, resolved sections)."""
    from ..config_loader import load_yaml_config
    cfg = load_yaml_config(config)
    cfg.setdefault("server", {}).update({"host": "127.0.0.1", "port": port})
    ft = cfg.setdefault("finetune_param", {})
    if not co:
        for s in ("finetune", "finetune_param"):
            if cfg.get(s) and "enable_finetuning" in cfg[s]:
                cfg[s]["enable_finetuning"] = False
        ft["enable_finetuning"] = False
    tel = cfg.setdefault("telemetry", {})
    tel["metrics_dir"] = os.path.abspath(os.path.join(out_dir, f"metrics_{tag}"))
    if step_trace:
        tel["step_trace_path"] = os.path.abspath(os.path.join(out_dir, f"step_trace_{tag}.csv"))
    if tp:
        cfg.setdefault("parallel", {})["tensor_parallel_size"] = tp
    path = os.path.join(out_dir, f"config_{tag}.yaml")
    with open(path, "w") as f:
        yaml.safe_dump(cfg, f, sort_keys=False)
    return path, cfg


def build_trace(a, vocab: int) -> list[dict]:
    from .trace import _read, from_timeline_csv, make_trace
    if a.trace:
        return _read(a.trace)
    if a.timeline_csv:
        return from_timeline_csv(a.timeline_csv, vocab, a.seed)
    rates = [float(x) for x in a.rates.split(",")] if a.rates else None
    return make_trace(a.rate, a.duration, vocab, a.seed, a.prompt_median, a.prompt_sigma, a.prompt_min,
                      a.prompt_max, a.out_min, a.out_max, a.adapters.split(",") if a.adapters else None,
                      rates, a.period, a.prompt_dist)


def _wait_ready(url: str, proc: subprocess.Popen, timeout_s: float, log_path: str) -> None:
    t0 = time.time()
    while time.time() - t0 < timeout_s:
        if proc.poll() is not None:
            raise RuntimeError(f"the server exited with code {proc.returncode} before it was ready:\n"
                               + _tail(log_path))
        try:
            if _get(url + "/health", timeout=2.0).get("ok"):
                return
        except Exception:
            pass
        time.sleep(0.5)
    raise TimeoutError(f"the server was not ready after {timeout_s:.0f} s:\n" + _tail(log_path))


def _tail(path: str, n: int = 30) -> str:
    try:
        with open(path) as f:
            return "".join(f.readlines()[-n:])
    except OSError:
        return ""


def _stop(url: str, proc: subprocess.Popen, timeout_s: float = 60.0) -> int:
    """POST /shutdown, then wait; the process group started here is signalled
    if it does not end in time."""
    try:
        _post(url + "/shutdown", timeout=10.0)
    except Exception:
        pass
    try:
        return proc.wait(timeout=timeout_s)
    except subprocess.TimeoutExpired:
        pass
    for sig in (signal.SIGTERM, signal.SIGKILL):
        try:
            os.killpg(proc.pid, sig)      # the group this script created for the server
        except ProcessLookupError:
            break
        try:
            return proc.wait(timeout=20.0)
        except subprocess.TimeoutExpired:
            continue
    return proc.returncode if proc.returncode is not None else -1


class GpuUtilSampler:
    """Whole-device GPU utilisation and memory (NVML, read only) sampled on a
    thread every ``period_s`` with unix timestamps, to set the served load
    against the GPU's busy share over the same window."""

    def __init__(self, path: str, period_s: float = 0.2, nvml=None):
        import threading
        self.path, self.period_s = path, float(period_s)
        self.rows: list[tuple] = []
        self.error = None
        self._stop = threading.Event()
        self._nvml = nvml
        self._t = threading.Thread(target=self._run, daemon=True, name="dsv-gpu-util")

    def _run(self) -> None:
        try:
            nv = self._nvml
            if nv is None:
                import pynvml as nv
            nv.nvmlInit()
            handles = [nv.nvmlDeviceGetHandleByIndex(i) for i in range(nv.nvmlDeviceGetCount())]
        except Exception as e:        # no driver or no NVML here: nothing to sample
            self.error = repr(e)
            return
        while not self._stop.is_set():
            t = time.time()
            for i, h in enumerate(handles):
                try:
                    u = nv.nvmlDeviceGetUtilizationRates(h)
                    m = nv.nvmlDeviceGetMemoryInfo(h)
                    self.rows.append((round(t, 3), i, int(u.gpu), int(m.used) // (1 << 20)))
                except Exception as e:
                    self.error = repr(e)
            self._stop.wait(self.period_s)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=5)
        with open(self.path, "w") as f:
            f.write("timestamp,gpu,util_pct,mem_used_mb\n")
            for r in self.rows:
                f.write(",".join(map(str, r)) + "\n")

    def summary(self) -> dict:
        if not self.rows:
            return {"samples": 0, "error": self.error}
        by_gpu: dict = {}
        for _, g, u, _m in self.rows:
            by_gpu.setdefault(g, []).append(u)
        return {"samples": len(self.rows),
                "util_mean_pct": {str(g): round(sum(v) / len(v), 1) for g, v in sorted(by_gpu.items())},
                "mem_used_max_mb": max(r[3] for r in self.rows)}


def run(a) -> dict:
    from ..models.configs import resolve_arch
    from .replay import _status, replay
    from .report import summarize
    from .trace import slice_trace
    os.makedirs(a.out_dir, exist_ok=True)
    tag = a.tag or time.strftime("%Y%m%d_%H%M%S")
    port = a.port or _free_port()
    cfg_path, cfg = derive_config(a.config, a.out_dir, tag, port, a.co, a.step_trace, a.tp)
    arch = resolve_arch(cfg.get("model", {}).get("model", "llama3-8b"))
    trace = build_trace(a, arch.vocab)
    url = f"http://127.0.0.1:{port}"
    log_path = os.path.join(a.out_dir, f"server_{tag}.log")
    cmd = [sys.executable, "-m", "deltaserve_vllm_b200.launch", "--config", cfg_path]
    if a.co:
        cmd.append("--start-finetuning")
    with open(log_path, "w") as log:
        proc = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, start_new_session=True)
    rc = None
    try:
        _wait_ready(url, proc, a.ready_timeout, log_path)
        warm = slice_trace(trace, 0.0, a.warmup_s) if a.warmup_s > 0 else []
        if warm:
            asyncio.run(replay(url, warm, a.model, a.speed))
        before = _status(url)
        util = GpuUtilSampler(os.path.join(a.out_dir, f"gpu_util_{tag}.csv")) if a.gpu_util else None
        if util is not None:
            util.__enter__()
        t0 = time.time()
        try:
            res = asyncio.run(replay(url, trace, a.model, a.speed))
        finally:
            wall = time.time() - t0
            if util is not None:
                util.__exit__(None, None, None)
        after = _status(url)
    finally:
        rc = _stop(url, proc)
    with open(os.path.join(a.out_dir, f"results_{tag}.jsonl"), "w") as f:
        for r in res:
            f.write(json.dumps(r) + "\n")
    s = summarize(res, a.ttft_slo, a.tbt_slo)
    ft = (after.get("total_trained_tokens") or 0) - (before.get("total_trained_tokens") or 0)
    s.update({"tag": tag, "wall_s": round(wall, 3), "ft_tokens_trained": ft,
              "ft_tok_s": round(ft / wall, 1) if wall > 0 else None, "server_exit_code": rc,
              "warmup_requests": len(warm)})
    if util is not None:
        s["gpu_util"] = util.summary()
    if a.step_trace:
        from .estimator_report import load_trace, report
        tp = os.path.join(a.out_dir, f"step_trace_{tag}.csv")
        if os.path.exists(tp):
            rows = [r for r in load_trace(tp) if r["t_done"] is not None and r["t_done"] >= t0]
            rep = report(rows, res, a.ttft_slo, 5, a.tbt_slo)
            s["estimator"] = {"steps": rep["steps"], "overall": rep["accuracy"]["overall"],
                              "margin_coverage": rep["accuracy"]["margin_coverage"],
                              "over_limit": rep["over_limit"]}
    with open(os.path.join(a.out_dir, f"summary_{tag}.json"), "w") as f:
        json.dump(s, f, indent=1)
    with open(os.path.join(a.out_dir, f"meta_{tag}.json"), "w") as f:
        json.dump({"t_first_wall": t0, "config": cfg_path, "command": cmd, "requests": len(trace),
                   "co": a.co}, f, indent=1)
    return s


def parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", required=True)
    ap.add_argument("--co", action="store_true", help="co-serving: open finetuning admission (else inference only)")
    ap.add_argument("--tp", type=int, default=None)
    ap.add_argument("--port", type=int, default=None)
    ap.add_argument("--out-dir", default="bench_out")
    ap.add_argument("--tag", default=None)
    ap.add_argument("--step-trace", action="store_true")
    ap.add_argument("--gpu-util", action="store_true", help="sample GPU utilisation and memory (NVML) while recording")
    ap.add_argument("--ready-timeout", type=float, default=900.0)
    ap.add_argument("--warmup-s", type=float, default=0.0, help="replay the trace's first seconds unrecorded first")
    ap.add_argument("--model", default=None, help="request model field (e.g. auto for routing)")
    ap.add_argument("--speed", type=float, default=1.0)
    ap.add_argument("--ttft-slo", type=float, default=0.5)
    ap.add_argument("--tbt-slo", type=float, default=0.06)
    src = ap.add_mutually_exclusive_group()
    src.add_argument("--trace", default=None, help="a trace JSONL (eval.trace)")
    src.add_argument("--timeline-csv", default=None, help="timestamp_s,prompt_length,max_new_tokens CSV")
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--rates", default=None)
    ap.add_argument("--period", type=float, default=15.0)
    ap.add_argument("--duration", type=float, default=60.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--prompt-dist", default="lognormal", choices=["lognormal", "loguniform"])
    ap.add_argument("--prompt-median", type=int, default=512)
    ap.add_argument("--prompt-sigma", type=float, default=0.8)
    ap.add_argument("--prompt-min", type=int, default=32)
    ap.add_argument("--prompt-max", type=int, default=4096)
    ap.add_argument("--out-min", type=int, default=32)
    ap.add_argument("--out-max", type=int, default=256)
    ap.add_argument("--adapters", default=None)
    return ap.parse_args(argv)


def main(argv=None) -> None:
    print(json.dumps(run(parse(argv))))


if __name__ == "__main__":
    main()
