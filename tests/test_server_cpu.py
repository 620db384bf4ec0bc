"""HTTP API, telemetry and launcher on CPU: the FastAPI app drives a tiny
co-serving engine (fp32 oracle ops) through its own engine thread, mirroring
the reference's API tests (``tests/test_metrics_e2e.py``,
``tests/test_adapter_save_e2e.py``) without a model download."""
import json
import os
import tempfile
import textwrap
import time

import pytest
import torch
from fastapi.testclient import TestClient

from deltaserve_vllm_b200.adapters import peft_io
from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
from deltaserve_vllm_b200.server.api import create_app
from deltaserve_vllm_b200.utils.tokenizer import ByteTokenizer


def make_engine(tmp, start=False, **ft):
    ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=512, block_size=16,
                        max_num_batched_tokens=256, max_loras=3, max_lora_rank=8)
    fcfg = FinetuneConfig(enable_finetuning=True, start_on_launch=start, max_saved_finetuning_tokens=96,
                          learning_rate=1e-3, adapter_save_path=os.path.join(tmp, "ckpt"),
                          metrics_dir=os.path.join(tmp, "metrics"), metrics_interval_s=0.2,
                          step_trace_path=os.path.join(tmp, "trace.csv"), **ft)
    store = FinetuningStore.synthetic(1024, 8, 16, 40, seed=0, max_saved_finetuning_tokens=96,
                                      total_epochs=1000)
    eng = CoServingEngine(ecfg, fcfg, ft_store=store, tokenizer=ByteTokenizer(1024))
    eng.load_inference_adapter("toy", rank=8, alpha=16)
    return eng


def _wait(pred, timeout=60.0):
    t0 = time.time()
    while time.time() - t0 < timeout:
        if pred():
            return True
        time.sleep(0.05)
    return False


def test_api_completions_and_finetuning_control():
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)
        app = create_app(eng)
        with TestClient(app) as c:
            assert c.get("/health").json()["ok"]
            data = c.get("/v1/models").json()["data"]
            names = [m["id"] for m in data]
            assert "qwen3-tiny" in names and "toy" in names
            by = {m["id"]: m for m in data}
            assert by["toy"]["parent"] == "qwen3-tiny" and by["qwen3-tiny"]["parent"] is None
            assert by["toy"]["max_model_len"] == 512
            r = c.post("/v1/completions", json={"prompt": "hello world", "max_tokens": 4})
            assert r.status_code == 200, r.text
            out = r.json()
            assert out["usage"]["completion_tokens"] == 4
            assert out["usage"]["prompt_tokens"] == len("hello world")
            assert out["metrics"]["ttft_s"] is not None
            # adapter by name, token-id prompt
            r = c.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 3, "model": "toy"})
            assert r.status_code == 200 and len(r.json()["choices"][0]["token_ids"]) == 3
            assert c.post("/v1/completions", json={"prompt": "x", "model": "nope"}).status_code == 404
            pc = c.get("/prefix_cache").json()
            assert pc["enabled"] is False and 0.0 <= pc["kv_usage"] <= 1.0
            assert c.post("/v1/completions", json={"max_tokens": 3}).status_code == 400
            # streaming: every token arrives, then [DONE]
            with c.stream("POST", "/v1/completions",
                          json={"prompt": "stream me", "max_tokens": 5, "stream": True}) as s:
                chunks = [ln for ln in s.iter_lines() if ln.startswith("data: ")]
            assert chunks[-1] == "data: [DONE]"
            n_tok = sum(len(json.loads(ch[6:])["choices"][0].get("token_ids") or []) for ch in chunks[:-1])
            assert n_tok == 5
            # finetuning: closed at launch, opened by the route, cycles complete
            st = c.get("/finetuning_status").json()
            assert not st["ft_started"]
            assert c.post("/start_finetuning").json()["status"]["ft_started"]
            assert _wait(lambda: c.get("/finetuning_status").json()["completed_cycles"] >= 1)
            # telemetry live feed
            snap = c.get("/system_metrics").json()
            assert snap["totals"]["requests"] >= 3
            data = c.get("/telemetry/data", params={"steps_since": 0}).json()
            assert data["steps"]
            mem = c.post("/telemetry/memory", json={}).json()
            assert mem["weights_gb"] > 0
            # PEFT save through the API, merged and readable
            r = c.post("/save_adapter", json={"path": os.path.join(tmp, "manual"), "wait": True})
            assert r.status_code == 200 and r.json()["saved"], r.text
            tensors, cfg = peft_io.read_adapter(os.path.join(tmp, "manual"))
            assert len(tensors) == 2 * 7 * eng.arch.num_layers
            r = c.post("/save_estimator_state", json={"path": os.path.join(tmp, "est.json")})
            assert r.status_code == 200
            assert c.post("/stop_finetuning").json()["status"]["ft_started"] is False
            # adapters: list, unload, reload by path
            peft_io.write_peft_adapter(os.path.join(tmp, "a2"), tensors, cfg, {"save_id": "t"})
            r = c.post("/adapters", json={"path": os.path.join(tmp, "a2")})
            assert r.status_code == 200, r.text
            assert "a2" in c.get("/adapters/available").json()["by_name"]
            assert c.delete("/adapters/a2").status_code == 200
            assert "a2" not in c.get("/adapters/available").json()["by_name"]
            jobs = c.get("/ft_jobs").json()["jobs"]
            assert isinstance(jobs, list)
            assert c.post("/ft_jobs", json={"bogus": 1}).status_code == 400
            assert c.post("/shutdown").json()["shutdown"]
        eng.shutdown()
        # telemetry files on disk
        mdir = os.path.join(tmp, "metrics")
        assert os.path.exists(os.path.join(mdir, "requests.csv"))
        with open(os.path.join(mdir, "requests.csv")) as f:
            assert len(f.read().strip().splitlines()) >= 4
        with open(os.path.join(tmp, "trace.csv")) as f:
            lines = f.read().strip().splitlines()
        assert lines[0].startswith("seq,kind") and len(lines) > 2
        with open(os.path.join(tmp, "est.json")) as f:
            st = json.load(f)
        assert st["version"] == 1 and st["tracker"]["cols"]["duration"]


def test_estimator_state_round_trip():
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "est.json")
        eng = make_engine(tmp, estimator_state_save_path=path)
        eng.profile_execution_model(repeats=1)
        assert eng.estimator.is_ready
        eng.shutdown()                      # saves once at shutdown
        with open(path) as f:
            saved = json.load(f)
        eng2 = make_engine(tmp, estimator_state_load_path=path, profile_num_repeats=1)
        eng2.profile_execution_model(shapes=[], repeats=1)
        assert eng2.tracker.size() == len(saved["tracker"]["cols"]["duration"])
        assert eng2.estimator.export_state()["regimes"] == saved["estimator"]["regimes"]
        # a missing file is a warning, not an error
        assert not eng2.load_estimator_state(os.path.join(tmp, "missing.json"))


def test_launcher_dry_run(capsys):
    from deltaserve_vllm_b200 import launch
    with tempfile.TemporaryDirectory() as tmp:
        cfg = os.path.join(tmp, "c.yaml")
        with open(cfg, "w") as f:
            f.write(textwrap.dedent("""
                finetune_param:
                  enable_finetuning: true
                  data_path: data.txt
                  max_saved_finetuning_tokens: 256
                slo:
                  ttft_slo: 0.5
                server:
                  host: 127.0.0.1
                  port: 8123
                model:
                  model: qwen3-tiny
                parallel:
                  tensor_parallel_size: 1
            """))
        assert launch.main(["--config", cfg, "--dry-run", "--tp", "2", "--port", "9000"]) == 0
        out = json.loads(capsys.readouterr().out)
        assert out["engine"]["tensor_parallel_size"] == 2
        assert out["server"]["port"] == 9000
        assert out["finetune"]["data_path"] == os.path.join(os.path.realpath(tmp), "data.txt")
        assert out["finetune"]["ttft_slo"] == 0.5


def test_shipped_config_templates_load():
    """Every YAML template under configs/ resolves through the launcher."""
    import glob
    from deltaserve_vllm_b200 import launch
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    files = sorted(glob.glob(os.path.join(root, "configs", "*.yaml")))
    assert len(files) >= 4
    for f in files:
        ecfg, ftcfg, rcfg, extras, host, port = launch.resolve(launch.parse(["--config", f]))
        assert ecfg.model and port > 0
        assert ftcfg.enable_finetuning


def test_toy_adapter_builder(tmp_path):
    """The toy-adapter CLI trains adapters with the engine itself and writes
    PEFT dirs, their -ft twins and the topic corpus."""
    from deltaserve_vllm_b200.adapters import peft_io, toy
    out = str(tmp_path / "adapters")
    assert toy.main(["--model", "qwen3-tiny", "--out", out, "--count", "2", "--rank", "8", "--alpha", "16",
                     "--epochs", "1", "--device", "cpu"]) == 0
    assert sorted(os.listdir(out)) == ["toy-00", "toy-00-ft", "toy-01", "toy-01-ft"]
    t0, cfg = peft_io.read_adapter(os.path.join(out, "toy-00"))
    t0ft, _ = peft_io.read_adapter(os.path.join(out, "toy-00-ft"))
    t1, _ = peft_io.read_adapter(os.path.join(out, "toy-01"))
    assert cfg["r"] == 8 and sorted(cfg["target_modules"]) == ["k_proj", "o_proj", "q_proj", "v_proj"]
    assert all(".mlp." not in k for k in t0)
    assert all(torch.equal(t0[k], t0ft[k]) for k in t0)
    bkeys = [k for k in t0 if ".lora_B." in k]
    assert any(t0[k].abs().max() > 0 for k in bkeys)            # trained away from B = 0
    assert any(not torch.equal(t0[k], t1[k]) for k in bkeys)
    lines = open(os.path.join(out, "toy-01", "data.txt")).read().splitlines()
    assert len(lines) == 96 and all(line.endswith(")") for line in lines)
    assert toy.topic_corpus(0)[0] != toy.topic_corpus(1)[0]



def test_api_sampling_options_stop_n_logprobs():
    """OpenAI sampling options: top_k / top_p (kept-set sampling), logprobs of
    the chosen tokens, stop strings (output cut before the match), n > 1."""
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)
        app = create_app(eng)
        with TestClient(app) as c:
            r = c.post("/v1/completions", json={"prompt": "abc", "max_tokens": 6, "temperature": 1.0,
                                                "top_k": 1, "seed": 3, "logprobs": 0}).json()
            g = c.post("/v1/completions", json={"prompt": "abc", "max_tokens": 6}).json()
            # top_k = 1 leaves only the argmax: equal to greedy whatever the noise
            assert r["choices"][0]["token_ids"] == g["choices"][0]["token_ids"]
            lps = r["choices"][0]["logprobs"]["token_logprobs"]
            assert len(lps) == 6 and all(x <= 0.0 for x in lps)
            many = c.post("/v1/completions", json={"prompt": "abc", "max_tokens": 5, "temperature": 1.5,
                                                   "top_p": 0.9, "n": 3, "seed": 7}).json()
            assert [ch["index"] for ch in many["choices"]] == [0, 1, 2]
            assert many["usage"]["completion_tokens"] == 15
            # stop string: the text of the greedy continuation, from its second token on
            full = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 8}).json()["choices"][0]
            ids = full["token_ids"]
            stop_text = eng.tokenizer.decode(ids[2:4])
            if stop_text:
                st = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 8,
                                                     "stop": [stop_text]}).json()["choices"][0]
                assert st["finish_reason"] == "stop"
                assert stop_text not in st["text"] and len(st["token_ids"]) <= 4
            assert c.post("/v1/completions", json={"prompt": "x", "top_p": 0}).status_code == 400


def test_api_chat_completions():
    with tempfile.TemporaryDirectory() as tmp:
        eng = make_engine(tmp)
        app = create_app(eng)
        with TestClient(app) as c:
            msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}]
            r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 4})
            assert r.status_code == 200, r.text
            out = r.json()
            assert out["object"] == "chat.completion"
            assert out["choices"][0]["message"]["role"] == "assistant"
            assert out["usage"]["completion_tokens"] == 4
            with c.stream("POST", "/v1/chat/completions",
                          json={"messages": msgs, "max_tokens": 3, "stream": True}) as s:
                lines = [ln for ln in s.iter_lines() if ln.startswith("data: ")]
            assert lines[-1] == "data: [DONE]"
            chunks = [json.loads(ln[6:]) for ln in lines[:-1]]
            assert chunks[0]["object"] == "chat.completion.chunk"
            assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
            assert chunks[-1]["choices"][0]["finish_reason"] == "length"
            two = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 2, "n": 2,
                                                       "temperature": 1.0, "logprobs": True}).json()
            assert len(two["choices"]) == 2 and len(two["choices"][1]["logprobs"]["content"]) == 2
            assert c.post("/v1/chat/completions", json={"max_tokens": 2}).status_code == 400


def test_api_vllm_compatible_extras(tmp_path):
    """The routes a client of vLLM's OpenAI server also uses: /metrics
    (Prometheus text), /tokenize and /detokenize, /version, /ping, and runtime
    LoRA loading (/v1/load_lora_adapter, /v1/unload_lora_adapter)."""
    from deltaserve_vllm_b200.models.configs import resolve_arch
    from deltaserve_vllm_b200.models.lora import LORA_PROJS, random_adapter
    eng = make_engine(str(tmp_path))
    arch = resolve_arch("qwen3-tiny")
    adir = str(tmp_path / "extra_ad")
    peft_io.write_peft_adapter(adir, random_adapter(arch, 8, seed=5),
                               peft_io.default_adapter_config(8, 16.0, LORA_PROJS), {"save_id": "x"})
    with TestClient(create_app(eng)) as c:
        assert c.get("/ping").status_code == 200
        assert c.get("/version").json()["version"]
        t = c.post("/tokenize", json={"prompt": "hello"}).json()
        assert t["count"] == 5 and t["max_model_len"] == 512
        assert c.post("/detokenize", json={"tokens": t["tokens"]}).json()["prompt"] == "hello"
        assert c.post("/tokenize", json={"messages": [{"role": "user", "content": "hi"}]}).json()["count"] > 2
        assert c.post("/tokenize", json={}).status_code == 400
        # runtime LoRA loading
        r = c.post("/v1/load_lora_adapter", json={"lora_name": "extra", "lora_path": adir})
        assert r.status_code == 200 and "Success" in r.text, r.text
        assert c.post("/v1/load_lora_adapter", json={"lora_name": "extra", "lora_path": adir}).status_code == 400
        assert "extra" in [m["id"] for m in c.get("/v1/models").json()["data"]]
        r = c.post("/v1/completions", json={"model": "extra", "prompt": "abc", "max_tokens": 3})
        assert r.status_code == 200 and r.json()["usage"]["completion_tokens"] == 3
        r = c.post("/v1/completions", json={"prompt": "abcd", "max_tokens": 2})
        assert r.status_code == 200
        r = c.post("/v1/unload_lora_adapter", json={"lora_name": "extra"})
        assert r.status_code == 200 and "removed" in r.text
        assert c.post("/v1/unload_lora_adapter", json={"lora_name": "extra"}).status_code == 404
        assert c.post("/v1/completions", json={"model": "extra", "prompt": "a", "max_tokens": 1}).status_code == 404
        # Prometheus exposition
        m = c.get("/metrics")
        assert m.status_code == 200 and m.headers["content-type"].startswith("text/plain")
        lines = m.text.splitlines()
        val = {ln.split(" ")[0]: float(ln.split(" ")[1]) for ln in lines if ln and not ln.startswith("#")}
        lab = '{model_name="qwen3-tiny"}'
        assert val["dserve:prompt_tokens_total" + lab] == 7
        assert val["dserve:generation_tokens_total" + lab] == 5
        assert val["dserve:time_to_first_token_seconds_count"] == 2
        assert val['dserve:time_to_first_token_seconds_bucket{le="+Inf"}'] == 2
        assert val["dserve:time_per_output_token_seconds_count"] == 3      # (3-1) + (2-1) gaps
        assert val["dserve:num_requests_running" + lab] == 0
        assert 0.0 <= val["dserve:kv_cache_usage_perc" + lab] <= 1.0
        assert "dserve:ft_tokens_trained_total" + lab in val
        # every sample line belongs to a declared family
        declared = {ln.split(" ")[2] for ln in lines if ln.startswith("# TYPE")}
        for name in val:
            base = name.split("{")[0]
            assert any(base == d or base.startswith(d + "_") for d in declared), name


def test_api_prompt_batches_echo_and_stream_usage(tmp_path):
    """A completions request with a batch of prompts gives n choices per
    prompt in prompt order (each equal to the prompt run alone with the same
    seed), ``echo`` prefixes the prompt text, and
    ``stream_options.include_usage`` adds a usage chunk before [DONE]."""
    eng = make_engine(str(tmp_path))
    with TestClient(create_app(eng)) as c:
        single = {}
        for p in ("abc", "hello"):
            r = c.post("/v1/completions", json={"prompt": p, "max_tokens": 4})
            single[p] = r.json()["choices"][0]["token_ids"]
        r = c.post("/v1/completions", json={"prompt": ["abc", "hello"], "max_tokens": 4})
        assert r.status_code == 200, r.text
        out = r.json()
        assert [ch["index"] for ch in out["choices"]] == [0, 1]
        assert out["choices"][0]["token_ids"] == single["abc"]           # greedy: seed-independent
        assert out["choices"][1]["token_ids"] == single["hello"]
        assert out["usage"] == {"prompt_tokens": 8, "completion_tokens": 8, "total_tokens": 16}
        r = c.post("/v1/completions", json={"prompt": [[10, 11, 12], [13, 14]], "max_tokens": 2, "n": 2,
                                            "temperature": 1.0, "seed": 3})
        assert r.status_code == 200 and len(r.json()["choices"]) == 4
        assert r.json()["usage"]["prompt_tokens"] == 5
        # echo
        r = c.post("/v1/completions", json={"prompt": "abc", "max_tokens": 4, "echo": True})
        assert r.json()["choices"][0]["text"].startswith("abc")
        assert r.json()["choices"][0]["token_ids"] == single["abc"]
        # streamed usage
        with c.stream("POST", "/v1/completions", json={"prompt": "abc", "max_tokens": 3, "stream": True,
                                                       "stream_options": {"include_usage": True}}) as s:
            events = [ln[6:] for ln in s.iter_lines() if ln.startswith("data: ")]
        assert events[-1] == "[DONE]"
        usage = json.loads(events[-2])
        assert usage["choices"] == [] and usage["usage"]["completion_tokens"] == 3
        # streamed batch x n: per-choice token streams equal the non-streamed choices
        body = {"prompt": ["abc", "hello"], "max_tokens": 3, "n": 2, "temperature": 1.0, "seed": 9}
        want = [ch["token_ids"] for ch in c.post("/v1/completions", json=body).json()["choices"]]
        with c.stream("POST", "/v1/completions", json=dict(body, stream=True,
                                                           stream_options={"include_usage": True})) as s:
            events = [ln[6:] for ln in s.iter_lines() if ln.startswith("data: ")]
        assert events[-1] == "[DONE]"
        got, fins = {}, {}
        for e in events[:-2]:
            ch = json.loads(e)["choices"][0]
            got.setdefault(ch["index"], []).extend(ch.get("token_ids", []))
            if ch["finish_reason"]:
                fins[ch["index"]] = ch["finish_reason"]
        assert [got[j] for j in range(4)] == want and sorted(fins) == [0, 1, 2, 3]
        assert json.loads(events[-2])["usage"]["completion_tokens"] == 12
        assert c.post("/v1/completions", json={"prompt": ["a", ""]}).status_code == 400


def test_api_client_disconnect_aborts_request(tmp_path):
    """A streaming client that goes away mid-generation has its request
    aborted: it leaves the batch and its KV pages are freed, instead of
    generating to max_tokens for nobody. Runs a real HTTP server (the test
    client buffers whole responses) and drops the socket after the first
    event."""
    import socket
    import threading
    import uvicorn
    eng = make_engine(str(tmp_path))
    app = create_app(eng)
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    try:
        assert _wait(lambda: srv.started, 30)
        body = json.dumps({"prompt": "abc", "max_tokens": 400, "stream": True, "ignore_eos": True}).encode()
        conn = socket.create_connection(("127.0.0.1", port), timeout=30)
        conn.sendall(b"POST /v1/completions HTTP/1.1\r\nHost: x\r\nContent-Type: application/json\r\n"
                     + f"Content-Length: {len(body)}\r\n\r\n".encode() + body)
        buf = b""
        while b"data: " not in buf:
            chunk = conn.recv(4096)
            assert chunk, buf
            buf += chunk
        live = [r for r in list(eng.requests.values()) if not r.is_ft]
        assert len(live) == 1
        req = live[0]
        conn.close()
        assert _wait(lambda: req.status.name == "ABORTED", 30), (req.status, len(req.output_ids))
        assert len(req.output_ids) < 400
        assert req.request_id not in eng.requests
        assert _wait(lambda: all(r.is_ft for r in list(eng.scheduler.running) + list(eng.scheduler.waiting)), 30)
        assert app.state.serving_stats.finished.get("abort") == 1     # /metrics counts the abort
    finally:
        srv.should_exit = True
        th.join(30)


def test_api_top_logprobs(tmp_path):
    """logprobs=k (completions) / top_logprobs=k (chat) return the k most
    likely tokens of every position; under greedy decoding the chosen token
    is the first of them."""
    eng = make_engine(str(tmp_path))
    with TestClient(create_app(eng)) as c:
        out = c.post("/v1/completions", json={"prompt": "abc", "max_tokens": 3, "logprobs": 3}).json()
        lp = out["choices"][0]["logprobs"]
        assert len(lp["top_logprobs"]) == 3 and all(len(d) <= 3 for d in lp["top_logprobs"])
        for pos, tokstr in zip(lp["top_logprobs"], lp["tokens"]):
            best = max(pos.values())
            assert pos.get(tokstr) is not None and abs(pos[tokstr] - best) < 1e-4
            assert all(v <= 0.0 for v in pos.values())
        ch = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                  "max_tokens": 2, "logprobs": True, "top_logprobs": 2}).json()
        content = ch["choices"][0]["logprobs"]["content"]
        assert len(content) == 2 and all(len(x["top_logprobs"]) == 2 for x in content)
        assert c.post("/v1/completions", json={"prompt": "a", "logprobs": 21}).status_code == 400


def test_api_chat_without_max_tokens_runs_to_context_end(tmp_path):
    """A chat request with no max_tokens may generate until the context
    (max_model_len) is full, as in vLLM; completions keep OpenAI's 16."""
    eng = make_engine(str(tmp_path))
    with TestClient(create_app(eng)) as c:
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                 "ignore_eos": True}).json()
        assert r["usage"]["prompt_tokens"] + r["usage"]["completion_tokens"] == 512
        r = c.post("/v1/completions", json={"prompt": "hi", "ignore_eos": True}).json()
        assert r["usage"]["completion_tokens"] == 16
