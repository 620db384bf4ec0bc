"""HTTP API: the OpenAI-compatible completions endpoint plus the co-serving
control surface of the reference (``deltaserve-plugin/deltaserve/api.py:41-455``):

=======================================  ==============================================
``POST /v1/completions``                  OpenAI completions (``stream`` supported);
                                          ``model`` = base model, an adapter name, or
                                          the routing model name (``auto``)
``GET  /v1/models``, ``GET /health``
``POST /start_finetuning`` / ``stop``     open / close finetuning admission
``GET  /finetuning_status``               coordinator, trainer, store and job state
``POST /save_adapter``                    PEFT checkpoint of the trained adapter now
                                          (``{"path"?, "wait"?, "timeout_s"?}``)
``POST /save_estimator_state``            estimator coefficients + samples as JSON
``GET  /system_metrics``                  telemetry window + totals
``GET  /telemetry/data``                  live step stream / series (``steps_since``)
``POST /telemetry/start|stop|memory``     recorder on/off, memory snapshot
``POST /ft_jobs`` / ``GET /ft_jobs``      submit / list finetuning jobs
``GET  /adapters``, ``/adapters/available``  adapter pool
``POST /adapters``, ``POST /adapters/{name}/{op}``, ``DELETE /adapters/{name}``
``POST /shutdown``                        stop the engine loop
=======================================  ==============================================
"""

from __future__ import annotations

import asyncio
import contextlib
import json
import os
import time
import uuid

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, PlainTextResponse, Response, StreamingResponse

from ..adapters.routing.router import DISABLED, RouteDecision, extract_text
from ..engine.request import SamplingParams
from .engine_thread import EngineThread


def _json_body(body) -> dict:
    return body if isinstance(body, dict) else {}


def create_app(engine, served_model_name: str | None = None, tokenizer=None) -> FastAPI:
    et = EngineThread(engine)

    @contextlib.asynccontextmanager
    async def lifespan(_app):
        et.start()
        try:
            yield
        finally:
            await asyncio.to_thread(et.stop)

    app = FastAPI(title="DeltaServe-B200", lifespan=lifespan)
    app.state.engine_thread = et
    app.state.engine = engine
    app.state.server = None        # a uvicorn.Server, set by the launcher for /shutdown
    app.state.started_at = time.time()
    model_name = served_model_name or engine.ecfg.served_model_name or engine.ecfg.model
    tok = tokenizer or engine.tokenizer
    if tok is None:
        from ..utils.tokenizer import ByteTokenizer
        tok = ByteTokenizer(engine.arch.vocab)
    if engine.tokenizer is None:
        engine.tokenizer = tok        # stop strings are matched on decoded text
    route_name = engine.rcfg.route_model_name if engine.router is not None else None
    from .prom import ServingStats
    serving_stats = ServingStats()
    engine.request_listeners.append(serving_stats.on_request)
    app.state.serving_stats = serving_stats

    def _choice(index: int, r, chat: bool = False, echo: bool = False) -> dict:
        text = tok.decode(r.output_ids)
        if r.stop_reason:
            text = text[:text.find(r.stop_reason)] if r.stop_reason in text else text
        if echo:
            text = tok.decode(r.prompt_ids) + text
        if chat:
            c = {"index": index, "message": {"role": "assistant", "content": text},
                 "finish_reason": _finish_reason(r)}
            if r.params.logprobs:
                tops = r.output_top_logprobs
                c["logprobs"] = {"content": [
                    {"token": tok.decode([t]), "logprob": lp,
                     **({"top_logprobs": [{"token": tok.decode([a]), "logprob": b} for a, b in tops[j]]}
                        if j < len(tops) else {})}
                    for j, (t, lp) in enumerate(zip(r.output_ids, r.output_logprobs))]}
            return c
        c = {"index": index, "text": text, "token_ids": r.output_ids, "finish_reason": _finish_reason(r)}
        if r.params.logprobs:
            c["logprobs"] = {"tokens": [tok.decode([t]) for t in r.output_ids],
                             "token_logprobs": list(r.output_logprobs[:len(r.output_ids)])}
            if r.params.top_logprobs > 0:
                c["logprobs"]["top_logprobs"] = [{tok.decode([a]): b for a, b in pos}
                                                 for pos in r.output_top_logprobs[:len(r.output_ids)]]
        return c

    def _release(rid: str, w) -> None:
        """Forget a request's waiter; a request still running (the client went
        away: a cancelled handler or a closed stream) is aborted, so it stops
        taking batch slots and KV pages."""
        et.unregister(rid)
        if not w.done.done():
            et.submit(lambda e: e.abort_request(rid))

    async def _stream_many(prompts, params, n, model, chat, echo, include_usage):
        """Streamed ``n`` completions of each prompt of a batch: one event
        stream whose chunks carry the choice index (``p * n + i``), tokens in
        the order they are generated, a finish chunk per choice."""
        import dataclasses as _dc
        model_adapter = None if model == model_name else model
        if model_adapter is not None and model_adapter not in engine.adapter_slots:
            return JSONResponse(status_code=404, content={"error": f"unknown model {model!r}"})
        base_seed = params.seed if params.seed is not None else int(uuid.uuid4().int % (1 << 31))
        rids, waits = [], []
        for k, ids in enumerate(prompts):
            for i in range(n):
                rid = f"{'chatcmpl' if chat else 'cmpl'}-{uuid.uuid4().hex[:24]}"
                p = _dc.replace(params, seed=base_seed + k * n + i)
                waits.append(et.register(rid, True))
                rids.append(rid)
                try:
                    await et.call(lambda e, rid=rid, p=p, ids=ids: e.add_request(rid, ids, p, model_adapter))
                except Exception as ex:
                    for x, w in zip(rids, waits):
                        _release(x, w)
                    return JSONResponse(status_code=400, content={"error": str(ex)})
        et.notify_arrival()
        created = int(time.time())
        obj = ("chat.completion" if chat else "text_completion") + (".chunk" if chat else "")
        sid = rids[0]

        def event(choice):
            return f"data: {json.dumps({'id': sid, 'object': obj, 'created': created, 'model': model, 'choices': [choice]})}\n\n"

        async def gen():
            merged: asyncio.Queue = asyncio.Queue()

            async def pump(idx, w):
                while True:
                    toks = await w.tokens.get()
                    await merged.put((idx, toks))
                    if toks is None:
                        return
            tasks = [asyncio.create_task(pump(j, w)) for j, w in enumerate(waits)]
            try:
                if echo:
                    for j in range(len(waits)):
                        yield event({"index": j, "text": tok.decode(prompts[j // n]), "token_ids": [],
                                     "finish_reason": None})
                started, left = set(), len(waits)
                while left:
                    j, toks = await merged.get()
                    if toks is None:
                        r = await waits[j].done
                        left -= 1
                        yield event({"index": j, "delta": {}, "finish_reason": _finish_reason(r)} if chat else
                                    {"index": j, "text": "", "finish_reason": _finish_reason(r)})
                        continue
                    if chat:
                        delta = {"content": tok.decode(toks)}
                        if j not in started:
                            delta["role"] = "assistant"
                        ch = {"index": j, "delta": delta, "finish_reason": None}
                    else:
                        ch = {"index": j, "text": tok.decode(toks), "token_ids": toks, "finish_reason": None}
                    started.add(j)
                    yield event(ch)
                if include_usage:
                    reqs = [w.done.result() for w in waits]
                    npr = sum(len(ids) for ids in prompts)
                    ntok = sum(len(r.output_ids) for r in reqs)
                    use = {"id": sid, "object": obj, "created": created, "model": model, "choices": [],
                           "usage": {"prompt_tokens": npr, "completion_tokens": ntok, "total_tokens": npr + ntok}}
                    yield f"data: {json.dumps(use)}\n\n"
                yield "data: [DONE]\n\n"
            finally:
                for t in tasks:
                    t.cancel()
                for x, w in zip(rids, waits):
                    _release(x, w)
        return StreamingResponse(gen(), media_type="text/event-stream")

    async def _completions_n(body, prompts, params, n, model, chat=False, echo=False):
        """``n`` independent completions of each prompt of a batch (seeds seed,
        seed+1, ...); choice ``p * n + i`` is completion ``i`` of prompt ``p``."""
        import dataclasses as _dc
        model_adapter = None if model == model_name else model
        if model_adapter is not None and model_adapter not in engine.adapter_slots:
            return JSONResponse(status_code=404, content={"error": f"unknown model {model!r}"})
        base_seed = params.seed if params.seed is not None else int(uuid.uuid4().int % (1 << 31))
        rids, waits = [], []
        for k, ids in enumerate(prompts):
            for i in range(n):
                rid = f"cmpl-{uuid.uuid4().hex[:24]}"
                p = _dc.replace(params, seed=base_seed + k * n + i)
                waits.append(et.register(rid, False))
                rids.append(rid)
                try:
                    await et.call(lambda e, rid=rid, p=p, ids=ids: e.add_request(rid, ids, p, model_adapter))
                except Exception as e:
                    for x in rids:
                        et.unregister(x)
                    return JSONResponse(status_code=400, content={"error": str(e)})
        et.notify_arrival()
        try:
            reqs = [await w.done for w in waits]
        finally:
            for x, w in zip(rids, waits):
                _release(x, w)
        ntok = sum(len(r.output_ids) for r in reqs)
        nprompt = sum(len(ids) for ids in prompts)
        return JSONResponse(content={
            "id": rids[0], "object": "chat.completion" if chat else "text_completion",
            "created": int(time.time()), "model": model,
            "choices": [_choice(i, r, chat, echo) for i, r in enumerate(reqs)],
            "usage": {"prompt_tokens": nprompt, "completion_tokens": ntok, "total_tokens": nprompt + ntok}})

    async def body_of(req: Request) -> dict:
        try:
            return _json_body(await req.json())
        except Exception:
            return {}

    # ------------------------------------------------------------ inference
    @app.get("/health")
    async def health():
        ok = et.alive and et.error is None
        return JSONResponse(status_code=200 if ok else 503, content={"ok": ok, "error": et.error})

    @app.get("/v1/models")
    async def models():
        names = [model_name] + [n for n in engine.adapter_slots if not n.startswith("__")]
        if engine.router is not None:
            names += [n for n in engine.router.pool.names() if n not in names]
        if route_name:
            names.append(route_name)
        created = int(app.state.started_at)
        ml = engine.ecfg.max_model_len
        # adapters name the base model as their parent (as vLLM lists LoRA modules)
        return {"object": "list", "data": [
            {"id": n, "object": "model", "created": created, "owned_by": "deltaserve", "root": model_name,
             "parent": None if n == model_name else model_name, "max_model_len": ml} for n in names]}

    def _top_logprobs(body: dict) -> int:
        """Alternatives per position: ``top_logprobs`` (chat) or an integer
        ``logprobs`` (completions); at most 20."""
        k = body.get("top_logprobs")
        if k is None and not isinstance(body.get("logprobs"), bool):
            k = body.get("logprobs")
        k = int(k or 0)
        if not 0 <= k <= 20:
            raise ValueError("top_logprobs / logprobs must be in [0, 20]")
        return k

    def _parse_params(body: dict):
        """SamplingParams and n of an OpenAI request body (or an error response)."""
        stop = body.get("stop") or ()
        if isinstance(stop, str):
            stop = (stop,)
        try:
            n_choices = int(body.get("n", 1) or 1)
            max_tokens = body.get("max_tokens", body.get("max_completion_tokens", 16))
            params = SamplingParams(max_tokens=int(max_tokens if max_tokens is not None else 16),
                                    temperature=float(body.get("temperature", 0.0) or 0.0),
                                    seed=body.get("seed"), ignore_eos=bool(body.get("ignore_eos", False)),
                                    stop_token_ids=tuple(body.get("stop_token_ids") or ()),
                                    top_k=max(0, int(body.get("top_k", 0) or 0)),
                                    top_p=float(body.get("top_p", 1.0) if body.get("top_p") is not None else 1.0),
                                    logprobs=bool(body.get("logprobs") is not None and body.get("logprobs") is not False),
                                    top_logprobs=_top_logprobs(body),
                                    stop=tuple(str(x) for x in stop),
                                    presence_penalty=float(body.get("presence_penalty") or 0.0),
                                    frequency_penalty=float(body.get("frequency_penalty") or 0.0),
                                    repetition_penalty=float(1.0 if body.get("repetition_penalty") is None
                                                             else body["repetition_penalty"]),
                                    min_tokens=int(body.get("min_tokens") or 0),
                                    logit_bias=tuple(sorted((int(k), max(-100.0, min(100.0, float(v))))
                                                            for k, v in (body.get("logit_bias") or {}).items())))
        except (TypeError, ValueError, AttributeError) as e:
            return None, 0, JSONResponse(status_code=400, content={"error": f"bad sampling parameter: {e}"})
        if not (-2.0 <= params.presence_penalty <= 2.0 and -2.0 <= params.frequency_penalty <= 2.0):
            return None, 0, JSONResponse(status_code=400,
                                         content={"error": "presence_penalty / frequency_penalty must be in [-2, 2]"})
        if params.repetition_penalty <= 0.0:
            return None, 0, JSONResponse(status_code=400, content={"error": "repetition_penalty must be > 0"})
        if not 0 <= params.min_tokens <= params.max_tokens:
            return None, 0, JSONResponse(status_code=400, content={"error": "min_tokens must be in [0, max_tokens]"})
        if not 0.0 < params.top_p <= 1.0:
            return None, 0, JSONResponse(status_code=400, content={"error": "top_p must be in (0, 1]"})
        if n_choices < 1:
            return None, 0, JSONResponse(status_code=400, content={"error": "n must be >= 1"})
        return params, n_choices, None

    def _chat_prompt(messages) -> list[int]:
        """Token ids of a chat: the tokenizer's chat template when it has one,
        else a plain role-tagged transcript ending with the assistant turn."""
        apply = getattr(tok, "apply_chat_template", None)
        if apply is not None:
            try:
                out = apply(messages, add_generation_prompt=True, tokenize=True)
                if isinstance(out, dict):
                    out = out.get("input_ids")
                return [int(t) for t in out]
            except Exception:
                pass
        text = "".join(f"<|{m.get('role', 'user')}|>\n{m.get('content', '')}\n" for m in messages)
        return tok.encode(text + "<|assistant|>\n")

    async def _generate(body: dict, prompts: list[list[int]], chat: bool):
        params, n_choices, err = _parse_params(body)
        if err is not None:
            return err
        if chat and body.get("max_tokens") is None and body.get("max_completion_tokens") is None:
            # chat with no limit: up to the end of the context (as vLLM)
            import dataclasses as _dc
            room = engine.ecfg.max_model_len - max(len(p) for p in prompts)
            if room < 1:
                return JSONResponse(status_code=400, content={"error": "the prompt fills the context"})
            params = _dc.replace(params, max_tokens=room)
        model = body.get("model") or model_name
        stream = bool(body.get("stream", False))
        echo = bool(body.get("echo", False)) and not chat
        include_usage = bool((body.get("stream_options") or {}).get("include_usage", False))
        if n_choices > 1 or len(prompts) > 1:
            if stream:
                return await _stream_many(prompts, params, n_choices, model, chat, echo, include_usage)
            return await _completions_n(body, prompts, params, n_choices, model, chat, echo)
        ids = prompts[0]
        rid = f"{'chatcmpl' if chat else 'cmpl'}-{uuid.uuid4().hex[:24]}"
        router = engine.router
        headers = {}
        routed = named_pool = False
        adapter = None
        if model == engine.rcfg.route_model_name and router is None:
            # Routing is off: the base model serves it, and the headers say so.
            headers = RouteDecision(None, None, DISABLED).headers()
        elif model == engine.rcfg.route_model_name:
            routed = True
        elif model != model_name:
            if model in engine.adapter_slots:
                adapter = model
            elif router is not None and model in router.pool:
                named_pool = True
            else:
                return JSONResponse(status_code=404, content={"error": f"unknown model {model!r}"})
        w = et.register(rid, stream)
        et.notify_arrival()
        try:
            if routed or named_pool:
                text = extract_text(body) if routed else None
                fut = await et.call(lambda e: e.router.submit(rid, ids, params, text=text,
                                                              adapter=None if routed else model))
                decision = await asyncio.wrap_future(fut)
                if routed:
                    headers = decision.headers()
            else:
                await et.call(lambda e: e.add_request(rid, ids, params, adapter))
        except asyncio.CancelledError:       # the client went away before the route decision
            _release(rid, w)
            raise
        except Exception as e:
            et.unregister(rid)
            return JSONResponse(status_code=400, content={"error": str(e)})
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"
        if stream:
            async def gen():
                try:
                    first = True
                    if echo:
                        ch = {"index": 0, "text": tok.decode(ids), "token_ids": [], "finish_reason": None}
                        yield f"data: {json.dumps({'id': rid, 'object': obj, 'created': created, 'model': model, 'choices': [ch]})}\n\n"
                    while True:
                        toks = await w.tokens.get()
                        if toks is None:
                            break
                        if chat:
                            delta = {"content": tok.decode(toks)}
                            if first:
                                delta["role"] = "assistant"
                            ch = {"index": 0, "delta": delta, "finish_reason": None}
                        else:
                            ch = {"index": 0, "text": tok.decode(toks), "token_ids": toks, "finish_reason": None}
                        first = False
                        chunk = {"id": rid, "object": obj + (".chunk" if chat else ""), "created": created,
                                 "model": model, "choices": [ch]}
                        yield f"data: {json.dumps(chunk)}\n\n"
                    r = await w.done
                    last = ({"index": 0, "delta": {}, "finish_reason": _finish_reason(r)} if chat else
                            {"index": 0, "text": "", "finish_reason": _finish_reason(r)})
                    fin = {"id": rid, "object": obj + (".chunk" if chat else ""), "created": created,
                           "model": model, "choices": [last]}
                    yield f"data: {json.dumps(fin)}\n\n"
                    if include_usage:
                        use = {"id": rid, "object": obj + (".chunk" if chat else ""), "created": created,
                               "model": model, "choices": [],
                               "usage": {"prompt_tokens": r.num_prompt, "completion_tokens": len(r.output_ids),
                                         "total_tokens": r.num_prompt + len(r.output_ids)}}
                        yield f"data: {json.dumps(use)}\n\n"
                    yield "data: [DONE]\n\n"
                finally:
                    _release(rid, w)
            return StreamingResponse(gen(), media_type="text/event-stream", headers=headers)
        try:
            r = await w.done
        finally:
            _release(rid, w)
        out = {"id": rid, "object": obj, "created": created, "model": model,
               "choices": [_choice(0, r, chat, echo)],
               "usage": {"prompt_tokens": r.num_prompt, "completion_tokens": len(r.output_ids),
                         "total_tokens": r.num_prompt + len(r.output_ids)},
               "metrics": {"ttft_s": r.ttft(), "tbt_mean_s": (sum(r.tbts()) / len(r.tbts()))
                           if r.tbts() else None}}
        return JSONResponse(content=out, headers=headers)

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await body_of(req)
        prompt = body.get("prompt")
        if prompt is None:
            return JSONResponse(status_code=400, content={"error": "prompt is required"})
        # a string, a token-id list, or a batch of either
        try:
            if isinstance(prompt, list) and prompt and isinstance(prompt[0], int):
                prompts = [[int(t) for t in prompt]]
            elif isinstance(prompt, list):
                prompts = [[int(t) for t in p] if isinstance(p, list) else tok.encode(str(p)) for p in prompt]
            else:
                prompts = [tok.encode(str(prompt))]
        except (TypeError, ValueError) as ex:
            return JSONResponse(status_code=400, content={"error": f"bad prompt: {ex}"})
        if not prompts or any(not p for p in prompts):
            return JSONResponse(status_code=400, content={"error": "empty prompt"})
        return await _generate(body, prompts, chat=False)

    @app.post("/v1/chat/completions")
    async def chat_completions(req: Request):
        body = await body_of(req)
        messages = body.get("messages")
        if not isinstance(messages, list) or not messages:
            return JSONResponse(status_code=400, content={"error": "messages is required"})
        ids = _chat_prompt(messages)
        if not ids:
            return JSONResponse(status_code=400, content={"error": "empty prompt"})
        return await _generate(body, [ids], chat=True)

    # ------------------------------------------------------------ finetuning
    @app.post("/start_finetuning")
    async def start_finetuning():
        st = await et.call(lambda e: (e.start_finetuning(), e.finetuning_status())[1])
        return {"started": True, "status": st}

    @app.post("/stop_finetuning")
    async def stop_finetuning():
        st = await et.call(lambda e: (e.stop_finetuning(), e.finetuning_status())[1])
        return {"stopped": True, "status": st}

    @app.get("/finetuning_status")
    async def finetuning_status():
        return await et.call(lambda e: e.finetuning_status())

    @app.post("/save_adapter")
    async def save_adapter(req: Request):
        body = await body_of(req)
        path = body.get("path")
        if not path:
            root = engine.ftcfg.adapter_save_path
            if not root:
                return JSONResponse(status_code=400, content={
                    "error": "no path given and finetune_param.adapter_save_path is not set"})
            path = os.path.join(root, time.strftime("manual-%Y%m%d-%H%M%S"))
        path = os.path.abspath(str(path))
        save_id = uuid.uuid4().hex
        if engine.trainer is None:
            return JSONResponse(status_code=409, content={"error": "finetuning is not enabled", "path": path})
        # The engine thread gathers the tensors; the files are written in the
        # background and this handler polls the save handshake for them.
        fut = et.submit(lambda e: e.save_adapter(path, save_id, background=True))
        if not body.get("wait", True):
            return JSONResponse(status_code=202, content={"scheduled": True, "path": path, "save_id": save_id})
        timeout = float(body.get("timeout_s", 300))
        t0 = time.time()
        try:
            await asyncio.wait_for(asyncio.wrap_future(fut), timeout)
        except asyncio.TimeoutError:
            return JSONResponse(status_code=202, content={"pending": True, "path": path, "save_id": save_id})
        except Exception as ex:
            return JSONResponse(status_code=500, content={"path": path, "saved": False, "error": str(ex)})
        from ..adapters.peft_io import wait_save_result
        res = await asyncio.to_thread(wait_save_result, path, save_id, max(0.0, timeout - (time.time() - t0)))
        if res is None:
            return JSONResponse(status_code=202, content={"pending": True, "path": path, "save_id": save_id})
        if "error" in res:
            return JSONResponse(status_code=500, content={"path": path, "saved": False, **res})
        return {"path": path, "saved": True, **res}

    @app.post("/save_estimator_state")
    async def save_estimator_state(req: Request):
        body = await body_of(req)
        path = body.get("path") or engine.ftcfg.estimator_state_save_path
        if not path:
            return JSONResponse(status_code=400, content={"error": "no path (estimator_state_save_path unset)"})
        await et.call(lambda e: e.save_estimator_state(path))
        return {"saved": True, "path": path}

    # ------------------------------------------------------------ telemetry
    @app.get("/prefix_cache")
    async def prefix_cache():
        return await et.call(lambda e: dict(e.scheduler.cache_stats(), kv_usage=e.kv.allocator.usage()))

    @app.get("/system_metrics")
    async def system_metrics():
        m = getattr(engine, "metrics", None)
        if m is None:
            return JSONResponse(status_code=404, content={"error": "telemetry is off (metrics_dir unset)"})
        return await et.call(lambda e: e.metrics.snapshot())

    @app.get("/telemetry/data")
    async def telemetry_data(steps_since: int = 0):
        m = getattr(engine, "metrics", None)
        if m is None:
            return JSONResponse(status_code=404, content={"error": "telemetry is off"})
        return await et.call(lambda e: e.metrics.data(steps_since))

    @app.post("/telemetry/start")
    async def telemetry_start(req: Request):
        body = await body_of(req)
        d = body.get("metrics_dir") or engine.ftcfg.metrics_dir
        await et.call(lambda e: e.start_telemetry(d))
        return {"started": True, "metrics_dir": d}

    @app.post("/telemetry/stop")
    async def telemetry_stop():
        await et.call(lambda e: e.stop_telemetry())
        return {"stopped": True}

    @app.post("/telemetry/memory")
    async def telemetry_memory(req: Request):
        body = await body_of(req)
        m = getattr(engine, "metrics", None)
        if m is None:
            return JSONResponse(status_code=404, content={"error": "telemetry is off"})
        return await et.call(lambda e: e.metrics.memory_snapshot(body.get("dir")))

    # ------------------------------------------------------------ jobs
    @app.post("/ft_jobs")
    async def submit_job(req: Request):
        body = await body_of(req)
        from ..engine.ft_job import FinetuneJobSpec
        known = set(FinetuneJobSpec.__dataclass_fields__)
        bad = sorted(set(body) - known)
        if bad:
            return JSONResponse(status_code=400, content={"error": f"unknown job key(s) {bad}"})
        try:
            spec = FinetuneJobSpec(**{**body, "stages": tuple(body.get("stages", ("init", "training")))})
            job = await et.call(lambda e: e.jobs.submit(spec, e.rcfg.enable_adapter_routing))
        except Exception as ex:
            return JSONResponse(status_code=400, content={"error": str(ex)})
        return job.status()

    @app.get("/ft_jobs")
    async def list_jobs():
        return {"jobs": await et.call(lambda e: e.jobs.status())}

    # ------------------------------------------------------------ adapters
    @app.get("/adapters")
    async def adapters():
        def info(e):
            out = [{"name": n, "slot": s, **{k: v for k, v in e.adapter_meta.get(n, {}).items()}}
                   for n, s in e.adapter_slots.items()]
            router = getattr(e, "router", None)
            return {"loaded": out, "pool": router.pool.status() if router is not None else None}
        return await et.call(info)

    @app.get("/adapters/available")
    async def adapters_available():
        def avail(e):
            names = [n for n in e.adapter_slots if not n.startswith("__")]
            router = getattr(e, "router", None)
            if router is not None:
                names = sorted(set(names) | set(router.pool.names()))
            return {"by_name": names, "routed_model": route_name}
        return await et.call(avail)

    @app.post("/adapters")
    async def add_adapter(req: Request):
        body = await body_of(req)
        if not body.get("path"):
            return JSONResponse(status_code=400, content={"error": "JSON body with 'path' required"})
        name = body.get("name") or os.path.basename(os.path.normpath(body["path"]))
        try:
            def add(e):
                router = getattr(e, "router", None)
                if router is not None:
                    return router.add(name, body["path"], data_path=body.get("data_path"),
                                           centroid_path=body.get("centroid_path"),
                                           prewarm=bool(body.get("prewarm", False)))
                return {"slot": e.load_inference_adapter(name, path=body["path"])}
            res = await et.call(add)
        except Exception as ex:
            return JSONResponse(status_code=400, content={"error": str(ex)})
        return {"name": name, "result": res}

    @app.post("/adapters/{name}/{op}")
    async def adapter_op(name: str, op: str):
        try:
            res = await et.call(lambda e: e.adapter_op(name, op))
        except Exception as ex:
            return JSONResponse(status_code=400, content={"error": str(ex)})
        return {"name": name, "op": op, "result": res}

    @app.delete("/adapters/{name}")
    async def remove_adapter(name: str):
        try:
            res = await et.call(lambda e: e.adapter_op(name, "remove"))
        except Exception as ex:
            return JSONResponse(status_code=400, content={"error": str(ex)})
        return {"name": name, "removed": True, "result": res}

    # ------------------------------------------------------------ vLLM-compatible extras
    @app.get("/metrics")
    async def metrics():
        from .prom import render
        return PlainTextResponse(render(serving_stats, engine, model_name),
                                 media_type="text/plain; version=0.0.4; charset=utf-8")

    @app.get("/version")
    async def version():
        from .. import __version__
        return {"version": __version__}

    @app.get("/ping")
    @app.post("/ping")
    async def ping():
        return Response(status_code=200 if (et.alive and et.error is None) else 503)

    @app.post("/tokenize")
    async def tokenize(req: Request):
        body = await body_of(req)
        if body.get("messages") is not None:
            ids = _chat_prompt(body["messages"])
        elif isinstance(body.get("prompt"), str):
            ids = tok.encode(body["prompt"])
        else:
            return JSONResponse(status_code=400, content={"error": "JSON body with 'prompt' or 'messages' required"})
        return {"count": len(ids), "max_model_len": engine.ecfg.max_model_len, "tokens": ids}

    @app.post("/detokenize")
    async def detokenize(req: Request):
        body = await body_of(req)
        ids = body.get("tokens")
        if not isinstance(ids, list):
            return JSONResponse(status_code=400, content={"error": "JSON body with 'tokens' required"})
        try:
            return {"prompt": tok.decode([int(t) for t in ids])}
        except (TypeError, ValueError) as ex:
            return JSONResponse(status_code=400, content={"error": str(ex)})

    @app.post("/v1/load_lora_adapter")
    async def load_lora_adapter(req: Request):
        """vLLM's runtime LoRA loading: ``{"lora_name", "lora_path"}``; the
        adapter then serves requests whose ``model`` is its name."""
        body = await body_of(req)
        name, path = body.get("lora_name"), body.get("lora_path")
        if not name or not path:
            return PlainTextResponse("'lora_name' and 'lora_path' are required", status_code=400)
        if name in engine.adapter_slots:
            return PlainTextResponse(f"The lora adapter '{name}' has already been loaded.", status_code=400)
        try:
            await et.call(lambda e: e.load_inference_adapter(name, path=path))
        except Exception as ex:
            return PlainTextResponse(f"Failed to load LoRA adapter '{name}': {ex}", status_code=400)
        return PlainTextResponse(f"Success: LoRA adapter '{name}' added successfully.")

    @app.post("/v1/unload_lora_adapter")
    async def unload_lora_adapter(req: Request):
        body = await body_of(req)
        name = body.get("lora_name")
        if not name:
            return PlainTextResponse("'lora_name' is required", status_code=400)
        if name not in engine.adapter_slots or name.startswith("__"):
            return PlainTextResponse(f"The lora adapter '{name}' cannot be found.", status_code=404)
        try:
            await et.call(lambda e: e.unload_inference_adapter(name))
        except Exception as ex:
            return PlainTextResponse(f"Failed to unload LoRA adapter '{name}': {ex}", status_code=400)
        return PlainTextResponse(f"Success: LoRA adapter '{name}' removed successfully.")

    # ------------------------------------------------------------ lifecycle
    @app.post("/shutdown")
    async def shutdown():
        await et.call(lambda e: e._drain_backward())
        await asyncio.to_thread(et.stop)
        srv = app.state.server
        if srv is not None:
            srv.should_exit = True
        return {"shutdown": True}

    return app


def _finish_reason(r) -> str:
    if r.status.name == "ABORTED":
        return "abort"
    if getattr(r, "stop_reason", None):
        return "stop"
    return "length" if len(r.output_ids) >= r.params.max_tokens else "stop"
