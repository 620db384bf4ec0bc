"""Sampling penalties (presence / frequency / repetition), logit_bias and
min_tokens: the logit adjustments against a plain restatement of their
definitions, and their effect through the engine and the HTTP API."""
import torch
from fastapi.testclient import TestClient

from deltaserve_vllm_b200.engine.penalties import apply_penalties
from deltaserve_vllm_b200.engine.request import Request, SamplingParams


def _ref(row, prompt, out, p, eos):
    row = row.clone()
    for t in set(out):
        c = out.count(t)
        row[t] -= p.frequency_penalty * c + p.presence_penalty
    if p.repetition_penalty != 1.0:
        for t in set(prompt) | set(out):
            row[t] = row[t] / p.repetition_penalty if row[t] > 0 else row[t] * p.repetition_penalty
    for t, b in p.logit_bias:
        row[t] += b
    if len(out) < p.min_tokens:
        for t in set(p.stop_token_ids) | (set() if p.ignore_eos else set(eos)):
            row[t] = float("-inf")
    return row


def test_penalty_math_matches_definitions():
    g = torch.Generator().manual_seed(0)
    V = 50
    cases = [
        SamplingParams(presence_penalty=0.5, frequency_penalty=0.25),
        SamplingParams(repetition_penalty=1.3),
        SamplingParams(repetition_penalty=0.7, presence_penalty=-0.4),
        SamplingParams(logit_bias=((3, 5.0), (7, -100.0))),
        SamplingParams(min_tokens=6, ignore_eos=False, stop_token_ids=(11,)),
        SamplingParams(min_tokens=6, ignore_eos=True, stop_token_ids=(11,)),
        SamplingParams(min_tokens=2, ignore_eos=False),              # already past min_tokens
        SamplingParams(),                                            # untouched row
    ]
    reqs = []
    for i, p in enumerate(cases):
        r = Request(f"r{i}", torch.randint(0, V, (6,), generator=g).tolist(), p)
        r.output_ids = torch.randint(0, V, (4,), generator=g).tolist() + [r.prompt_ids[0]] * 2
        reqs.append(r)
    logits = torch.randn(len(reqs), V, generator=g)
    want = torch.stack([_ref(logits[i], r.prompt_ids, r.output_ids, r.params, (2,))
                        for i, r in enumerate(reqs)])
    got = logits.clone()
    apply_penalties(got, reqs, eos_ids=(2,))
    assert torch.equal(torch.isinf(got), torch.isinf(want))
    fin = ~torch.isinf(want)
    assert torch.allclose(got[fin], want[fin], atol=1e-6)
    assert torch.equal(got[-1], logits[-1])
    assert not SamplingParams().has_penalties and SamplingParams(min_tokens=1).needs_full_sampler


def _engine(tmp):
    from test_engine_cpu import make_engine
    return make_engine(tmp, start_on_launch=False)


def test_engine_logit_bias_and_min_tokens(tmp_path):
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

    class Tok:
        eos_token_id = None

    eng = _engine(str(tmp_path))
    eng.tokenizer = Tok()
    # a large bias makes greedy decoding pick that token every step
    eng.add_request("bias", [5, 6, 7], SamplingParams(max_tokens=5, logit_bias=((42, 100.0),)))
    eng.add_request("plain", [5, 6, 7], SamplingParams(max_tokens=8, ignore_eos=True))
    eng.run_until_idle(max_steps=200)
    got = {r.request_id: r.output_ids for r in eng.finished[-2:]}
    assert got["bias"] == [42] * 5
    full = got["plain"]
    # min_tokens: the end-of-sequence id cannot end the request early
    tok = Tok()
    tok.eos_token_id = full[0]
    eng.tokenizer = tok
    eng.add_request("min", [5, 6, 7], SamplingParams(max_tokens=8, min_tokens=4, ignore_eos=False))
    eng.add_request("nomin", [5, 6, 7], SamplingParams(max_tokens=8, ignore_eos=False))
    eng.run_until_idle(max_steps=200)
    got = {r.request_id: r.output_ids for r in eng.finished[-2:]}
    assert got["nomin"] == [full[0]]                          # ends on its first token
    assert len(got["min"]) >= 4 and full[0] not in got["min"][:4]
    assert eng.kv.allocator.num_free == eng.kv.allocator.num_blocks


def test_api_penalty_options(tmp_path):
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_server_cpu import make_engine
    from deltaserve_vllm_b200.server.api import create_app
    eng = make_engine(str(tmp_path))
    with TestClient(create_app(eng)) as c:
        r = c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 4, "logit_bias": {"77": 100},
                                            "presence_penalty": 0.5, "frequency_penalty": 0.5,
                                            "repetition_penalty": 1.2, "min_tokens": 2})
        assert r.status_code == 200, r.text
        assert r.json()["choices"][0]["token_ids"] == [77] * 4
        for bad in ({"presence_penalty": 3}, {"repetition_penalty": 0}, {"min_tokens": 9},
                    {"logit_bias": {"x": 1}}):
            r = c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 4, **bad})
            assert r.status_code == 400, (bad, r.text)
