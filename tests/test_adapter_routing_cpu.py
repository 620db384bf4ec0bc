"""Adapter routing on CPU: centroid index and resumable indexing, the
confidence-gated decision, the pool's tiers / eviction / admission with a fake
backend, and the engine-integrated router (encode step, held requests, slot
placement) behind the HTTP ``model: "auto"`` path. Mirrors the reference's
``tests/test_adapter_{decision,pool,indexing,engine,route_path}.py`` with this
package's own fixtures (the pool is tested against a fake LoRA backend, as
the reference's pool docstring prescribes)."""
import os
import tempfile

import numpy as np
import pytest

from deltaserve_vllm_b200.adapters.routing.decision import CENTRED, RAW, UNGATED, PoolGeometry, admission_report
from deltaserve_vllm_b200.adapters.routing.encoder import HashingEncoder
from deltaserve_vllm_b200.adapters.routing.index import CentroidIndex, Indexer, fingerprint, l2_normalize, select_samples
from deltaserve_vllm_b200.adapters.routing.pool import ACTIVE, CPU, DISK, GPU, RETIRED, AdapterPool, PoolFull, read_registry
from deltaserve_vllm_b200.adapters.routing.router import BELOW_THRESHOLD, LOW_CONFIDENCE, NO_ADAPTERS, NO_TEXT, Router, extract_text


def _clusters(n_adapters=6, dim=32, per=40, spread=0.15, seed=0):
    rng = np.random.default_rng(seed)
    centres = l2_normalize(rng.normal(size=(n_adapters, dim)))
    samples = {f"a{i}": l2_normalize(centres[i] + spread * rng.normal(size=(per, dim)))
               for i in range(n_adapters)}
    return centres, samples


def _index(samples, n_ref=16):
    idx = CentroidIndex("test", "", 0)
    for n, S in samples.items():
        idx.add(n, S.mean(0), refs=S[:n_ref])
    return idx


# ---------------------------------------------------------------- index
def test_indexer_resumes_and_matches_mean():
    rng = np.random.default_rng(1)
    texts = [f"t{i}" for i in range(37)]
    emb = rng.normal(size=(37, 8))
    with tempfile.TemporaryDirectory() as d:
        ck = os.path.join(d, "ck.npz")
        ix = Indexer(texts, "fp", ck, reference_samples=5)
        s, chunk = ix.next_chunk(10)
        assert (s, len(chunk)) == (0, 10)
        assert ix.commit(0, emb[:10])
        assert not ix.commit(0, emb[:10])          # stale chunk refused
        ix2 = Indexer(texts, "fp", ck, reference_samples=5)   # restart resumes
        assert ix2.resumed_from == 10
        while not ix2.done:
            s, chunk = ix2.next_chunk(7)
            ix2.commit(s, emb[s:s + len(chunk)])
        want = l2_normalize(l2_normalize(emb).mean(0))
        np.testing.assert_allclose(ix2.centroid(), want, rtol=1e-5, atol=1e-6)
        assert ix2.references().shape == (5, 8)
        assert Indexer(texts, "other-fp", ck, 5).resumed_from == 0   # another dataset
        idx = CentroidIndex("enc", "q: ", 64)
        idx.add("x", ix2.centroid(), refs=ix2.references())
        idx.save(os.path.join(d, "c.npz"))
        back = CentroidIndex.load(os.path.join(d, "c.npz"))
        assert back.names == ["x"] and back.encoder == "enc" and back.refs["x"].shape == (5, 8)


def test_select_samples_and_fingerprint():
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "data.txt")
        with open(p, "w") as f:
            f.write("q1 ### Response: a1\n\nq2 ### Response: a2\nq3\n")
        t = select_samples(p, 10, input_until="### Response:")
        assert t == ["q1", "q2", "q3"]
        assert len(select_samples(p, 2)) == 2
        assert fingerprint(t, "e", "p", 1) != fingerprint(t, "e", "p", 2)


# ---------------------------------------------------------------- decision
def test_decision_centred_routes_and_gates():
    centres, samples = _clusters()
    idx = _index(samples)
    m = PoolGeometry(idx, keep_percent=90, close_band=0.0, min_pool=4)
    assert m.mode == CENTRED and m.threshold is not None
    # typical requests (near a cluster's centre) route to their adapter
    hits = sum(m.decide(samples[n][-8:].mean(0)).adapter == n for n in samples)
    assert hits == len(samples)
    # the top candidate is right for individual samples even when gated
    assert sum(m.decide(samples[n][-1]).shortlist[0] == n for n in samples) == len(samples)
    # a request unlike every adapter falls back with low confidence
    far = -centres.mean(0)
    c = m.decide(far)
    assert c.adapter is None and c.below_gate
    # keep_percent 100 disables the gate
    assert PoolGeometry(idx, keep_percent=100).threshold is None


def test_decision_small_pool_raw_and_ungated():
    _, samples = _clusters(n_adapters=2)
    idx = _index(samples)
    assert PoolGeometry(idx, min_pool=4).mode == RAW
    bare = CentroidIndex()
    for n, S in samples.items():
        bare.add(n, S.mean(0))
    m = PoolGeometry(bare)
    assert m.mode == UNGATED and m.decide(samples["a1"][0]).adapter == "a1"


def test_decision_close_band_prefers():
    idx = CentroidIndex()
    base = l2_normalize(np.ones(8))
    idx.add("x", base)
    idx.add("y", base + 1e-4)
    m = PoolGeometry(idx, close_band=0.5, min_pool=99)
    assert m.decide(base, prefer=lambda n: n == "y").adapter in ("x", "y")


def test_admission_report_detects_duplicates():
    _, samples = _clusters()
    idx = _index(samples)
    dup = samples["a2"][16:]              # the same task, other samples
    rep = admission_report(idx, "dup", dup.mean(0), dup[:16])
    assert rep["nearest"] == "a2" and rep["stolen_from"] == "a2" and rep["stolen_max"] > 0
    assert rep["nearest_cosine"] > 0.9
    _, other = _clusters(n_adapters=1, seed=99)
    new = other["a0"]
    rep2 = admission_report(idx, "new", new.mean(0), new[:16])
    assert rep2["self_recall"] == 1.0 and rep2["stolen_max"] == 0.0
    assert rep["self_recall"] < rep2["self_recall"]


# ---------------------------------------------------------------- pool
class FakeBackend:
    def __init__(self):
        self.calls = []

    def load(self, e):
        self.calls.append(("load", e.name))

    def activate(self, e):
        self.calls.append(("activate", e.name))

    def deactivate(self, e):
        self.calls.append(("deactivate", e.name))

    def unload(self, e):
        self.calls.append(("unload", e.name))


class Clock:
    t = 0.0

    def __call__(self):
        return self.t


def test_pool_tiers_eviction_and_protection():
    clk = Clock()
    be = FakeBackend()
    pool = AdapterPool(be, capacity=8, gpu_slots=2, protected=1, half_life_s=10, clock=clk, grace_s=0)
    for n in "abc":
        pool.register(n, f"/p/{n}", prewarm=True)
    assert [pool.entries[n].tier for n in "abc"] == [GPU, GPU, CPU]    # prewarm never evicts
    for _ in range(3):
        pool.note_hit("a")
    clk.t = 1.0
    pool.note_hit("c")                     # evicts b (a is protected and hotter)
    assert pool.entries["c"].tier == GPU and pool.entries["b"].tier == CPU and pool.evictions == 1
    # in-use adapters are never evicted
    assert not pool.ensure_gpu("b", in_use={"c"})
    pool.offload("b")
    assert pool.entries["b"].tier == DISK
    pool.note_hit("b", place=False)
    assert pool.cold_loads == 1
    with pytest.raises(ValueError):
        pool.op("a", "explode")


def test_pool_admission_full_and_persistence():
    clk = Clock()
    _, samples = _clusters()
    with tempfile.TemporaryDirectory() as d:
        pool = AdapterPool(FakeBackend(), capacity=3, gpu_slots=1, clock=clk, directory=d, grace_s=5,
                           min_pool=2)
        for n in ["a0", "a1", "a2"]:
            rep = pool.admit(n, f"/p/{n}", samples[n].mean(0), samples[n][:16])
            assert rep["level"] == ACTIVE
        clk.t = 1.0
        rep = pool.admit("a3", "/p/a3", samples["a3"].mean(0), samples["a3"][:16])
        assert rep["level"] == RETIRED            # everybody within the grace period
        clk.t = 100.0
        pool.note_hit("a0")
        pool.note_hit("a1")
        rep = pool.admit("a4", "/p/a4", samples["a4"].mean(0), samples["a4"][:16])
        assert rep["level"] == ACTIVE and rep["retired"] == "a2"
        pool.pin("a4")
        reg = read_registry(d)
        assert {a["name"] for a in reg["adapters"]} == {"a0", "a1", "a2", "a3", "a4"}
        assert os.path.exists(os.path.join(d, reg["index_file"]))
        # restore into a new pool: levels, pins and routable set survive
        p2 = AdapterPool(FakeBackend(), capacity=3, gpu_slots=1, clock=clk, directory=d)
        assert p2.restore(d) == 5
        assert sorted(p2.routable_names()) == ["a0", "a1", "a4"]
        assert p2.entries["a4"].pinned and p2.entries["a2"].level == RETIRED
        strict = AdapterPool(FakeBackend(), capacity=1, gpu_slots=1, when_full="reject", clock=clk)
        strict.admit("x", "/x", samples["a0"].mean(0))
        with pytest.raises(PoolFull):
            strict.admit("y", "/y", samples["a1"].mean(0))


# ---------------------------------------------------------------- router
def test_router_outcomes_and_headers():
    enc = HashingEncoder(dim=256)
    r = Router(enc, keep_percent=100)
    assert r.route("hello").reason == NO_ADAPTERS
    topics = {"cooking": ["bake the bread with flour and yeast", "roast the chicken in the oven",
                          "whisk eggs and sugar for the cake"],
              "finance": ["the stock market fell on interest rates", "bond yields and inflation data",
                          "quarterly earnings beat analyst estimates"]}
    idx = CentroidIndex(enc.name)
    for n, texts in topics.items():
        E = enc.encode(texts)
        idx.add(n, E.mean(0), refs=E)
    r.set_index(idx)
    d = r.route("how long to bake bread with yeast")
    assert d.adapter == "cooking" and d.headers()["x-deltaserve-adapter"] == "cooking"
    assert r.route("   ").reason == NO_TEXT
    assert r.route_many(["bond yields rise", ""])[0].adapter == "finance"
    h = r.route("").headers()
    assert h["x-deltaserve-routing"] == "fallback" and "x-deltaserve-routing-message" in h
    assert extract_text({"messages": [{"role": "user", "content": "hi"}]}) == "hi"
    assert extract_text({"prompt": [1, 2]}) is None


def test_hashing_encoder_deterministic_unit_norm():
    a = HashingEncoder(dim=64).encode(["alpha beta gamma", ""])
    b = HashingEncoder(dim=64).encode(["alpha beta gamma", ""])
    np.testing.assert_array_equal(a, b)
    assert abs(np.linalg.norm(a[0]) - 1) < 1e-5 and np.linalg.norm(a[1]) == 0


# ---------------------------------------------------------------- engine + HTTP
TOPICS = {
    "cooking": ["bake the bread with flour and yeast", "roast the chicken in a hot oven",
                "whisk the eggs and sugar for the sponge cake", "simmer the tomato sauce with basil"],
    "finance": ["the stock market fell as interest rates rose", "bond yields climbed on inflation data",
                "quarterly earnings beat analyst estimates", "the central bank held rates steady"],
    "sports": ["the striker scored twice in the second half", "the team won the championship final",
               "the pitcher threw a perfect game", "the marathon runner set a new record"],
    "code": ["the python function returns a sorted list", "compile the rust crate with cargo",
             "the compiler reports a type error in main", "write a unit test for the parser"],
}


def _routing_engine(tmp, slots=2, encoder=None):
    import torch
    from deltaserve_vllm_b200.adapters import peft_io
    from deltaserve_vllm_b200.adapters.routing import AdapterRouter
    from deltaserve_vllm_b200.config import AdapterRoutingConfig, EngineConfig, FinetuneConfig
    from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
    from deltaserve_vllm_b200.models.configs import resolve_arch
    from deltaserve_vllm_b200.models.lora import random_adapter
    from deltaserve_vllm_b200.utils.tokenizer import ByteTokenizer
    arch = resolve_arch("qwen3-tiny")
    entries = []
    for i, (name, texts) in enumerate(TOPICS.items()):
        ad = os.path.join(tmp, "adapters", name)
        t = random_adapter(arch, 8, seed=100 + i)
        peft_io.write_peft_adapter(ad, t, peft_io.default_adapter_config(8, 16.0, ["q", "k", "v", "o", "gate", "up", "down"]), {"save_id": name})
        data = os.path.join(tmp, f"{name}.txt")
        with open(data, "w") as f:
            f.write("\n".join(texts * 3) + "\n")
        entries.append({"name": name, "path": ad, "data_path": data})
    ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=512, block_size=16,
                        max_num_batched_tokens=256, max_loras=slots, max_lora_rank=8)
    rcfg = AdapterRoutingConfig(enable_adapter_routing=True, index_path=os.path.join(tmp, "index"),
                                adapters=entries, route_min_pool=2, route_keep_percent=100.0,
                                route_reference_samples=8, indexing_chunk_samples=4,
                                **({"encoder": encoder, "encoder_query_prefix": "query: "} if encoder else {}))
    eng = CoServingEngine(ecfg, FinetuneConfig(enable_finetuning=False), rcfg,
                          tokenizer=ByteTokenizer(arch.vocab))
    eng.router = AdapterRouter(eng, rcfg)
    return eng


def test_routing_engine_http_auto():
    import time
    from fastapi.testclient import TestClient
    from deltaserve_vllm_b200.server.api import create_app
    with tempfile.TemporaryDirectory() as tmp:
        eng = _routing_engine(tmp, slots=2)
        t0 = time.time()
        while eng.router.indexing and time.time() - t0 < 60:
            eng.router.tick()
            time.sleep(0.01)
        assert sorted(eng.router.pool.routable_names()) == sorted(TOPICS)
        with TestClient(create_app(eng)) as c:
            models = [m["id"] for m in c.get("/v1/models").json()["data"]]
            assert "auto" in models and "cooking" in models
            seen = {}
            for name, q in [("cooking", "bake bread with yeast and flour"),
                            ("finance", "bond yields and interest rates"),
                            ("sports", "the striker scored in the final"),
                            ("code", "the python function returns a list"),
                            ("cooking", "roast the chicken in the oven")]:
                r = c.post("/v1/completions", json={"model": "auto", "prompt": q, "max_tokens": 3})
                assert r.status_code == 200, r.text
                assert r.headers["x-deltaserve-routing"] == "routed"
                seen[q] = r.headers["x-deltaserve-adapter"]
                assert seen[q] == name, (q, seen[q])
                assert len(r.json()["choices"][0]["token_ids"]) == 3
            st = c.get("/adapters").json()["pool"]
            assert st["evictions"] >= 2 and st["gpu_slots"] == 2
            # a pool adapter by name (cold: held until it gets a slot)
            r = c.post("/v1/completions", json={"model": "finance", "prompt": "x", "max_tokens": 2})
            assert r.status_code == 200 and "x-deltaserve-routing" not in r.headers
            # retire: no longer routable, still servable by name
            assert c.post("/adapters/sports/retire").status_code == 200
            r = c.post("/v1/completions", json={"model": "auto", "prompt": "the striker scored",
                                                "max_tokens": 2})
            assert r.headers.get("x-deltaserve-adapter") != "sports"
            assert c.post("/v1/completions", json={"model": "sports", "prompt": "x",
                                                   "max_tokens": 2}).status_code == 200
            r = c.post("/v1/completions", json={"model": "auto", "prompt": [5, 6], "max_tokens": 2})
            assert r.headers["x-deltaserve-routing-reason"] == "no-text"
        # slots never over-committed; every request finished
        assert len(eng.adapter_slots) <= 2
        assert not eng.has_unfinished()


def test_routing_disabled_auto_serves_base_model():
    from fastapi.testclient import TestClient
    from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
    from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
    from deltaserve_vllm_b200.server.api import create_app
    eng = CoServingEngine(EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=256, block_size=16,
                                       max_num_batched_tokens=128, max_loras=1, max_lora_rank=8),
                          FinetuneConfig(enable_finetuning=False))
    with TestClient(create_app(eng)) as c:
        r = c.post("/v1/completions", json={"model": "auto", "prompt": "hi", "max_tokens": 2})
        assert r.status_code == 200
        assert r.headers["x-deltaserve-routing-reason"] == "adapter-routing-disabled"


def test_job_switch_with_indexing_and_admission_stages():
    """A second finetuning job (own corpus, stages init -> training ->
    indexing -> admission) runs after the launch job: the trainer switches
    corpus and adapter, indexes the corpus, saves the trained adapter and
    admits it to the routing pool, where ``auto`` requests then find it."""
    import time
    from fastapi.testclient import TestClient
    from deltaserve_vllm_b200.adapters.routing import AdapterRouter
    from deltaserve_vllm_b200.config import AdapterRoutingConfig, EngineConfig, FinetuneConfig
    from deltaserve_vllm_b200.engine.ft.store import FinetuningStore
    from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
    from deltaserve_vllm_b200.server.api import create_app
    from deltaserve_vllm_b200.utils.tokenizer import ByteTokenizer
    with tempfile.TemporaryDirectory() as tmp:
        data = os.path.join(tmp, "sports.txt")
        with open(data, "w") as f:
            f.write("\n".join(TOPICS["sports"] * 2) + "\n")
        ecfg = EngineConfig(model="qwen3-tiny", device="cpu", max_model_len=512, block_size=16,
                            max_num_batched_tokens=256, max_loras=3, max_lora_rank=8)
        fcfg = FinetuneConfig(enable_finetuning=True, max_saved_finetuning_tokens=128, learning_rate=1e-3,
                              adapter_save_path=os.path.join(tmp, "ckpt"))
        rcfg = AdapterRoutingConfig(enable_adapter_routing=True, index_path=os.path.join(tmp, "index"),
                                    route_min_pool=2, route_keep_percent=100.0)
        store = FinetuningStore.synthetic(1024, 6, 16, 30, seed=0, max_saved_finetuning_tokens=128,
                                          total_epochs=1)
        eng = CoServingEngine(ecfg, fcfg, rcfg, ft_store=store, tokenizer=ByteTokenizer(1024))
        eng.router = AdapterRouter(eng, rcfg)
        with TestClient(create_app(eng)) as c:
            r = c.post("/ft_jobs", json={"name": "sports-ft", "data_path": data, "num_epochs": 1,
                                         "learning_rate": 2e-3, "stages": ["init", "training", "indexing",
                                                                           "admission"]})
            assert r.status_code == 200, r.text
            t0 = time.time()
            while time.time() - t0 < 120:
                jobs = {j["name"]: j for j in c.get("/ft_jobs").json()["jobs"]}
                if jobs["sports-ft"]["state"] in ("done", "failed"):
                    break
                time.sleep(0.05)
            assert jobs["sports-ft"]["state"] == "done", jobs
            assert jobs["default"]["state"] == "done"
            assert "sports-ft" in eng.router.pool.routable_names()
            assert eng.trainer.lr == 2e-3
            r = c.post("/v1/completions", json={"model": "auto", "prompt": "the striker scored a goal",
                                                "max_tokens": 2})
            assert r.headers["x-deltaserve-adapter"] == "sports-ft"


def test_router_cancel_drops_pending_request(tmp_path):
    """Aborting a routed request that still waits for its decision removes it
    from the router's queue (its future is cancelled; nothing is scheduled)."""
    from deltaserve_vllm_b200.engine.request import SamplingParams
    eng = _routing_engine(str(tmp_path), slots=2)
    fut = eng.router.submit("gone", [5, 6, 7], SamplingParams(max_tokens=4), text="bake bread")
    keep = eng.router.submit("kept", [5, 6, 7], SamplingParams(max_tokens=4), text="bond yields")
    assert eng.abort_request("gone")
    assert fut.cancelled() and not keep.done()
    assert [p[0] for p in eng.router.pending] == ["kept"]
    assert not eng.abort_request("gone")


def test_routing_with_a_sentence_encoder_directory():
    """The Hugging Face encoder path end to end on CPU: a local encoder
    directory (a random 2-layer BERT whose vocabulary covers the topics)
    selects SentenceEncoder; indexing runs it in the CPU encoder process;
    a request carrying one of a topic's own samples routes to that topic."""
    import time
    import torch
    from transformers import BertConfig, BertModel, BertTokenizerFast
    from deltaserve_vllm_b200.adapters.routing.encoder import SentenceEncoder
    with tempfile.TemporaryDirectory() as tmp:
        enc_dir = os.path.join(tmp, "encoder")
        words = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]", "query", ":"]
        for texts in TOPICS.values():
            for t in texts:
                words += [w for w in t.split() if w not in words]
        BertTokenizerFast(vocab={w: i for i, w in enumerate(words)}).save_pretrained(enc_dir)
        torch.manual_seed(0)
        BertModel(BertConfig(vocab_size=len(words), hidden_size=64, num_hidden_layers=2, num_attention_heads=2,
                             intermediate_size=128, max_position_embeddings=64)).save_pretrained(enc_dir)
        eng = _routing_engine(tmp, slots=2, encoder=enc_dir)
        assert isinstance(eng.router.encoder, SentenceEncoder)
        t0 = time.time()
        while eng.router.indexing and time.time() - t0 < 120:
            eng.router.tick()
            time.sleep(0.02)
        assert sorted(eng.router.pool.routable_names()) == sorted(TOPICS)
        svc = eng.router.indexer_service.describe()
        assert svc["executors"]["cpu"]["running"] and svc["executors"]["cpu"]["priority"] in ("SCHED_IDLE", "nice 19")
        hits = 0
        for name, texts in TOPICS.items():
            d = eng.router.router.route_many([texts[0]])[0]
            hits += d.adapter == name
        assert hits >= 3, hits
        eng.close()


def test_encode_step_runs_off_the_engine_thread():
    """With the asynchronous encode step the engine thread only hands the
    batch over: the decisions land on a later tick, a request cancelled while
    its batch is encoded is dropped, and has_pending covers the batch in
    flight."""
    import threading
    import time
    with tempfile.TemporaryDirectory() as tmp:
        eng = _routing_engine(tmp, slots=2)
        t0 = time.time()
        while eng.router.indexing and time.time() - t0 < 60:
            eng.router.tick()
            time.sleep(0.01)
        r = eng.router
        gate = threading.Event()
        inner = r.router.encoder

        class Slow:
            def encode(self, texts):
                gate.wait(10)
                return inner.encode(texts)

        r.router.encoder = Slow()
        f1 = r.submit("a1", [1, 2, 3], None, text="bake bread with yeast and flour")
        f2 = r.submit("a2", [1, 2, 3], None, text="bond yields and interest rates")
        r.tick()
        assert r._inflight is not None and r.has_pending() and not f1.done()
        assert r.cancel("a2")
        gate.set()
        t0 = time.time()
        while r._inflight is not None and time.time() - t0 < 10:
            time.sleep(0.01)
            r.tick()
        assert f1.done() and f1.result().adapter == "cooking"
        assert f2.cancelled()
        assert "a1" in eng.requests and "a2" not in eng.requests
        eng.close()
