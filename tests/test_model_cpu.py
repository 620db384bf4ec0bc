"""Paged, chunked, multi-LoRA serving forward == independent dense forward (fp32, CPU)."""
import pytest
import torch

from deltaserve_vllm_b200.engine.kv_cache import KVCache
from deltaserve_vllm_b200.engine.model_runner import ModelRunner
from deltaserve_vllm_b200.engine.request import Request, SamplingParams
from deltaserve_vllm_b200.engine.scheduler import Scheduler
from deltaserve_vllm_b200.models.configs import PRESETS
from deltaserve_vllm_b200.models.decoder import DecoderModel
from deltaserve_vllm_b200.models.lora import LoraServeBuffers, random_adapter
from deltaserve_vllm_b200.models.weights import full_layer_tensors, init_weights

from dense_ref import dense_forward


def build(arch_name, with_lora):
    arch = PRESETS[arch_name]
    w = init_weights(arch, seed=3, dtype=torch.float32)
    kv = KVCache(arch.num_layers, 64, arch.num_kv_heads, 16, arch.head_dim, "cpu", torch.float32)
    lora = None
    ad = None
    if with_lora:
        lora = LoraServeBuffers(arch, w.tp, slots=2, max_rank=16, device="cpu", dtype=torch.float32)
        ad = random_adapter(arch, 8, seed=5, b_std=0.05)
        lora.load_slot(1, ad, rank=8, alpha=16)
    model = DecoderModel(w, kv.k, kv.v, lora)
    full = [full_layer_tensors(arch, i, 3, "cpu", torch.float32) for i in range(arch.num_layers)]
    return arch, w, kv, model, full, ad


@pytest.mark.parametrize("arch_name", ["qwen3-tiny", "llama3-tiny"])
@pytest.mark.parametrize("with_lora", [False, True])
def test_paged_forward_matches_dense(arch_name, with_lora):
    arch, w, kv, model, full, ad = build(arch_name, with_lora)
    sched = Scheduler(kv.allocator, 16, max_num_batched_tokens=20, max_model_len=256)
    runner = ModelRunner(model, 16, "cpu")
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, arch.vocab, (37,), generator=g).tolist()
    other = torch.randint(0, arch.vocab, (9,), generator=g).tolist()
    r1 = Request("a", prompt, SamplingParams(max_tokens=5))
    r2 = Request("b", other, SamplingParams(max_tokens=3))
    if with_lora:
        r1.lora_slot = 1
    sched.add(r1)
    sched.add(r2)
    for _ in range(12):
        out = sched.schedule()
        if out.is_empty():
            break
        toks, logits = runner.execute(out)
        i = 0
        for s in out.seqs:
            if not s.sample:
                continue
            req = s.req
            seq = torch.tensor(req.all_ids[: s.start + s.num_new])
            ref = dense_forward(arch, full, w.embed, w.lm_head, w.final_norm, seq,
                                lora=ad if req.lora_slot == 1 else None, scaling=16 / 8)[-1]
            torch.testing.assert_close(logits[i], ref, rtol=2e-4, atol=2e-4)
            i += 1
        sched.update(out, toks)
    assert r1.finished() and r2.finished()
    assert len(r1.output_ids) == 5 and len(r2.output_ids) == 3
    assert kv.allocator.num_free == kv.allocator.num_blocks


def _serve(num_blocks, prompts, max_tokens, block_size=16, caching=False, waves=1, budget=64):
    """Greedy outputs of ``prompts`` served with ``num_blocks`` KV pages; with
    ``waves`` > 1 the prompts arrive in that many groups, each after the
    previous one finished (so later groups can hit pages cached by earlier ones)."""
    arch = PRESETS["qwen3-tiny"]
    # large init: the greedy continuations vary token to token (a small-init
    # random model repeats one token, which would hide ordering mistakes)
    w = init_weights(arch, seed=3, dtype=torch.float32, std=0.3)
    kv = KVCache(arch.num_layers, num_blocks, arch.num_kv_heads, block_size, arch.head_dim, "cpu", torch.float32,
                 prefix_caching=caching)
    model = DecoderModel(w, kv.k, kv.v, None)
    sched = Scheduler(kv.allocator, block_size, max_num_batched_tokens=budget, max_model_len=256)
    runner = ModelRunner(model, block_size, "cpu")
    reqs = [Request(f"r{i}", p, SamplingParams(max_tokens=max_tokens)) for i, p in enumerate(prompts)]
    preempted = 0
    per = -(-len(reqs) // waves)
    for w0 in range(0, len(reqs), per):
        for r in reqs[w0:w0 + per]:
            sched.add(r)
        for _ in range(2000):
            out = sched.schedule()
            preempted += len(out.preempted)
            if out.is_empty():
                break
            toks, _ = runner.execute(out)
            sched.update(out, toks)
    assert all(r.finished() for r in reqs)
    assert kv.allocator.num_free == kv.allocator.num_blocks
    _serve.last = (sched, reqs)
    return [list(r.output_ids) for r in reqs], preempted


def test_preemption_by_recompute_keeps_outputs():
    """A request pre-empted after it produced tokens recomputes prompt AND
    outputs, then continues: its output equals an uninterrupted run."""
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 1024, (20 + 3 * i,), generator=g).tolist() for i in range(5)]
    ref, p0 = _serve(256, prompts, 40)
    got, p1 = _serve(14, prompts, 40)
    assert p0 == 0 and p1 > 0
    assert all(len(set(o)) > 5 for o in ref)       # non-degenerate continuations
    assert got == ref



def test_prefix_caching_reuses_pages_and_matches_uncached():
    """Automatic prefix caching: prompts sharing a system prefix (and exact
    repeats) reuse cached full pages; outputs equal the uncached run; a tiny
    cache evicts and still matches."""
    g = torch.Generator().manual_seed(11)
    system = torch.randint(0, 1024, (70,), generator=g).tolist()
    prompts = [system + torch.randint(0, 1024, (5 + i,), generator=g).tolist() for i in range(4)]
    prompts += [prompts[0], prompts[2][:40]]          # an exact repeat, a strict prefix
    ref, _ = _serve(256, prompts, 12, waves=3)
    got, _ = _serve(256, prompts, 12, caching=True, waves=3)
    assert got == ref
    sched, reqs = _serve.last
    st = sched.cache_stats()
    assert st["hit_pages"] > 0
    # the first wave computes the shared system prompt; later waves reuse its
    # 4 full pages (64 of 70 tokens); the exact repeat reuses every page but
    # the one holding its last token; the 40-token prefix reuses 2 pages
    assert reqs[2].num_cached_tokens == 64 and reqs[3].num_cached_tokens == 64
    assert reqs[4].num_cached_tokens == ((len(prompts[0]) - 1) // 16) * 16
    assert reqs[5].num_cached_tokens == 32
    tight, _ = _serve(24, prompts, 12, caching=True, waves=3)
    assert tight == ref


def test_prefix_caching_with_preemption():
    g = torch.Generator().manual_seed(12)
    base = torch.randint(0, 1024, (40,), generator=g).tolist()
    prompts = [base + torch.randint(0, 1024, (3 * i + 1,), generator=g).tolist() for i in range(5)]
    ref, _ = _serve(256, prompts, 40)
    got, pre = _serve(16, prompts, 40, caching=True)
    assert pre > 0 and got == ref


def test_mixed_rank_adapters_in_one_batch_match_dense():
    """Adapters of ranks 2, 4, 8 and 16 (alpha = 2 x rank) in the slots of a
    rank-16 engine, one request on each plus one on the base model, served in
    the same batches: each request's logits == the dense forward with its own
    adapter at its own rank (the smaller ranks are zero-padded in their
    slots), as a pool of adapters with ranks drawn from {8, 16, 32, 64}
    serves them."""
    arch = PRESETS["llama3-tiny"]
    w = init_weights(arch, seed=3, dtype=torch.float32)
    kv = KVCache(arch.num_layers, 96, arch.num_kv_heads, 16, arch.head_dim, "cpu", torch.float32)
    lora = LoraServeBuffers(arch, w.tp, slots=5, max_rank=16, device="cpu", dtype=torch.float32)
    ranks = {1: 2, 2: 4, 3: 8, 4: 16}
    ads = {}
    for slot, r in ranks.items():
        ads[slot] = random_adapter(arch, r, seed=20 + slot, b_std=0.05)
        lora.load_slot(slot, ads[slot], rank=r, alpha=2 * r)
    model = DecoderModel(w, kv.k, kv.v, lora)
    full = [full_layer_tensors(arch, i, 3, "cpu", torch.float32) for i in range(arch.num_layers)]
    sched = Scheduler(kv.allocator, 16, max_num_batched_tokens=48, max_model_len=256)
    runner = ModelRunner(model, 16, "cpu")
    g = torch.Generator().manual_seed(1)
    reqs = []
    for i, slot in enumerate([1, 2, 3, 4, -1]):
        r = Request(f"m{i}", torch.randint(0, arch.vocab, (11 + 5 * i,), generator=g).tolist(),
                    SamplingParams(max_tokens=3))
        r.lora_slot = slot
        reqs.append(r)
        sched.add(r)
    checked = 0
    for _ in range(20):
        out = sched.schedule()
        if out.is_empty():
            break
        toks, logits = runner.execute(out)
        i = 0
        for s in out.seqs:
            if not s.sample:
                continue
            req = s.req
            seq = torch.tensor(req.all_ids[: s.start + s.num_new])
            slot = req.lora_slot
            ref = dense_forward(arch, full, w.embed, w.lm_head, w.final_norm, seq,
                                lora=ads.get(slot), scaling=2.0)[-1]
            torch.testing.assert_close(logits[i], ref, rtol=2e-4, atol=2e-4)
            i += 1
            checked += 1
        sched.update(out, toks)
    assert all(r.finished() for r in reqs) and checked == 15
