"""Inference correctness against an independent implementation: transformers.

A tiny Llama-3 (llama3 RoPE scaling) and a tiny Qwen3 are built with
transformers, saved as safetensors, and served through the engine's own
loader (``load_format: auto``), paged KV, chunked prefill and decode. The
engine's logits must match the transformers model's at every sampled position
(fp32, CPU). A PEFT adapter written in this package's checkpoint format must
give the logits of the transformers model with that adapter merged into its
weights (``W + alpha/r * B @ A``). This is the reference's "PEFT-loadable with
matching logits vs a transformers Llama" check (``tests/test_adapter_save.py``)
and its inference-correctness gate (``tests/test_phase1_m1.py``).
"""

import os

import pytest
import torch

transformers = pytest.importorskip("transformers")

from deltaserve_vllm_b200.adapters import peft_io
from deltaserve_vllm_b200.config import EngineConfig, FinetuneConfig
from deltaserve_vllm_b200.engine.kv_cache import KVCache
from deltaserve_vllm_b200.engine.llm_engine import CoServingEngine
from deltaserve_vllm_b200.engine.model_runner import ModelRunner
from deltaserve_vllm_b200.engine.request import Request, SamplingParams
from deltaserve_vllm_b200.engine.scheduler import Scheduler
from deltaserve_vllm_b200.models.configs import resolve_arch
from deltaserve_vllm_b200.models.decoder import DecoderModel
from deltaserve_vllm_b200.models.loader import load_hf_weights
from deltaserve_vllm_b200.models.lora import LORA_PROJS, PEFT_MODULE, peft_key, random_adapter
from deltaserve_vllm_b200.models.weights import TPInfo, shard_layer

COMMON = dict(hidden_size=128, num_attention_heads=4, num_key_value_heads=2, head_dim=32,
              intermediate_size=256, num_hidden_layers=2, vocab_size=512, max_position_embeddings=1024,
              rms_norm_eps=1e-6)


def _hf_model(family: str, tie: bool):
    torch.manual_seed(11)
    if family == "llama":
        cfg = transformers.LlamaConfig(**COMMON, tie_word_embeddings=tie, rope_theta=500000.0,
                                       rope_scaling={"rope_type": "llama3", "factor": 8.0,
                                                     "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                                     "original_max_position_embeddings": 64})
        model = transformers.LlamaForCausalLM(cfg)
    else:
        cfg = transformers.Qwen3Config(**COMMON, tie_word_embeddings=tie, rope_theta=1000000.0)
        model = transformers.Qwen3ForCausalLM(cfg)
    model = model.float().eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight"):        # all-ones norms would hide layout bugs
                p.uniform_(0.8, 1.2)
            elif p.dim() == 2:
                p.normal_(0.0, 0.05)
    return model


def _save(model, path):
    model.save_pretrained(path, safe_serialization=True)
    assert any(f.endswith(".safetensors") for f in os.listdir(path))


def _hf_logits(model, ids):
    with torch.no_grad():
        return model(torch.tensor([ids])).logits[0].float()


def _merged(model, tensors, rank, alpha):
    """A copy of ``model`` with the LoRA delta folded into each target weight."""
    import copy
    m = copy.deepcopy(model)
    sd = dict(m.named_parameters())
    with torch.no_grad():
        for i in range(model.config.num_hidden_layers):
            for proj in LORA_PROJS:
                A, B = tensors[peft_key(i, proj, "A")], tensors[peft_key(i, proj, "B")]
                sd[f"model.layers.{i}.{PEFT_MODULE[proj]}.weight"] += (alpha / rank) * (B @ A)
    return m


def _serve_logits(weights, lora, slot, prompts, decode_steps):
    """Logits of every sampled position: the last prompt token, then each decode step."""
    arch = weights.arch
    kv = KVCache(arch.num_layers, 64, arch.num_kv_heads, 16, arch.head_dim, "cpu", torch.float32)
    model = DecoderModel(weights, kv.k, kv.v, lora)
    sched = Scheduler(kv.allocator, 16, max_num_batched_tokens=24, max_model_len=512)
    runner = ModelRunner(model, 16, "cpu")
    reqs = []
    for j, ids in enumerate(prompts):
        r = Request(f"r{j}", list(ids), SamplingParams(max_tokens=decode_steps))
        r.lora_slot = slot
        sched.add(r)
        reqs.append(r)
    seen = {r.request_id: [] for r in reqs}
    for _ in range(64):
        out = sched.schedule()
        if out.is_empty():
            break
        toks, logits = runner.execute(out)
        i = 0
        for s in out.seqs:
            if s.sample:
                seen[s.req.request_id].append((list(s.req.all_ids[: s.start + s.num_new]), logits[i].clone()))
                i += 1
        sched.update(out, toks)
    assert all(r.finished() for r in reqs)
    return seen


@pytest.mark.parametrize("family,tie", [("llama", False), ("qwen3", False), ("qwen3", True)])
def test_engine_matches_transformers(tmp_path, family, tie):
    hf = _hf_model(family, tie)
    mdir = str(tmp_path / "model")
    _save(hf, mdir)
    arch = resolve_arch(mdir)
    assert arch.family == family and arch.tie_embeddings == tie
    if family == "llama":
        assert arch.rope_scaling["rope_type"] == "llama3" and arch.rope_theta == 500000.0
    else:
        assert arch.rope_scaling is None and arch.rope_theta == 1000000.0
    # the engine loads the checkpoint itself (load_format auto)
    eng = CoServingEngine(EngineConfig(model=mdir, device="cpu", max_model_len=512, block_size=16,
                                       max_num_batched_tokens=64, max_loras=2, max_lora_rank=8),
                          FinetuneConfig(enable_finetuning=False))
    ref_w = load_hf_weights(arch, mdir, dtype=torch.float32, keep_full_head=False)
    torch.testing.assert_close(eng.weights.layers[1].gate_up, ref_w.layers[1].gate_up, rtol=0, atol=0)
    torch.testing.assert_close(eng.weights.embed, hf.model.embed_tokens.weight.detach(), rtol=0, atol=0)

    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (45, 7, 19)]
    served = _serve_logits(eng.weights, eng.lora, -1, prompts, decode_steps=4)
    for rid, rows in served.items():
        assert len(rows) == 4
        for ids, lg in rows:
            torch.testing.assert_close(lg, _hf_logits(hf, ids)[-1], rtol=1e-4, atol=1e-4)

    # a PEFT adapter in this package's format == the transformers model with it merged
    rank, alpha = 8, 16.0
    ad = random_adapter(arch, rank, seed=4, b_std=0.05)
    adir = str(tmp_path / "adapter")
    peft_io.write_peft_adapter(adir, ad, peft_io.default_adapter_config(rank, alpha, LORA_PROJS, mdir),
                               {"save_id": "t"})
    slot = eng.load_inference_adapter("hf_lora", path=adir)
    merged = _merged(hf, ad, rank, alpha)
    served = _serve_logits(eng.weights, eng.lora, slot, prompts[:2], decode_steps=3)
    for rows in served.values():
        for ids, lg in rows:
            ref = _hf_logits(merged, ids)[-1]
            torch.testing.assert_close(lg, ref, rtol=1e-4, atol=1e-4)
            assert (ref - _hf_logits(hf, ids)[-1]).abs().max() > 1e-2   # the adapter matters


def test_loader_tp_slices_match_full_shard(tmp_path):
    hf = _hf_model("qwen3", False)
    mdir = str(tmp_path / "m")
    _save(hf, mdir)
    arch = resolve_arch(mdir)
    full = load_hf_weights(arch, mdir, dtype=torch.float32)
    sd = {k: v.detach() for k, v in hf.state_dict().items()}
    for r in range(2):
        tp = TPInfo(r, 2)
        w = load_hf_weights(arch, mdir, tp, dtype=torch.float32, keep_full_head=True)
        assert w.embed.shape[0] == arch.vocab // 2
        torch.testing.assert_close(w.lm_head_full, sd["lm_head.weight"], rtol=0, atol=0)
        torch.testing.assert_close(w.lm_head, sd["lm_head.weight"][r * 256:(r + 1) * 256], rtol=0, atol=0)
        for i in range(arch.num_layers):
            pre = f"model.layers.{i}."
            t = {"q": sd[pre + "self_attn.q_proj.weight"], "k": sd[pre + "self_attn.k_proj.weight"],
                 "v": sd[pre + "self_attn.v_proj.weight"], "o": sd[pre + "self_attn.o_proj.weight"],
                 "gate": sd[pre + "mlp.gate_proj.weight"], "up": sd[pre + "mlp.up_proj.weight"],
                 "down": sd[pre + "mlp.down_proj.weight"], "in_ln": sd[pre + "input_layernorm.weight"],
                 "post_ln": sd[pre + "post_attention_layernorm.weight"],
                 "q_norm": sd[pre + "self_attn.q_norm.weight"], "k_norm": sd[pre + "self_attn.k_norm.weight"]}
            ref = shard_layer(arch, t, tp)
            for f in ("qkv", "o", "gate_up", "down", "in_ln", "post_ln", "q_norm", "k_norm"):
                torch.testing.assert_close(getattr(w.layers[i], f), getattr(ref, f), rtol=0, atol=0)
    assert full.layers[0].qkv.shape[0] == arch.q_size + 2 * arch.kv_size


def test_load_format_checks(tmp_path):
    with pytest.raises(FileNotFoundError):
        CoServingEngine(EngineConfig(model="qwen3-tiny", device="cpu", load_format="safetensors",
                                     max_model_len=256, block_size=16),
                        FinetuneConfig(enable_finetuning=False))
    with pytest.raises(ValueError):
        CoServingEngine(EngineConfig(model="qwen3-tiny", device="cpu", load_format="gguf",
                                     max_model_len=256, block_size=16),
                        FinetuneConfig(enable_finetuning=False))
    hf = _hf_model("llama", False)
    mdir = str(tmp_path / "m")
    _save(hf, mdir)
    eng = CoServingEngine(EngineConfig(model=mdir, device="cpu", load_format="dummy", max_model_len=256,
                                       block_size=16), FinetuneConfig(enable_finetuning=False))
    assert not torch.equal(eng.weights.embed, hf.model.embed_tokens.weight.detach())
