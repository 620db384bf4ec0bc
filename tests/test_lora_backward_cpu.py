"""TP=1 part of the CPU plumbing check: the hand-written LoRA backward over the
captured activations == torch autograd, fp32, tiny Qwen3-style and Llama-style
models, LoRA r=8 alpha=16 on all 7 projections, first 16 label positions masked."""
import pytest
import torch

from deltaserve_vllm_b200.models.configs import PRESETS
from deltaserve_vllm_b200.models.lora import random_adapter

from lora_harness import autograd_reference, config1_data, manual_backward


@pytest.mark.parametrize("name", ["qwen3-tiny", "llama3-tiny"])
def test_manual_backward_matches_autograd(name):
    arch = PRESETS[name]
    seqs = config1_data(arch)
    ad = random_adapter(arch, 8, seed=7, b_std=0.01)
    # lr=0: one full cycle (head, layers, clip, AdamW, publish) leaves the
    # masters unchanged; the gradient buffer holds the unclipped gradient.
    trainer, _ = manual_backward(arch, seqs, ad, 8, 16, lr=0.0)
    ref_loss, ref_grads = autograd_reference(arch, seqs, ad, 8, 16)
    got = trainer.masters.export_peft(8, grads=True)
    assert abs(trainer.losses[-1] - ref_loss) <= 1e-5 * max(1.0, abs(ref_loss))
    scale = max(g.abs().max().item() for g in ref_grads.values())
    for k, g_ref in ref_grads.items():
        torch.testing.assert_close(got[k], g_ref, rtol=1e-5, atol=1e-5 * scale, msg=k)


def test_training_reduces_loss():
    arch = PRESETS["qwen3-tiny"]
    seqs = config1_data(arch, n_seq=2, seq_len=32)
    ad = random_adapter(arch, 8, seed=7, b_std=0.01)
    trainer, res = manual_backward(arch, seqs, ad, 8, 16, lr=5e-3, steps=8, mask_prefix=0)
    losses = [r.loss for r in res]
    assert losses[-1] < losses[0] - 0.05, losses


def test_dense_attention_reference_matches_autograd():
    """The packed varlen attention oracle (the fused kernels' reference) and
    the batched fp32 trainer path both equal autograd of causal GQA attention."""
    import math
    from deltaserve_vllm_b200 import ops
    from deltaserve_vllm_b200.models.lora_backward import attn_backward
    torch.manual_seed(0)
    lens, Hq, Hkv, hd = [5, 17, 64, 3], 4, 2, 128
    n = sum(lens) + 3
    starts = [sum(lens[:i]) for i in range(len(lens))]
    q = torch.randn(n, Hq, hd, dtype=torch.float64, requires_grad=True)
    k = torch.randn(n, Hkv, hd, dtype=torch.float64, requires_grad=True)
    v = torch.randn(n, Hkv, hd, dtype=torch.float64, requires_grad=True)
    do = torch.randn(n, Hq, hd, dtype=torch.float64)
    scale = 1 / math.sqrt(hd)
    out = torch.zeros(n, Hq, hd, dtype=torch.float64)
    for st, ln in zip(starts, lens):
        sl = slice(st, st + ln)
        kk, vv = k[sl].repeat_interleave(2, 1), v[sl].repeat_interleave(2, 1)
        s = torch.einsum("qhd,khd->hqk", q[sl], kk) * scale
        s = s.masked_fill(torch.triu(torch.ones(ln, ln, dtype=torch.bool), 1), float("-inf"))
        out[sl] = torch.einsum("hqk,khd->qhd", s.softmax(-1), vv)
    (out * do).sum().backward()
    tiles = ops.dense_attn_tiles(starts, lens, "cpu")
    assert tiles[:, 2].tolist() == sorted(tiles[:, 2].tolist())
    dq, dk, dv = ops.attn_bwd(q.detach().float(), k.detach().float(), v.detach().float(),
                              do.float().reshape(n, Hq * hd), tiles, scale)
    for got, exp in ((dq, q.grad), (dk, k.grad), (dv, v.grad)):
        torch.testing.assert_close(got.double(), exp, rtol=1e-4, atol=1e-5)
    dq2, dk2, dv2 = attn_backward(q.detach().float(), k.detach().float(), v.detach().float(), do.float(),
                                  starts, lens, scale)
    torch.testing.assert_close(dq2.double(), q.grad, rtol=1e-4, atol=1e-5)
    o = ops.attn_fwd_dense(q.detach().float(), k.detach().float(), v.detach().float(), tiles, scale,
                           torch.zeros(n, Hq * hd))
    torch.testing.assert_close(o.double().view(n, Hq, hd), out.detach(), rtol=1e-4, atol=1e-5)


def test_attn_bwd_wrapper_rope_and_dqkv_cpu():
    """The CPU path of ops.attn_bwd with RoPE and bf16 d(qkv) outputs equals
    the plain fp32 outputs rotated back, written into the fused rows."""
    import math
    from deltaserve_vllm_b200 import ops
    from deltaserve_vllm_b200.models.rope import cos_sin, rope_backward
    torch.manual_seed(1)
    lens, Hq, Hkv, hd = [9, 30], 4, 2, 128
    n = 40
    starts = [0, 9]
    q, k, v = torch.randn(n, Hq, hd), torch.randn(n, Hkv, hd), torch.randn(n, Hkv, hd)
    d_o = torch.randn(n, Hq * hd)
    tiles = ops.dense_attn_tiles(starts, lens, "cpu")
    cos, sin = cos_sin(torch.arange(n), hd, 10000.0)
    dq, dk, dv = ops.attn_bwd(q, k, v, d_o, tiles, 1 / math.sqrt(hd))
    dqkv = torch.full((n, (Hq + 2 * Hkv) * hd), 5.0)
    out = ops.attn_bwd(q, k, v, d_o, tiles, 1 / math.sqrt(hd), rope=(cos, sin), dqkv=dqkv, bf16_mask=6)
    torch.testing.assert_close(out[0], rope_backward(dq, cos, sin))
    assert out[1] is None and out[2] is None
    torch.testing.assert_close(dqkv[:39, Hq * hd:(Hq + Hkv) * hd], rope_backward(dk, cos, sin)[:39].reshape(39, -1))
    torch.testing.assert_close(dqkv[:39, (Hq + Hkv) * hd:], dv[:39].reshape(39, -1))
    assert (dqkv[39:] == 5.0).all() and (dqkv[:, :Hq * hd] == 5.0).all()
