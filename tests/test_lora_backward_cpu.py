"""BASELINE config 1 (tp=1 part): the hand-written LoRA backward over the
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
