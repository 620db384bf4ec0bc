"""Independent dense (non-paged, unfused) decoder forward used as a test oracle:
plain HF-orientation weights, full causal attention per sequence, fp32."""
import math

import torch
import torch.nn.functional as F

from deltaserve_vllm_b200.models.rope import cos_sin, apply_rope


def rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def dense_forward(arch, full_layers, embed, lm_head, final_norm, ids, lora=None, scaling=0.0):
    """full_layers: list of dicts (q,k,v,o,gate,up,down,in_ln,post_ln[,q_norm,k_norm]) fp32.
    lora: dict peft_key -> tensor (optional). Returns logits [n, V] fp32."""
    from deltaserve_vllm_b200.models.lora import peft_key
    n = ids.shape[0]
    H, Hk, hd = arch.num_heads, arch.num_kv_heads, arch.head_dim
    x = embed[ids].float()
    pos = torch.arange(n)
    c, s = cos_sin(pos, hd, arch.rope_theta, arch.rope_scaling)

    def proj(t, i, name, w):
        y = t @ w.t()
        if lora is not None and peft_key(i, name, "A") in lora:
            A, B = lora[peft_key(i, name, "A")].float(), lora[peft_key(i, name, "B")].float()
            y = y + scaling * (t @ A.t()) @ B.t()
        return y

    for i, L in enumerate(full_layers):
        L = {k: v.float() for k, v in L.items()}
        h = rms(x, L["in_ln"], arch.rms_eps)
        q = proj(h, i, "q", L["q"]).view(n, H, hd)
        k = proj(h, i, "k", L["k"]).view(n, Hk, hd)
        v = proj(h, i, "v", L["v"]).view(n, Hk, hd)
        if arch.qk_norm:
            q = rms(q, L["q_norm"], arch.rms_eps)
            k = rms(k, L["k_norm"], arch.rms_eps)
        q, k = apply_rope(q, c, s), apply_rope(k, c, s)
        k = k.repeat_interleave(H // Hk, 1)
        v = v.repeat_interleave(H // Hk, 1)
        sc = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd)
        sc = sc.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool), 1)[None], float("-inf"))
        ctx = torch.einsum("hqk,khd->qhd", sc.softmax(-1), v).reshape(n, H * hd)
        x = x + proj(ctx, i, "o", L["o"])
        h2 = rms(x, L["post_ln"], arch.rms_eps)
        g = proj(h2, i, "gate", L["gate"])
        u = proj(h2, i, "up", L["up"])
        x = x + proj(F.silu(g) * u, i, "down", L["down"])
    return rms(x, final_norm.float(), arch.rms_eps) @ lm_head.float().t()
