"""Plain PyTorch restatements of every kernel in ``ops/csrc`` — the oracle the
tests compare the CUDA kernels against, and the path CPU tensors take.

Each function mirrors the exact contract (layouts, rounding points) of its
kernel so that CPU runs of the engine and GPU runs agree up to bf16 rounding.
"""

from __future__ import annotations


import math

import torch
import torch.nn.functional as F

EPI_BF16, EPI_F32, EPI_SWIGLU, EPI_F32_ACCUM = 0, 1, 2, 3
EPI_SWIGLU_BWD = 7  # MN-major only: SwiGLU backward over saved interleaved gate/up


def deinterleave64(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Split a [..., 2I] tensor laid out as [g(64) u(64) g(64) u(64) ...] into (g, u)."""
    shp = x.shape
    v = x.reshape(*shp[:-1], shp[-1] // 128, 2, 64)
    return v[..., 0, :].reshape(*shp[:-1], -1), v[..., 1, :].reshape(*shp[:-1], -1)


def interleave64(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    shp = g.shape
    gv = g.reshape(*shp[:-1], shp[-1] // 64, 1, 64)
    uv = u.reshape(*shp[:-1], shp[-1] // 64, 1, 64)
    return torch.cat([gv, uv], dim=-2).reshape(*shp[:-1], 2 * shp[-1])


def gemm(a, b, out, b_mn=False, epi=EPI_BF16, z=None, b2=None, tile_slots=None, lora_seg=0,
         save=None, save_lo=0, save_hi=0, save_dst=0, aux=None, aux_out=None):
    acc = a.float() @ (b.float() if b_mn else b.float().t())
    if lora_seg and z is not None:  # b_mn: b2 is [S*SEG, N] like b (rows past its end are zero); else [N, S*SEG]
        if b_mn:
            acc = acc + z[: a.shape[0], : b2.shape[0]].float() @ b2.float()
        else:
            acc = acc + z[: a.shape[0]].float() @ b2.float().t()
    if save is not None and save_hi > save_lo:
        save[save_dst: save_dst + save_hi - save_lo] = acc[save_lo:save_hi].to(save.dtype)
    if epi == EPI_SWIGLU:
        g, u = deinterleave64(acc)
        out.copy_((F.silu(g) * u).to(out.dtype))
    elif epi == EPI_SWIGLU_BWD:
        swiglu_bwd(aux[: a.shape[0]], acc, out, aux_out)
    elif epi == EPI_F32_ACCUM:
        out.add_(acc)
    else:
        out.copy_(acc.to(out.dtype))
    return out


def rms_norm(x, residual, w, out, eps, save=None, save_lo=0, save_hi=0, save_dst=0):
    if residual is not None:
        r = (x.float() + residual.float()).to(residual.dtype)
        residual.copy_(r)
        src = r
    else:
        src = x
    if save is not None and save_hi > save_lo:
        save[save_dst: save_dst + save_hi - save_lo] = src[save_lo:save_hi]
    xf = src.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    out.copy_((xf * inv * w.float()).to(out.dtype))
    return out


def rope_cos_sin_table(max_pos: int, head_dim: int, theta: float, rope_scaling=None,
                       device=None) -> torch.Tensor:
    """fp32 [max_pos, head_dim] table laid out as [cos(hd/2) | sin(hd/2)]."""
    from ..models.rope import rope_inv_freq
    inv = rope_inv_freq(head_dim, theta, rope_scaling, device=device)
    pos = torch.arange(max_pos, dtype=torch.float32, device=device)
    f = torch.outer(pos, inv)
    return torch.cat([f.cos(), f.sin()], dim=-1).contiguous()


def _apply_rope(x, cos, sin):
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def qk_norm_rope_cache(qkv, positions, cos_sin, q_norm, k_norm, eps, Hq, Hkv,
                       k_cache=None, v_cache=None, slot_mapping=None):
    T = qkv.shape[0]
    if T == 0:
        return
    hd = qkv.shape[1] // (Hq + 2 * Hkv)
    v3 = qkv.view(T, Hq + 2 * Hkv, hd)
    q = v3[:, :Hq].float()
    k = v3[:, Hq:Hq + Hkv].float()
    if q_norm is not None:
        def _n(t, w):
            inv = torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps)
            return (t * inv * w.float()).to(qkv.dtype).float()
        q, k = _n(q, q_norm), _n(k, k_norm)
    cs = cos_sin[positions]
    cos, sin = cs[:, None, : hd // 2], cs[:, None, hd // 2:]
    v3[:, :Hq] = _apply_rope(q, cos, sin).to(qkv.dtype)
    v3[:, Hq:Hq + Hkv] = _apply_rope(k, cos, sin).to(qkv.dtype)
    if k_cache is not None:
        bs = k_cache.shape[2]
        ok = slot_mapping >= 0
        sl = slot_mapping[ok]
        blk, off = sl // bs, sl % bs
        k_cache[blk, :, off] = v3[ok, Hq:Hq + Hkv]
        v_cache[blk, :, off] = v3[ok, Hq + Hkv:]


def _gather_kv(cache, btab, n, hd_heads):
    bs = cache.shape[2]
    pos = torch.arange(n, device=cache.device)
    pages = btab[pos // bs].long()
    return cache[pages, :, pos % bs]  # [n, Hkv, hd]


def paged_prefill(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, out, num_heads, scale):
    Hkv = k_cache.shape[1]
    G = num_heads // Hkv
    S = ctx_lens.shape[0]
    for s in range(S):
        q0, q1 = int(cu_q[s]), int(cu_q[s + 1])
        ql = q1 - q0
        if ql == 0:
            continue
        ctx = int(ctx_lens[s])
        k = _gather_kv(k_cache, block_tables[s], ctx, Hkv).float()
        v = _gather_kv(v_cache, block_tables[s], ctx, Hkv).float()
        qs = q[q0:q1].reshape(ql, num_heads, -1).float()
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
        sc = torch.einsum("qhd,khd->hqk", qs, k) * scale
        qpos = torch.arange(ctx - ql, ctx, device=q.device)[:, None]
        kpos = torch.arange(ctx, device=q.device)[None, :]
        sc = sc.masked_fill((kpos > qpos)[None], float("-inf"))
        p = torch.softmax(sc, dim=-1)
        o = torch.einsum("hqk,khd->qhd", p, v)
        out[q0:q1] = o.reshape(ql, -1).to(out.dtype)
    return out


def paged_decode(q, k_cache, v_cache, block_tables, ctx_lens, out, num_heads, scale):
    B = ctx_lens.shape[0]
    cu = torch.arange(B + 1, dtype=torch.int32)
    return paged_prefill(q, k_cache, v_cache, block_tables, cu, ctx_lens, out, num_heads, scale)


def lora_shrink(x, A, slot_ids, Z, seg):
    slots, PR, K = A.shape
    Z.zero_()
    T = x.shape[0]
    for s in range(slots):
        rows = (slot_ids[:T] == s).nonzero().flatten()
        if rows.numel() == 0:
            continue
        Z[rows, s * seg: s * seg + PR] = (x[rows].float() @ A[s].float().t()).to(Z.dtype)
    return Z


def embedding(ids, table, out, v0):
    local = ids - v0
    ok = (local >= 0) & (local < table.shape[0])
    out.zero_()
    out[ok] = table[local[ok]]
    return out


def ce_fwd_bwd(logits, targets, loss, grad=None, gscale=1.0):
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=-1)
    ok = targets >= 0
    tl = lf.gather(1, targets.clamp(min=0)[:, None])[:, 0]
    loss.copy_(torch.where(ok, lse - tl, torch.zeros_like(lse)))
    if grad is not None:
        p = torch.softmax(lf, dim=-1)
        p[torch.arange(p.shape[0]), targets.clamp(min=0)] -= 1.0
        p = p * ok[:, None].float() * gscale
        grad.copy_(p.to(grad.dtype))


def seg_sumsq(g, seg_len, out):
    out.copy_(g.view(-1, seg_len).float().pow(2).sum(-1))


def adamw(p, g, m, v, seg_len, seg_sumsq_t, max_norm, grad_scale, lr, b1, b2, eps, wd, step):
    coef = torch.full((p.numel() // seg_len,), float(grad_scale))
    if seg_sumsq_t is not None and max_norm > 0:
        nrm = seg_sumsq_t.sqrt() * grad_scale
        coef = coef * torch.clamp(max_norm / (nrm + 1e-6), max=1.0)
    gi = (g.view(-1, seg_len) * coef[:, None]).view(-1)
    p.mul_(1 - lr * wd)
    m.mul_(b1).add_(gi, alpha=1 - b1)
    v.mul_(b2).addcmul_(gi, gi, value=1 - b2)
    bc1 = 1 - b1 ** step
    bc2 = 1 - b2 ** step
    p.addcdiv_(m / bc1, (v / bc2).sqrt() + eps, value=-lr)


def lora_publish(A_src, A_dst, Bt_src, B2_dst, col0, b1, b2, interleave, scale):
    A_dst.copy_(A_src.view_as(A_dst).to(A_dst.dtype))
    R, N = Bt_src.shape
    n = torch.arange(N)
    if interleave:
        p = (n // 64) % 2
    else:
        p = torch.where(n < b1, 0, torch.where(n < b2, 1, 2))
    vals = (Bt_src.t() * scale).clamp(-65504, 65504).to(B2_dst.dtype)  # [N, R]
    cols = col0 + p[:, None] * R + torch.arange(R)[None, :]
    B2_dst[n[:, None], cols] = vals


def sample_keep_mask(z: torch.Tensor, k: int, p: float) -> torch.Tensor:
    """Tokens kept by top-k then top-p on scaled logits ``z`` (one row)."""
    keep = torch.ones_like(z, dtype=torch.bool)
    if 0 < k < z.numel():
        keep &= z >= torch.topk(z, k).values[-1]
    if p < 1.0:
        zs = torch.where(keep, z, torch.full_like(z, float("-inf")))
        order = torch.argsort(zs, descending=True)
        probs = torch.softmax(zs[order], -1)
        cum = torch.cumsum(probs, -1)
        n_keep = int((cum < p).sum()) + 1               # up to and including the token crossing p
        thr = zs[order[min(n_keep, z.numel()) - 1]]
        keep &= z >= thr
    return keep


def sample(logits, temps, seeds, out, top_k=None, top_p=None, logprobs=None):
    # The CPU path is greedy for temperature <= 0 and uses torch's RNG
    # otherwise (the GPU kernel uses a counter-based hash per row).
    lf = logits.float()
    res = lf.argmax(-1)
    for r in range(lf.shape[0]):
        t = float(temps[r])
        if t > 0:
            gen = torch.Generator().manual_seed(int(seeds[r]))
            u = torch.rand(lf.shape[1], generator=gen).clamp(1e-7, 1 - 1e-7)
            z = lf[r] / t
            k = int(top_k[r]) if top_k is not None else 0
            p = float(top_p[r]) if top_p is not None else 1.0
            g = z - torch.log(-torch.log(u))
            g = torch.where(sample_keep_mask(z, k, p), g, torch.full_like(g, float("-inf")))
            res[r] = g.argmax()
    out.copy_(res)
    if logprobs is not None:
        lp = torch.log_softmax(lf, -1).gather(1, res.view(-1, 1)).view(-1)
        logprobs.copy_(lp)


def rms_norm_bwd(x, dy, w, eps, add=None, out=None, out_bf16=None):
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    xhat = xf * inv
    g = dy.float() * w.float()
    dx = (g - xhat * (g * xhat).mean(-1, keepdim=True)) * inv
    if add is not None:
        dx = dx + add
    if out is not None:
        out.copy_(dx)
    if out_bf16 is not None:
        out_bf16.copy_(dx.to(out_bf16.dtype))
    return dx


def swiglu_bwd(gu, dact, dgu, act=None):
    g, u = deinterleave64(gu.float())
    sg = torch.sigmoid(g)
    silu = g * sg
    d_u = dact * silu
    d_g = dact * u * sg * (1 + g * (1 - sg))
    dgu.copy_(interleave64(d_g, d_u).to(dgu.dtype))
    if act is not None:
        act.copy_((silu * u).to(act.dtype))


# ----------------------------------------------------------------- trainer attention

def _tile_samples(tiles: torch.Tensor) -> list[tuple[int, int]]:
    return [(st, ln) for st, ln, r in tiles.cpu().tolist() if r == 0]


def _dense_attn_probs(q, k, scale):
    """fp32 causal softmax of one sample: q [l, Hq, d], k [l, Hkv, d] -> [Hq, l, l]."""
    ln, hq, _ = q.shape
    kk = k.float().repeat_interleave(hq // k.shape[1], 1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk) * scale
    mask = torch.triu(torch.ones(ln, ln, dtype=torch.bool, device=q.device), 1)
    return s.masked_fill(mask, float("-inf")).softmax(-1)


def dense_attn_fwd(q, k, v, tiles, scale, out):
    hq, hd = q.shape[1], q.shape[2]
    for st, ln in _tile_samples(tiles):
        p = _dense_attn_probs(q[st:st + ln], k[st:st + ln], scale)
        vv = v[st:st + ln].float().repeat_interleave(hq // v.shape[1], 1)
        o = torch.einsum("hqk,khd->qhd", p, vv).reshape(ln, hq * hd)
        out[st:st + ln, :hq * hd] = o.to(out.dtype)
    return out


def dense_attn_stats(q, k, v, tiles, scale, lse, d_o, dd):
    """Per packed row and query head: the base-2 log-sum-exp of the scaled
    causal scores (``lse`` [Hq, >= n]) and rowsum(dO * O) (``dd``, from
    ``d_o`` [n, Hq * 128]); either may be None."""
    hq, hd = q.shape[1], q.shape[2]
    for st, ln in _tile_samples(tiles):
        qq = q[st:st + ln].float()
        kk = k[st:st + ln].float().repeat_interleave(hq // k.shape[1], 1)
        s = torch.einsum("qhd,khd->hqk", qq, kk) * scale
        mask = torch.triu(torch.ones(ln, ln, dtype=torch.bool, device=q.device), 1)
        s = s.masked_fill(mask, float("-inf"))
        if lse is not None:
            lse[:hq, st:st + ln] = (torch.logsumexp(s, -1) / math.log(2.0)).to(lse.dtype)
        if dd is not None:
            vv = v[st:st + ln].float().repeat_interleave(hq // v.shape[1], 1)
            o = torch.einsum("hqk,khd->qhd", s.softmax(-1), vv)
            g = d_o[st:st + ln].float().reshape(ln, hq, hd)
            dd[:hq, st:st + ln] = (o * g).sum(-1).t().to(dd.dtype)


def dense_attn_bwd(q, k, v, d_o, tiles, scale, dq, dk, dv):
    """fp32 gradients of causal GQA attention per packed sample (d_o [n, Hq, d])."""
    hq, hkv, hd = q.shape[1], k.shape[1], q.shape[2]
    G = hq // hkv
    for st, ln in _tile_samples(tiles):
        sl = slice(st, st + ln)
        p = _dense_attn_probs(q[sl], k[sl], scale)                       # [Hq, l, l]
        kk = k[sl].float().repeat_interleave(G, 1)
        vv = v[sl].float().repeat_interleave(G, 1)
        do = d_o[sl].float()
        dvv = torch.einsum("hqk,qhd->khd", p, do)
        dp = torch.einsum("qhd,khd->hqk", do, vv)
        ds = p * (dp - (dp * p).sum(-1, keepdim=True))
        dq[sl] = torch.einsum("hqk,khd->qhd", ds, kk) * scale
        dkk = torch.einsum("hqk,qhd->khd", ds, q[sl].float()) * scale
        dk[sl] = dkk.view(ln, hkv, G, hd).sum(2)
        dv[sl] = dvv.view(ln, hkv, G, hd).sum(2)


def rope_bwd(g: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Transpose of the NeoX rotate-half RoPE on g [n, H, d] (cos / sin [n, d/2]),
    in fp32: the rotation by the opposite angles."""
    from ..models.rope import rope_backward
    return rope_backward(g.float(), cos.float(), sin.float())


# ----------------------------------------------------------------- LM head + CE on vocabulary slices
# fp32 restatements of ops.ce_stats / ce_merge / ce_finalize / ce_grad (one
# statistics pair per row instead of per tile: n_tiles = 1).

def ce_stats(h, w, labels, v0, stats, tgt):
    logits = h.float() @ w.float().t()
    m = logits.max(-1).values
    s = torch.exp(logits - m[:, None]).sum(-1)
    M = h.shape[0]
    stats[:M, 0] = m
    stats[:M, 1] = s
    lab = labels[:M] - v0
    inside = (labels[:M] >= 0) & (lab >= 0) & (lab < w.shape[0])
    rows = torch.nonzero(inside).view(-1)
    tgt[rows] = logits[rows, lab[rows]]
    return 1


def ce_merge(stats, n_tiles, tgt, part):
    M = part.shape[0]
    part[:, 0] = stats[:M, 0]
    part[:, 1] = stats[:M, 1]
    part[:, 2] = tgt[:M]
    return part


def ce_finalize(parts, labels, lse, loss):
    m = parts[:, :, 0].max(0).values
    s = (parts[:, :, 1] * torch.exp(parts[:, :, 0] - m[None])).sum(0)
    lse.copy_(m + torch.log(s))
    M = parts.shape[1]
    loss.copy_(torch.where(labels[:M] >= 0, lse - parts[:, :, 2].sum(0), torch.zeros_like(lse)))
    return lse, loss


def ce_grad(h, w, labels, v0, lse, scale, dlog):
    logits = h.float() @ w.float().t()
    g = torch.exp(logits - lse[:, None])
    M = h.shape[0]
    lab = labels[:M] - v0
    inside = (labels[:M] >= 0) & (lab >= 0) & (lab < w.shape[0])
    rows = torch.nonzero(inside).view(-1)
    g[rows, lab[rows]] -= 1.0
    g = g * scale
    g[labels[:M] < 0] = 0.0
    dlog.copy_(g.to(dlog.dtype))
    return dlog


def gemm_wgrad(a, b, out, kind, n_valid, R, b1, b2, interleave, scale):
    prod = a.float().t() @ b[:, :n_valid].float()          # [M, n_valid]
    M = a.shape[1]
    if kind == 0:
        out[:n_valid, :M] = prod.t()
        return out
    m = torch.arange(M)
    p = ((m // 64) % 2) if interleave else torch.where(m < b1, 0, torch.where(m < b2, 1, 2))
    cols = p[:, None] * R + torch.arange(R)[None, :]        # [M, R]
    out[:R, :M] = (scale * prod.gather(1, cols.to(prod.device))).t()
    return out
