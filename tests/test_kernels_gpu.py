"""sm_100a kernels vs their fp32 PyTorch restatements (ops/reference.py)."""
import math

import pytest
import torch

from deltaserve_vllm_b200 import ops
from deltaserve_vllm_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert ops.check_device_error() == 0


def rnd(*shape, scale=1.0, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(dtype)


def test_native_loaded():
    assert ops.native_available()


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (77, 640, 320), (128, 128, 64), (300, 1000, 512),
                                   (1024, 4096, 1024), (4096, 1536, 4096)])
@pytest.mark.parametrize("bn", [0, 64, 128, 256])
def test_gemm_kmajor(M, N, K, bn):
    a, b = rnd(M, K, seed=1), rnd(N, K, scale=0.05, seed=2)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm(a, b, out, force_bn=bn)
    exp = a.float() @ b.float().t()
    torch.testing.assert_close(out.float(), exp, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M,N,K", [(64, 256, 128), (200, 512, 384), (4096, 1024, 2048)])
def test_gemm_mn_major_f32(M, N, K):
    a, w = rnd(M, K, seed=3), rnd(K, N, scale=0.05, seed=4)   # out = a @ w (w is [K, N] row-major)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    ops.gemm(a, w, out, b_mn=True, epi=ops.EPI_F32)
    torch.testing.assert_close(out, a.float() @ w.float(), rtol=1e-2, atol=1e-2)
    acc = torch.ones_like(out)
    ops.gemm(a, w, acc, b_mn=True, epi=ops.EPI_F32_ACCUM)
    torch.testing.assert_close(acc, 1 + a.float() @ w.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("M", [300, 2048])
def test_gemm_mn_major_lora_block_unpadded_b2(M):
    """dX = dY . W + dZ . A with A given unpadded ([P*R, N], fewer rows than the
    64-deep K-block): rows past A's end read as zero (dZ's padding columns are
    zero too)."""
    Kred, N, PR = 1024, 2048, 48
    dy, W = rnd(M, Kred, seed=80), rnd(Kred, N, scale=0.02, seed=81)
    zp = torch.zeros(M, 64, dtype=torch.bfloat16, device=DEV)
    zp[:, :PR] = rnd(M, PR, seed=82)
    A = rnd(PR, N, scale=0.05, seed=83)
    ts = torch.ones((M + 127) // 128, dtype=torch.int32, device=DEV)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    ops.gemm(dy, W, out, b_mn=True, epi=ops.EPI_F32, z=zp, b2=A, tile_slots=ts, lora_seg=64, max_ctas=1 << 30)
    exp = dy.float() @ W.float() + zp[:, :PR].float() @ A.float()
    torch.testing.assert_close(out, exp, rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("M,N,K,b_mn", [(48, 4096, 4096, True), (48, 28672, 4096, True), (4096, 48, 4096, True),
                                        (4096, 48, 14336, False), (16, 1024, 8192, True), (2048, 64, 2048, False)])
@pytest.mark.parametrize("epi", [1, 3, 0])
def test_gemm_skinny_splitk(M, N, K, b_mn, epi):
    """The trainer's rank-sized LoRA products (one side <= 64): split-K with a
    deterministic fp32 reduction, for MN-major and K-major B, with the grid
    uncapped as the backward launches it."""
    a = rnd(M, K, seed=50)
    b = rnd(K, N, scale=0.05, seed=51) if b_mn else rnd(N, K, scale=0.05, seed=51)
    exp = a.float() @ (b.float() if b_mn else b.float().t())
    if epi == 0:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    else:
        out = torch.full((M, N), 0.5 if epi == 3 else 0.0, device=DEV)
    ops.gemm(a, b, out, b_mn=b_mn, epi=epi, max_ctas=1 << 30)
    if epi == 3:
        exp = exp + 0.5
    torch.testing.assert_close(out.float(), exp, rtol=2e-2, atol=3e-2)
    out2 = out.clone() if epi != 3 else None
    if out2 is not None:
        ops.gemm(a, b, out2, b_mn=b_mn, epi=epi, max_ctas=1 << 30)
        assert torch.equal(out, out2)


# ---------------------------------------------------------------- CTA-pair GEMM
# Shapes with >= 74 tiles of 256 x 256 take the pair (cta_group::2) kernel;
# ragged M / N exercise rows and columns past the end in either CTA.
@pytest.mark.parametrize("M,N,K", [(2000, 4000, 512), (4096, 4096, 1024), (2304, 8192, 256)])
@pytest.mark.parametrize("max_ctas", [0, 1 << 30])
def test_gemm_pair_kmajor_bf16(M, N, K, max_ctas):
    a, b = rnd(M, K, seed=60), rnd(N, K, scale=0.05, seed=61)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm(a, b, out, max_ctas=max_ctas)
    torch.testing.assert_close(out.float(), a.float() @ b.float().t(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("epi", [1, 3])
def test_gemm_pair_mn_major_f32(epi):
    M, N, K = 2304, 4096, 1024
    a, w = rnd(M, K, seed=62), rnd(K, N, scale=0.05, seed=63)
    out = torch.full((M, N), 0.25, device=DEV)
    ops.gemm(a, w, out, b_mn=True, epi=epi, max_ctas=1 << 30)
    exp = a.float() @ w.float() + (0.25 if epi == 3 else 0.0)
    torch.testing.assert_close(out, exp, rtol=1e-2, atol=1e-2)


def test_gemm_pair_swiglu_save():
    M, K, I = 2048, 512, 4096
    x, w = rnd(M, K, seed=64), rnd(2 * I, K, scale=0.05, seed=65)
    out = torch.empty(M, I, dtype=torch.bfloat16, device=DEV)
    save = torch.zeros(M, 2 * I, dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, out, epi=ops.EPI_SWIGLU, save=save, save_lo=100, save_hi=1900, save_dst=0)
    acc = x.float() @ w.float().t()
    g, u = ref.deinterleave64(acc)
    torch.testing.assert_close(out.float(), torch.nn.functional.silu(g) * u, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(save[:1800].float(), acc[100:1900], rtol=2e-2, atol=2e-2)
    assert save[1800:].abs().sum() == 0


def test_gemm_pair_lora_expand_mixed_slots():
    """LoRA K-blocks: the two 128-row halves of a pair tile carry different
    slots; the pair loads the union."""
    M, N, K, slots, seg = 2048, 4096, 512, 4, 64
    x, w = rnd(M, K, seed=66), rnd(N, K, scale=0.05, seed=67)
    Z = rnd(M, slots * seg, scale=0.5, seed=68)
    B2 = rnd(N, slots * seg, scale=0.05, seed=69)
    nt = M // 128
    mask = torch.tensor([1 << (t % slots) for t in range(nt)], dtype=torch.int32)
    rows_slot = torch.repeat_interleave(torch.tensor([t % slots for t in range(nt)]), 128)
    Zm = Z.float().cpu().clone()
    for s in range(slots):   # a row's Z is zero outside its own slot segment
        Zm[rows_slot != s, s * seg:(s + 1) * seg] = 0
    Zm = Zm.to(DEV).to(torch.bfloat16)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, out, z=Zm, b2=B2, tile_slots=mask.to(DEV), lora_seg=seg)
    exp = x.float() @ w.float().t() + Zm.float() @ B2.float().t()
    torch.testing.assert_close(out.float(), exp, rtol=2e-2, atol=3e-2)


def test_gemm_pair_mn_major_lora_block():
    """The backward's dX GEMM: MN-major B plus one 64-deep adapter K-block."""
    M, Kred, N, PR = 2048, 4096, 4096, 48
    dy, W = rnd(M, Kred, seed=70), rnd(Kred, N, scale=0.02, seed=71)
    zp = torch.zeros(M, 64, dtype=torch.bfloat16, device=DEV)
    zp[:, :PR] = rnd(M, PR, seed=72)
    ap = torch.zeros(64, N, dtype=torch.bfloat16, device=DEV)
    ap[:PR] = rnd(PR, N, scale=0.05, seed=73)
    ts = torch.ones(M // 128, dtype=torch.int32, device=DEV)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    ops.gemm(dy, W, out, b_mn=True, epi=ops.EPI_F32, z=zp, b2=ap, tile_slots=ts, lora_seg=64, max_ctas=1 << 30)
    exp = dy.float() @ W.float() + zp.float() @ ap.float()
    torch.testing.assert_close(out, exp, rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("M", [5, 130, 600])
def test_gemm_swiglu_save(M):
    K, I = 512, 768
    x, w = rnd(M, K, seed=5), rnd(2 * I, K, scale=0.05, seed=6)
    out = torch.empty(M, I, dtype=torch.bfloat16, device=DEV)
    save = torch.zeros(M + 10, 2 * I, dtype=torch.bfloat16, device=DEV)
    lo, hi = M // 3, M
    ops.gemm(x, w, out, epi=ops.EPI_SWIGLU, save=save, save_lo=lo, save_hi=hi, save_dst=7)
    exp_out = torch.empty_like(out, dtype=torch.float32)
    exp_save = torch.zeros(M + 10, 2 * I)
    ref.gemm(x.float().cpu(), w.float().cpu(), exp_out.cpu(), epi=ref.EPI_SWIGLU)
    acc = x.float() @ w.float().t()
    g, u = ref.deinterleave64(acc)
    torch.testing.assert_close(out.float(), torch.nn.functional.silu(g) * u, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(save[7:7 + hi - lo].float(), acc[lo:hi], rtol=2e-2, atol=2e-2)
    assert save[:7].abs().sum() == 0


@pytest.mark.parametrize("T,K,P,R,slots", [(1, 4096, 3, 16, 2), (16, 4096, 3, 16, 2), (16, 14336, 1, 16, 2),
                                             (64, 4096, 2, 16, 4), (13, 1000, 3, 8, 3), (40, 4096, 1, 64, 2)])
def test_lora_shrink_decode_sizes(T, K, P, R, slots):
    """The decode shrink (K split over a CTA's warps): every row's own slot
    segment against fp32, the other slots' columns and the padding zero."""
    seg = -(-P * R // 64) * 64
    x = rnd(T, K, seed=61)
    A = rnd(slots, P * R, K, scale=0.05, seed=62)
    sid = torch.randint(-1, slots, (T,), device=DEV, dtype=torch.int32, generator=torch.Generator(device=DEV).manual_seed(63))
    Z = torch.full((T, slots * seg), 9.0, dtype=torch.bfloat16, device=DEV)
    ops.lora_shrink(x, A, sid, Z, seg)
    Zr = torch.empty_like(Z).cpu()
    ref.lora_shrink(x.cpu().float(), A.cpu().float(), sid.cpu(), Zr, seg)
    torch.testing.assert_close(Z.float().cpu(), Zr.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M,N,K,graph", [(16, 6144, 4096, False), (16, 6144, 4096, True), (300, 1024, 512, False),
                                          (2048, 4096, 1024, True)])
def test_gemm_overlapping_the_shrink(M, N, K, graph):
    """A LoRA GEMM launched to overlap the shrink right before it (programmatic
    dependent launch: base K blocks first, a wait before the LoRA blocks) gives
    the serialised result, eagerly and replayed from a CUDA graph; shapes cover
    the swapped decode path, a one-CTA tile and the CTA-pair kernel."""
    slots, PR, seg = 2, 48, 64
    x, w = rnd(M, K, seed=71), rnd(N, K, scale=0.05, seed=72)
    A = rnd(slots, PR, K, scale=0.05, seed=73)
    B2 = rnd(N, slots * seg, scale=0.05, seed=74)
    sid = (torch.arange(M, device=DEV, dtype=torch.int32) % slots)
    mask = torch.full(((M + 127) // 128,), 3, dtype=torch.int32, device=DEV)
    Z = torch.empty(M, slots * seg, dtype=torch.bfloat16, device=DEV)
    ref_out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.lora_shrink(x, A, sid, Z, seg)
    ops.gemm(x, w, ref_out, z=Z, b2=B2, tile_slots=mask, lora_seg=seg)
    out = torch.zeros_like(ref_out)
    Z2 = torch.zeros_like(Z)

    def run():
        ops.lora_shrink(x, A, sid, Z2, seg)
        ops.gemm(x, w, out, z=Z2, b2=B2, tile_slots=mask, lora_seg=seg, after_shrink=True)

    if graph:
        run()                                  # warm (allocations, tensor maps)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run()
        out.zero_()
        Z2.zero_()
        for _ in range(3):
            g.replay()
    else:
        for _ in range(3):
            run()
    torch.cuda.synchronize()
    assert ops.check_device_error() == 0
    torch.testing.assert_close(Z2, Z, rtol=0, atol=0)
    torch.testing.assert_close(out.float(), ref_out.float(), rtol=0, atol=0)


def test_gemm_lora_expand_segmented():
    M, N, K, slots, P, R = 300, 384, 256, 4, 3, 16
    seg = 64
    x, w = rnd(M, K, seed=7), rnd(N, K, scale=0.05, seed=8)
    A = rnd(slots, P * R, K, scale=0.05, seed=9)
    B2 = rnd(N, slots * seg, scale=0.05, seed=10)
    slot_ids = torch.randint(-1, slots, (M,), device=DEV, dtype=torch.int32)
    slot_ids, _ = slot_ids.sort()
    Z = torch.empty(M, slots * seg, dtype=torch.bfloat16, device=DEV)
    ops.lora_shrink(x, A, slot_ids, Z, seg)
    Zr = torch.empty_like(Z).cpu()
    ref.lora_shrink(x.cpu().float(), A.cpu().float(), slot_ids.cpu(), Zr, seg)
    torch.testing.assert_close(Z.float().cpu(), Zr.float(), rtol=2e-2, atol=2e-2)
    nt = -(-M // 128)
    mask = torch.zeros(nt, dtype=torch.int32)
    for t in range(nt):
        for s in slot_ids[t * 128:(t + 1) * 128].cpu().unique().tolist():
            if s >= 0:
                mask[t] |= 1 << s
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, out, z=Z, b2=B2, tile_slots=mask.to(DEV), lora_seg=seg)
    exp = x.float() @ w.float().t() + Z.float() @ B2.float().t()
    torch.testing.assert_close(out.float(), exp, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("D", [256, 1024, 4096, 5120])
def test_rms_norm_fused_add_save(D):
    T = 37
    x, r, w = rnd(T, D, seed=11), rnd(T, D, seed=12), rnd(D, scale=0.1, seed=13) + 1
    out = torch.empty_like(x)
    res = r.clone()
    save = torch.zeros(40, D, dtype=torch.bfloat16, device=DEV)
    ops.rms_norm(x, w, out, 1e-6, residual=res, save=save, save_lo=30, save_hi=37, save_dst=2)
    ro, rr = torch.empty(T, D), r.float().cpu().to(torch.bfloat16)
    ref.rms_norm(x.cpu(), rr, w.cpu(), ro, 1e-6)
    torch.testing.assert_close(res.cpu(), rr)
    torch.testing.assert_close(out.float().cpu(), ro, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(save[2:9].cpu(), rr[30:37])


@pytest.mark.parametrize("qk_norm", [False, True])
def test_qk_norm_rope_cache(qk_norm):
    T, Hq, Hkv, bs = 45, 8, 2, 16
    qkv = rnd(T, (Hq + 2 * Hkv) * 128, seed=14)
    pos = torch.randint(0, 900, (T,), device=DEV)
    cs = ref.rope_cos_sin_table(1024, 128, 1e6, device=DEV)
    qn = rnd(128, scale=0.1, seed=15) + 1 if qk_norm else None
    kn = rnd(128, scale=0.1, seed=16) + 1 if qk_norm else None
    kc = torch.zeros(8, Hkv, bs, 128, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(8 * bs, device=DEV)[:T]
    a = qkv.clone()
    ops.qk_norm_rope_cache(a, pos, cs, qn, kn, 1e-6, Hq, Hkv, kc, vc, slots)
    b = qkv.cpu().clone()
    kr, vr = torch.zeros_like(kc).cpu(), torch.zeros_like(vc).cpu()
    ref.qk_norm_rope_cache(b, pos.cpu(), cs.cpu(), None if qn is None else qn.cpu(),
                           None if kn is None else kn.cpu(), 1e-6, Hq, Hkv, kr, vr, slots.cpu())
    torch.testing.assert_close(a.float().cpu(), b.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(kc.float().cpu(), kr.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(vc.cpu(), vr)


def _paged_setup(lens, qlens, Hq, Hkv, bs, seed=0):
    nb = sum(-(-l // bs) for l in lens) + 4
    kc = rnd(nb, Hkv, bs, 128, seed=seed)
    vc = rnd(nb, Hkv, bs, 128, seed=seed + 1)
    perm = torch.randperm(nb).tolist()
    maxb = max(-(-l // bs) for l in lens)
    bt = torch.zeros(len(lens), maxb, dtype=torch.int32)
    k = 0
    for i, l in enumerate(lens):
        n = -(-l // bs)
        bt[i, :n] = torch.tensor(perm[k:k + n])
        k += n
    cu = [0]
    for q in qlens:
        cu.append(cu[-1] + q)
    q = rnd(cu[-1], Hq * 128, seed=seed + 2)
    return kc, vc, bt.to(DEV), torch.tensor(cu, dtype=torch.int32, device=DEV), \
        torch.tensor(lens, dtype=torch.int32, device=DEV), q


@pytest.mark.parametrize("bs", [16, 64, 128, 256, 48])
@pytest.mark.parametrize("Hq,Hkv", [(8, 2), (4, 4)])
def test_paged_prefill(bs, Hq, Hkv):
    """Block sizes that tile 128 keys run the tcgen05 kernel, 48 the warp-level one."""
    lens = [1, 63, 64, 65, 200, 513, 1100]
    qlens = [1, 63, 10, 65, 200, 100, 700]
    kc, vc, bt, cu, ctx, q = _paged_setup(lens, qlens, Hq, Hkv, bs)
    assert ops.prefill_uses_tc(bs) == (bs != 48)
    tiles = torch.tensor(ops.prefill_tiles(cu.tolist()), dtype=torch.int32, device=DEV)
    out = torch.zeros(q.shape[0], Hq * 128, dtype=torch.bfloat16, device=DEV)
    ops.paged_prefill(q, kc, vc, bt, cu, ctx, tiles, out, Hq, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    assert ops.check_device_error() == 0
    exp = torch.zeros_like(out, dtype=torch.float32).cpu()
    ref.paged_prefill(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), cu.cpu(), ctx.cpu(), exp, Hq, 1 / math.sqrt(128))
    torch.testing.assert_close(out.float().cpu(), exp, rtol=2e-2, atol=2e-2)


def test_paged_prefill_tc_matches_warp_kernel():
    """Both prefill kernels on one batch (64-key pages): same outputs to bf16 rounding."""
    lens, qlens = [300, 1024, 77], [300, 512, 77]
    kc, vc, bt, cu, ctx, q = _paged_setup(lens, qlens, 32, 8, 64)
    tiles = torch.tensor(ops.prefill_tiles(cu.tolist()), dtype=torch.int32, device=DEV)
    a = torch.zeros(q.shape[0], 32 * 128, dtype=torch.bfloat16, device=DEV)
    b = torch.zeros_like(a)
    nat = ops._native()
    nat.paged_prefill_tc(q, kc, vc, bt, cu, ctx, tiles, a, 32, 1 / math.sqrt(128))
    nat.paged_prefill(q, kc, vc, bt, cu, ctx, tiles, b, 32, 1 / math.sqrt(128), ops.PREFILL_TILE)
    torch.cuda.synchronize()
    assert ops.check_device_error() == 0
    torch.testing.assert_close(a.float(), b.float(), rtol=1.6e-2, atol=1.6e-2)


def _packed_qkv(lens, Hq, Hkv, seed, pad=8):
    """q/k/v as strided head views of one fused [n, (Hq+2Hkv)*128] bf16 buffer
    (the trainer's layout), samples packed back to back, padding rows at the end."""
    n = -(-sum(lens) // pad) * pad
    qkv = rnd(n, (Hq + 2 * Hkv) * 128, seed=seed)
    ql, kl = Hq * 128, Hkv * 128
    q = qkv[:, :ql].view(n, Hq, 128)
    k = qkv[:, ql:ql + kl].view(n, Hkv, 128)
    v = qkv[:, ql + kl:].view(n, Hkv, 128)
    starts = [sum(lens[:i]) for i in range(len(lens))]
    return q, k, v, starts, n


@pytest.mark.parametrize("Hq,Hkv", [(8, 2), (4, 4), (32, 8)])
def test_attn_bwd_varlen_gqa(Hq, Hkv):
    lens = [1, 37, 64, 65, 130, 200, 513] if Hq <= 8 else [512, 512, 300, 7]
    q, k, v, starts, n = _packed_qkv(lens, Hq, Hkv, seed=31)
    g = torch.Generator(device=DEV).manual_seed(32)
    d_o = torch.randn(n, Hq * 128, generator=g, device=DEV)
    tiles = ops.dense_attn_tiles(starts, lens, DEV)
    scale = 1 / math.sqrt(128)
    dq, dk, dv = ops.attn_bwd(q, k, v, d_o, tiles, scale)
    eq = torch.zeros(n, Hq, 128)
    ek, ev = torch.zeros(n, Hkv, 128), torch.zeros(n, Hkv, 128)
    ref.dense_attn_bwd(q.cpu(), k.cpu(), v.cpu(), d_o.cpu().view(n, Hq, 128), tiles.cpu(), scale, eq, ek, ev)
    for got, exp in ((dq, eq), (dk, ek), (dv, ev)):
        got = got.cpu()
        err = (got - exp).abs().max() / exp.abs().max()
        assert err < 2e-2, float(err)
    used = sum(lens)
    assert dq[used:].abs().max() == 0 and dk[used:].abs().max() == 0
    # deterministic: a second run is bit-identical
    dq2, dk2, dv2 = ops.attn_bwd(q, k, v, d_o, tiles, scale)
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)


@pytest.mark.parametrize("mask", [7, 4])
def test_attn_bwd_rope_epilogue_into_dqkv(mask):
    """RoPE backward + bf16 stores into the fused d(qkv) rows (the trainer's
    call) == the fp32 kernel outputs rotated back by the reference."""
    Hq, Hkv = 8, 2
    lens = [5, 64, 130, 77]
    q, k, v, starts, n = _packed_qkv(lens, Hq, Hkv, seed=35)
    g = torch.Generator(device=DEV).manual_seed(36)
    d_o = torch.randn(n, Hq * 128, generator=g, device=DEV)
    pos = torch.cat([torch.arange(ln) for ln in lens] + [torch.zeros(n - sum(lens), dtype=torch.long)]).to(DEV)
    from deltaserve_vllm_b200.models.rope import cos_sin
    cos, sin = cos_sin(pos, 128, 500000.0)
    tiles = ops.dense_attn_tiles(starts, lens, DEV)
    scale = 1 / math.sqrt(128)
    dq0, dk0, dv0 = ops.attn_bwd(q, k, v, d_o, tiles, scale)
    dqkv = torch.full((n, (Hq + 2 * Hkv) * 128), 7.0, dtype=torch.bfloat16, device=DEV)
    dq, dk, dv = ops.attn_bwd(q, k, v, d_o, tiles, scale, rope=(cos, sin), dqkv=dqkv, bf16_mask=mask)
    eq, ek = ref.rope_bwd(dq0.cpu(), cos.cpu(), sin.cpu()), ref.rope_bwd(dk0.cpu(), cos.cpu(), sin.cpu())
    used = sum(lens)
    ql, kl = Hq * 128, Hkv * 128
    torch.testing.assert_close(dqkv[:used, ql + kl:].float().cpu(), dv0[:used].reshape(used, kl).cpu(),
                               rtol=1e-2, atol=1e-2)
    if mask == 7:
        assert dq is None and dk is None and dv is None
        torch.testing.assert_close(dqkv[:used, :ql].float().cpu(), eq[:used].reshape(used, ql), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(dqkv[:used, ql:ql + kl].float().cpu(), ek[:used].reshape(used, kl),
                                   rtol=1e-2, atol=1e-2)
    else:
        torch.testing.assert_close(dq.cpu(), eq, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(dk.cpu(), ek, rtol=1e-5, atol=1e-5)
        assert (dqkv[:, :ql + kl] == 7.0).all()          # untouched
    assert (dqkv[used:] == 7.0).all()                       # rows past the samples untouched


@pytest.mark.parametrize("Hq,Hkv,lse_from_fwd,many", [(8, 2, True, False), (4, 4, False, False),
                                                      (32, 8, True, False), (32, 8, True, True)])
def test_attn_bwd_tc_varlen_gqa(Hq, Hkv, lse_from_fwd, many):
    """tcgen05 attention backward (dQ pass + dK/dV pass) against the fp32
    reference, elementwise; the forward's statistics either come from the
    tcgen05 forward (the trainer's path) or are recomputed inside attn_bwd.
    Few (key tile, KV head) pairs run the dK/dV pass split by query head
    (partials + finish kernel); ``many`` has enough of them for one pass."""
    lens = [1, 37, 64, 65, 130, 200, 513] if Hq <= 8 else ([512] * 6 if many else [512, 512, 300, 7])
    q, k, v, starts, n = _packed_qkv(lens, Hq, Hkv, seed=41)
    g = torch.Generator(device=DEV).manual_seed(42)
    d_o = torch.randn(n, Hq * 128, generator=g, device=DEV).to(torch.bfloat16)
    tiles = ops.dense_attn_tiles(starts, lens, DEV)
    t128 = ops.dense_attn_tiles(starts, lens, DEV, bm=128)
    scale = 1 / math.sqrt(128)
    o = lse = None
    if lse_from_fwd:
        o = torch.zeros(n, Hq * 128, dtype=torch.bfloat16, device=DEV)
        lse = torch.zeros(Hq, n, device=DEV)
        ops.attn_fwd_dense(q, k, v, tiles, scale, o, tiles128=t128, lse=lse)
    dq, dk, dv = ops.attn_bwd(q, k, v, d_o, tiles, scale, o=o, lse=lse, tiles128=t128)
    torch.cuda.synchronize()
    assert ops.check_device_error() == 0
    eq = torch.zeros(n, Hq, 128)
    ek, ev = torch.zeros(n, Hkv, 128), torch.zeros(n, Hkv, 128)
    ref.dense_attn_bwd(q.cpu(), k.cpu(), v.cpu(), d_o.float().cpu().view(n, Hq, 128), tiles.cpu(), scale, eq, ek, ev)
    used = sum(lens)
    for got, exp in ((dq, eq), (dk, ek), (dv, ev)):
        got = got.cpu()[:used]
        exp = exp[:used]
        tol = 2e-2 * exp.abs().max()
        assert (got - exp).abs().max() < tol, float((got - exp).abs().max() / exp.abs().max())
        rel = (got - exp).norm() / exp.norm()
        assert rel < 1e-2, float(rel)
    if used < n:
        assert dq[used:].abs().max() == 0 and dk[used:].abs().max() == 0
    dq2, dk2, dv2 = ops.attn_bwd(q, k, v, d_o, tiles, scale, o=o, lse=lse, tiles128=t128)
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)   # deterministic


def test_attn_bwd_tc_rope_epilogue_matches_warp_kernels():
    """The trainer's call (RoPE backward, bf16 stores into d(qkv)) on both
    backward implementations: same values to bf16 rounding."""
    Hq, Hkv = 8, 2
    lens = [5, 64, 130, 77, 300]
    q, k, v, starts, n = _packed_qkv(lens, Hq, Hkv, seed=45)
    g = torch.Generator(device=DEV).manual_seed(46)
    d_o = torch.randn(n, Hq * 128, generator=g, device=DEV).to(torch.bfloat16)
    pos = torch.cat([torch.arange(ln) for ln in lens] + [torch.zeros(n - sum(lens), dtype=torch.long)]).to(DEV)
    from deltaserve_vllm_b200.models.rope import cos_sin
    cos, sin = cos_sin(pos, 128, 500000.0)
    tiles = ops.dense_attn_tiles(starts, lens, DEV)
    t128 = ops.dense_attn_tiles(starts, lens, DEV, bm=128)
    scale = 1 / math.sqrt(128)
    a = torch.full((n, (Hq + 2 * Hkv) * 128), 7.0, dtype=torch.bfloat16, device=DEV)
    b = a.clone()
    ops.attn_bwd(q, k, v, d_o.float(), tiles, scale, rope=(cos, sin), dqkv=a, bf16_mask=7)
    ops.attn_bwd(q, k, v, d_o, tiles, scale, rope=(cos, sin), dqkv=b, bf16_mask=7, tiles128=t128)
    torch.cuda.synchronize()
    assert ops.check_device_error() == 0
    used = sum(lens)
    torch.testing.assert_close(b[:used].float(), a[:used].float(), rtol=3e-2, atol=3e-2)
    assert (b[used:] == 7.0).all()


@pytest.mark.parametrize("M,K,I", [(300, 512, 640), (2048, 1024, 4608)])
def test_gemm_swiglu_bwd_epilogue(M, K, I):
    """d(act) GEMM (MN-major, with the LoRA K block) whose epilogue applies the
    SwiGLU backward == fp32 product then the SwiGLU backward reference (the
    second shape has enough 256 x 256 tiles for the CTA-pair kernel)."""
    a = rnd(M, K, seed=40)
    w = rnd(K, I, scale=0.05, seed=41)
    gu = rnd(M, 2 * I, seed=42)
    z = rnd(M, 64, seed=43)
    b2 = rnd(64, I, scale=0.05, seed=44)
    ts = torch.ones((M + 127) // 128, dtype=torch.int32, device=DEV)
    out = torch.empty(M, 2 * I, dtype=torch.bfloat16, device=DEV)
    act = torch.empty(M, I, dtype=torch.bfloat16, device=DEV)
    ops.gemm(a, w, out, b_mn=True, epi=ops.EPI_SWIGLU_BWD, z=z, b2=b2, tile_slots=ts, lora_seg=64,
             aux=gu, aux_out=act)
    exp = torch.empty(M, 2 * I)
    eact = torch.empty(M, I)
    ref.gemm(a.cpu(), w.cpu(), exp, True, ops.EPI_SWIGLU_BWD, z.cpu(), b2.cpu(), ts.cpu(), 64,
             aux=gu.cpu(), aux_out=eact)
    torch.testing.assert_close(out.float().cpu(), exp, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(act.float().cpu(), eact, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("Hq,Hkv", [(8, 2), (32, 8)])
def test_attn_fwd_dense(Hq, Hkv):
    lens = [3, 64, 129, 500]
    q, k, v, starts, n = _packed_qkv(lens, Hq, Hkv, seed=33)
    tiles = ops.dense_attn_tiles(starts, lens, DEV)
    out = torch.zeros(n, Hq * 128, dtype=torch.bfloat16, device=DEV)
    ops.attn_fwd_dense(q, k, v, tiles, 1 / math.sqrt(128), out)
    exp = torch.zeros(n, Hq * 128)
    ref.dense_attn_fwd(q.cpu(), k.cpu(), v.cpu(), tiles.cpu(), 1 / math.sqrt(128), exp)
    torch.testing.assert_close(out.float().cpu(), exp, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("Hq,Hkv", [(8, 2), (32, 8)])
def test_attn_fwd_dense_tc_with_stats(Hq, Hkv):
    """tcgen05 dense forward: O, base-2 row log-sum-exp and rowsum(dO * O) against fp32."""
    lens = [3, 64, 129, 500, 1000]
    q, k, v, starts, n = _packed_qkv(lens, Hq, Hkv, seed=35)
    tiles = ops.dense_attn_tiles(starts, lens, DEV, bm=128)
    g = torch.Generator(device=DEV).manual_seed(36)
    d_o = torch.randn(n, Hq * 128, generator=g, device=DEV)
    out = torch.zeros(n, Hq * 128, dtype=torch.bfloat16, device=DEV)
    lse = torch.zeros(Hq, n, device=DEV)
    dd = torch.zeros(Hq, n, device=DEV)
    scale = 1 / math.sqrt(128)
    ops.attn_fwd_dense(q, k, v, None, scale, out, tiles128=tiles, lse=lse, d_o=d_o, dd=dd)
    torch.cuda.synchronize()
    assert ops.check_device_error() == 0
    exp = torch.zeros(n, Hq * 128)
    else_, edd = torch.zeros(Hq, n), torch.zeros(Hq, n)
    ref.dense_attn_fwd(q.cpu(), k.cpu(), v.cpu(), tiles.cpu(), scale, exp)
    ref.dense_attn_stats(q.cpu(), k.cpu(), v.cpu(), tiles.cpu(), scale, else_, d_o.cpu(), edd)
    torch.testing.assert_close(out.float().cpu(), exp, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(lse.cpu(), else_, rtol=1e-3, atol=2e-3)
    # dd sums 128 products of O (bf16-level error) and dO ~ N(0, 1)
    torch.testing.assert_close(dd.cpu(), edd, rtol=2e-2, atol=5e-2)


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_paged_decode(G):
    Hkv, bs = 2, 64
    Hq = G * Hkv
    lens = [1, 64, 65, 700, 2049, 33]
    kc, vc, bt, _, ctx, _ = _paged_setup(lens, [1] * len(lens), Hq, Hkv, bs)
    q = rnd(len(lens), Hq * 128, seed=21)
    out = torch.zeros(len(lens), Hq * 128, dtype=torch.bfloat16, device=DEV)
    splits, kps = ops.decode_splits(len(lens), Hkv, max(lens))
    po = torch.empty(len(lens) * Hq * splits * 128, device=DEV)
    pml = torch.empty(len(lens) * Hq * splits * 2, device=DEV)
    ops.paged_decode(q, kc, vc, bt, ctx, out, Hq, 1 / math.sqrt(128), po, pml, splits, kps)
    exp = torch.zeros(len(lens), Hq * 128)
    ref.paged_decode(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), ctx.cpu(), exp, Hq, 1 / math.sqrt(128))
    torch.testing.assert_close(out.float().cpu(), exp, rtol=2e-2, atol=2e-2)


def test_embedding_vocab_parallel():
    table = rnd(100, 256, seed=22)
    ids = torch.tensor([0, 5, 99, 100, 150, 210], device=DEV)
    out = torch.empty(6, 256, dtype=torch.bfloat16, device=DEV)
    ops.embedding(ids, table, out, 100)
    exp = torch.zeros(6, 256, dtype=torch.bfloat16)
    ref.embedding(ids.cpu(), table.cpu(), exp, 100)
    torch.testing.assert_close(out.cpu(), exp)


def test_cross_entropy():
    R, V = 33, 50000
    logits = rnd(R, V, scale=3.0, dtype=torch.float32, seed=23)
    tgt = torch.randint(0, V, (R,), device=DEV)
    tgt[3] = -1
    loss = torch.empty(R, device=DEV)
    grad = torch.empty(R, V, dtype=torch.bfloat16, device=DEV)
    ops.ce_fwd_bwd(logits, tgt, loss, grad, 0.25)
    l2, g2 = torch.empty(R), torch.empty(R, V, dtype=torch.bfloat16)
    ref.ce_fwd_bwd(logits.cpu(), tgt.cpu(), l2, g2, 0.25)
    torch.testing.assert_close(loss.cpu(), l2, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(grad.float().cpu(), g2.float(), rtol=2e-2, atol=1e-4)


def test_adamw_clip():
    L, seg = 5, 10000
    p = rnd(L * seg, dtype=torch.float32, seed=24)
    g = rnd(L * seg, scale=3.0, dtype=torch.float32, seed=25)
    m = torch.zeros_like(p); v = torch.zeros_like(p)
    ss = torch.empty(L, device=DEV)
    ops.seg_sumsq(g, seg, ss)
    pr, mr, vr = p.cpu().clone(), m.cpu().clone(), v.cpu().clone()
    ssr = torch.empty(L)
    ref.seg_sumsq(g.cpu(), seg, ssr)
    torch.testing.assert_close(ss.cpu(), ssr, rtol=1e-4, atol=1e-3)
    for step in (1, 2):
        ops.adamw(p, g, m, v, seg_len=seg, seg_sumsq_t=ss, max_norm=1.0, grad_scale=0.5, lr=1e-3,
                  wd=0.01, step=step)
        ref.adamw(pr, g.cpu(), mr, vr, seg, ssr, 1.0, 0.5, 1e-3, 0.9, 0.999, 1e-8, 0.01, step)
    torch.testing.assert_close(p.cpu(), pr, rtol=1e-5, atol=1e-6)


def test_lora_publish():
    N, R, K, slots = 384, 16, 256, 3
    A = rnd(3 * R, K, dtype=torch.float32, seed=26)
    Bt = rnd(R, N, dtype=torch.float32, seed=27)
    Ad = torch.zeros(slots, 3 * R, K, dtype=torch.bfloat16, device=DEV)
    B2 = torch.zeros(N, slots * 64, dtype=torch.bfloat16, device=DEV)
    ops.lora_publish(A, Ad[1], Bt, B2, 64, 128, 256, False, 2.0)
    Adr, B2r = torch.zeros_like(Ad).cpu(), torch.zeros_like(B2).cpu()
    ref.lora_publish(A.cpu(), Adr[1], Bt.cpu(), B2r, 64, 128, 256, False, 2.0)
    torch.testing.assert_close(Ad.cpu(), Adr)
    torch.testing.assert_close(B2.cpu(), B2r)


def test_sample_greedy():
    logits = rnd(7, 30000, dtype=torch.float32, seed=28)
    out = torch.empty(7, dtype=torch.int64, device=DEV)
    ops.sample(logits, torch.zeros(7, device=DEV), torch.arange(7, device=DEV), out)
    assert torch.equal(out, logits.argmax(-1))
    ops.sample(logits, torch.ones(7, device=DEV), torch.arange(7, device=DEV), out)
    assert ((out >= 0) & (out < 30000)).all()


def test_sample_topk_topp_logprobs():
    """Top-k / top-p restricted sampling: every sampled token lies in the kept
    set of the reference rules; top_k = 1 is the argmax; the log-probability
    is the chosen token's raw log-softmax."""
    R, V = 48, 32000
    logits = rnd(R, V, scale=3.0, dtype=torch.float32, seed=90)
    g = torch.Generator().manual_seed(91)
    topk = torch.randint(0, 60, (R,), generator=g).to(torch.int32)
    topk[:4] = 1
    topp = (torch.rand(R, generator=g) * 0.9 + 0.1)
    topp[4:8] = 1.0
    temps = torch.rand(R, generator=g) * 1.5 + 0.3
    out = torch.empty(R, dtype=torch.int64, device=DEV)
    lps = torch.empty(R, device=DEV)
    for trial in range(3):
        seeds = torch.arange(R, device=DEV) * 7919 + trial
        ops.sample(logits, temps.to(DEV), seeds, out, top_k=topk.to(DEV), top_p=topp.to(DEV), logprobs=lps)
        lc, oc = logits.cpu(), out.cpu()
        for r in range(R):
            z = lc[r] / float(temps[r])
            keep = ref.sample_keep_mask(z, int(topk[r]), min(1.0, float(topp[r]) + 1e-4))
            assert keep[oc[r]], (r, int(topk[r]), float(topp[r]))
        assert torch.equal(oc[:4], lc[:4].argmax(-1))
        exp_lp = torch.log_softmax(lc, -1).gather(1, oc.view(-1, 1)).view(-1)
        torch.testing.assert_close(lps.cpu(), exp_lp, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (16, 6144, 4096), (64, 4096, 14336), (100, 1024, 2048)])
def test_gemm_splitk_decode_shapes(M, N, K):
    a, b = rnd(M, K, seed=31), rnd(N, K, scale=0.05, seed=32)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm(a, b, out)
    torch.testing.assert_close(out.float(), a.float() @ b.float().t(), rtol=2e-2, atol=3e-2)
    o32 = torch.empty(M, N, dtype=torch.float32, device=DEV)
    ops.gemm(a, b, o32, epi=ops.EPI_F32)
    torch.testing.assert_close(o32, a.float() @ b.float().t(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("M", [3, 40])
def test_gemm_splitk_swiglu_lora_save(M):
    K, I, slots, seg = 4096, 1792, 2, 64
    x, w = rnd(M, K, seed=33), rnd(2 * I, K, scale=0.02, seed=34)
    A = rnd(slots, 2 * 16, K, scale=0.02, seed=35)
    B2 = rnd(2 * I, slots * seg, scale=0.05, seed=36)
    sid = torch.zeros(M, dtype=torch.int32, device=DEV)
    sid[M // 2:] = 1
    Z = torch.empty(M, slots * seg, dtype=torch.bfloat16, device=DEV)
    ops.lora_shrink(x, A, sid, Z, seg)
    mask = torch.tensor([3], dtype=torch.int32, device=DEV)
    out = torch.empty(M, I, dtype=torch.bfloat16, device=DEV)
    save = torch.zeros(M, 2 * I, dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, out, epi=ops.EPI_SWIGLU, z=Z, b2=B2, tile_slots=mask, lora_seg=seg,
             save=save, save_lo=1, save_hi=M, save_dst=0)
    acc = x.float() @ w.float().t() + Z.float() @ B2.float().t()
    g, u = ref.deinterleave64(acc)
    torch.testing.assert_close(out.float(), torch.nn.functional.silu(g) * u, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(save[:M - 1].float(), acc[1:M], rtol=2e-2, atol=3e-2)


def test_gemm_decode_gateup_full_width_swiglu():
    """The decode gate_up at Llama-3-8B width (224 output tiles of one M tile)
    against fp32."""
    M, K, I = 16, 4096, 14336
    x, w = rnd(M, K, seed=51), rnd(2 * I, K, scale=0.02, seed=52)
    out = torch.empty(M, I, dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, out, epi=ops.EPI_SWIGLU)
    g, u = ref.deinterleave64(x.float() @ w.float().t())
    torch.testing.assert_close(out.float(), torch.nn.functional.silu(g) * u, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("T,D", [(50, 4096), (9, 5120), (7, 1024), (33, 8192), (301, 128), (5, 96), (3, 200)])
def test_rms_norm_bwd_shapes(T, D):
    """Vector (one CTA per row), warp-per-row (q/k norms) and scalar paths."""
    x = rnd(T, D, seed=37)
    dy = rnd(T, D, dtype=torch.float32, seed=38)
    w = rnd(D, scale=0.1, seed=39) + 1
    add = rnd(T, D, dtype=torch.float32, seed=40)
    bf = torch.empty(T, D, dtype=torch.bfloat16, device=DEV)
    out = ops.rms_norm_bwd(x, dy, w, 1e-5, add=add, out_bf16=bf)
    exp = ref.rms_norm_bwd(x.cpu(), dy.cpu(), w.cpu(), 1e-5, add.cpu())
    torch.testing.assert_close(out.cpu(), exp, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(bf.float().cpu(), exp, rtol=1e-2, atol=1e-2)
    out2 = ops.rms_norm_bwd(x, dy, w, 1e-5)
    torch.testing.assert_close(out2.cpu(), ref.rms_norm_bwd(x.cpu(), dy.cpu(), w.cpu(), 1e-5, None),
                               rtol=1e-4, atol=1e-4)


def test_rms_norm_bwd_and_swiglu_bwd():
    T = 50
    I = 1792
    gu = rnd(T, 2 * I, seed=41)
    dact = rnd(T, I, dtype=torch.float32, seed=42)
    dgu = torch.empty(T, 2 * I, dtype=torch.bfloat16, device=DEV)
    act = torch.empty(T, I, dtype=torch.bfloat16, device=DEV)
    ops.swiglu_bwd(gu, dact, dgu, act)
    dgu_r, act_r = torch.empty(T, 2 * I, dtype=torch.bfloat16), torch.empty(T, I, dtype=torch.bfloat16)
    ref.swiglu_bwd(gu.cpu(), dact.cpu(), dgu_r, act_r)
    torch.testing.assert_close(dgu.float().cpu(), dgu_r.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(act.float().cpu(), act_r.float(), rtol=2e-2, atol=2e-2)


# ---------------------------------------------------------------- fused GEMM + all-reduce
@pytest.mark.parametrize("M,N,K,splits", [(1, 4096, 4096, 0), (16, 4096, 1792, 0), (200, 1024, 512, 0),
                                          (1000, 2048, 512, 0), (130, 512, 1024, 4), (7, 256, 4096, 0)])
def test_gemm_allreduce_single_rank(M, N, K, splits):
    """One rank: the kernel's push / owner-reduce / broadcast / wait phases all
    run against this GPU's own workspace; repeated calls exercise the flag and
    ticket resets."""
    from deltaserve_vllm_b200.parallel.peer import PeerWorkspace
    ws = PeerWorkspace(None, 1024 + 8, N)
    try:
        for it in range(3):
            a, b = rnd(M, K, seed=11 + it), rnd(N, K, scale=0.05, seed=12 + it)
            out = ops.gemm_ar(a, b, ws, force_splits=splits)
            exp = a.float() @ b.float().t()
            torch.testing.assert_close(out.float(), exp, rtol=2e-2, atol=3e-2)
        torch.cuda.synchronize()
    finally:
        ws.close()


def test_gemm_allreduce_single_rank_lora():
    from deltaserve_vllm_b200.parallel.peer import PeerWorkspace
    M, N, K, slots, P, R, seg = 150, 512, 256, 2, 1, 16, 64
    x, w = rnd(M, K, seed=21), rnd(N, K, scale=0.05, seed=22)
    A = rnd(slots, P * R, K, scale=0.05, seed=23)
    B2 = rnd(N, slots * seg, scale=0.05, seed=24)
    slot_ids = torch.randint(-1, slots, (M,), device=DEV, dtype=torch.int32).sort()[0]
    Z = torch.empty(M, slots * seg, dtype=torch.bfloat16, device=DEV)
    ops.lora_shrink(x, A, slot_ids, Z, seg)
    nt = -(-M // 128)
    mask = torch.zeros(nt, dtype=torch.int32)
    for t in range(nt):
        for s in slot_ids[t * 128:(t + 1) * 128].cpu().unique().tolist():
            if s >= 0:
                mask[t] |= 1 << s
    ws = PeerWorkspace(None, 256, N)
    try:
        out = ops.gemm_ar(x, w, ws, z=Z, b2=B2, tile_slots=mask.to(DEV), lora_seg=seg)
        exp = x.float() @ w.float().t() + Z.float() @ B2.float().t()
        torch.testing.assert_close(out.float(), exp, rtol=2e-2, atol=3e-2)
    finally:
        ws.close()


@pytest.mark.parametrize("M,N,K", [(5, 1024, 512), (64, 4096, 2048), (100, 768, 4096)])
def test_gemm_decode_swapped_lora(M, N, K):
    """Decode-sized GEMM (swapped operands: weights on the MMA's 128-row side)
    with the multi-LoRA expand over the slots of the batch."""
    slots, P, R, seg = 3, 1, 16, 64
    x, w = rnd(M, K, seed=31), rnd(N, K, scale=0.05, seed=32)
    A = rnd(slots, P * R, K, scale=0.05, seed=33)
    B2 = rnd(N, slots * seg, scale=0.05, seed=34)
    slot_ids = torch.randint(-1, slots, (M,), device=DEV, dtype=torch.int32).sort()[0]
    Z = torch.empty(M, slots * seg, dtype=torch.bfloat16, device=DEV)
    ops.lora_shrink(x, A, slot_ids, Z, seg)
    mask = torch.zeros(1, dtype=torch.int32)
    for s in slot_ids.cpu().unique().tolist():
        if s >= 0:
            mask[0] |= 1 << s
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, out, z=Z, b2=B2, tile_slots=mask.to(DEV), lora_seg=seg)
    exp = x.float() @ w.float().t() + Z.float() @ B2.float().t()
    torch.testing.assert_close(out.float(), exp, rtol=2e-2, atol=3e-2)
    plain = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm(x, w, plain)
    torch.testing.assert_close(plain.float(), x.float() @ w.float().t(), rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("M,N,K", [(300, 512, 384), (4096, 1024, 2048)])
def test_gemm_mn_major_with_lora_block(M, N, K):
    """MN-major GEMM with the adapter term as an extra K block (the backward's
    fused dX = dY . W + dZ . A)."""
    a, b = rnd(M, K, seed=41), rnd(K, N, scale=0.05, seed=42)
    z = torch.zeros(M, 64, dtype=torch.bfloat16, device=DEV)
    z[:, :48] = rnd(M, 48, seed=43)
    b2 = torch.zeros(64, N, dtype=torch.bfloat16, device=DEV)
    b2[:48] = rnd(48, N, scale=0.05, seed=44)
    ts = torch.ones(-(-M // 128), dtype=torch.int32, device=DEV)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    ops.gemm(a, b, out, b_mn=True, epi=ops.EPI_F32, z=z, b2=b2, tile_slots=ts, lora_seg=64, max_ctas=1 << 30)
    exp = a.float() @ b.float() + z.float() @ b2.float()
    torch.testing.assert_close(out, exp, rtol=2e-2, atol=3e-2)


def test_sample_gumbel_never_picks_a_negligible_token():
    """One dominant logit over a 128k vocabulary: with every other token 30
    nats below it, no sample over ~10k seeds may land elsewhere (the Gumbel
    noise is finite for every token)."""
    R, V = 64, 128256
    logits = torch.full((R, V), -30.0, dtype=torch.float32, device=DEV)
    hot = torch.randint(0, V, (R,), generator=torch.Generator().manual_seed(3)).to(DEV)
    logits[torch.arange(R, device=DEV), hot] = 0.0
    out = torch.empty(R, dtype=torch.int64, device=DEV)
    temps = torch.ones(R, device=DEV)
    misses = 0
    for trial in range(160):
        seeds = torch.arange(R, device=DEV) * 104729 + trial * 7
        ops.sample(logits, temps, seeds, out)
        misses += int((out != hot).sum())
    assert misses == 0, misses


def test_sample_topk_topp_with_masked_tokens():
    """Top-k / top-p still apply when some logits are -inf (tokens masked by
    min_tokens or logit_bias): the kept set matches the reference rules."""
    R, V = 24, 32000
    logits = rnd(R, V, scale=3.0, dtype=torch.float32, seed=93)
    g = torch.Generator().manual_seed(94)
    masked = torch.randint(0, V, (R, 40), generator=g)
    logits[torch.arange(R)[:, None].to(DEV), masked.to(DEV)] = float("-inf")
    topk = torch.randint(1, 30, (R,), generator=g).to(torch.int32)
    topp = torch.rand(R, generator=g) * 0.8 + 0.1
    topp[:6] = 1.0          # top-k alone
    topk[6:12] = 0          # top-p alone
    temps = torch.rand(R, generator=g) * 1.5 + 0.3
    out = torch.empty(R, dtype=torch.int64, device=DEV)
    for trial in range(4):
        seeds = torch.arange(R, device=DEV) * 31 + trial
        ops.sample(logits, temps.to(DEV), seeds, out, top_k=topk.to(DEV), top_p=topp.to(DEV))
        lc, oc = logits.cpu(), out.cpu()
        for r in range(R):
            z = lc[r] / float(temps[r])
            keep = ref.sample_keep_mask(z, int(topk[r]), min(1.0, float(topp[r]) + 1e-4))
            assert keep[oc[r]] and torch.isfinite(lc[r, oc[r]]), (r, int(topk[r]), float(topp[r]))


def _ce_ref(h, W, labels, n_valid):
    logits = h.float() @ W.float().t()
    lse = torch.logsumexp(logits, -1)
    lab = labels.clamp_min(0)
    loss = torch.where(labels >= 0, lse - logits.gather(1, lab[:, None]).view(-1), torch.zeros_like(lse))
    g = torch.softmax(logits, -1)
    g[torch.arange(h.shape[0], device=h.device), lab] -= 1.0
    g = torch.where((labels >= 0)[:, None], g / n_valid, torch.zeros_like(g))
    return lse, loss, g


@pytest.mark.parametrize("n,V,D", [(300, 5000, 512), (128, 16032, 1024)])
def test_ce_head_stats_and_grad_vs_fp32(n, V, D):
    """Vocabulary-slice cross-entropy: the statistics GEMM + merge + finalize
    give the fp32 log-sum-exp and loss, the gradient GEMM gives
    (softmax - onehot) / n_valid; with the vocabulary split in two slices (two
    ranks' shards on one GPU) the merged statistics are the same."""
    h = rnd(n, D, seed=61)
    W = rnd(V, D, scale=0.3, seed=62)
    labels = torch.randint(0, V, (n,), generator=torch.Generator().manual_seed(63)).to(DEV)
    labels[::7] = -1
    n_valid = int((labels >= 0).sum())
    lse_r, loss_r, g_r = _ce_ref(h, W, labels, n_valid)
    for split in (V, V // 2 + 13):
        slices = [(0, split), (split, V)] if split < V else [(0, V)]
        parts = torch.empty(len(slices), n, 3, device=DEV)
        for i, (a, b) in enumerate(slices):
            stats = torch.empty(n, 2 * (-(-(b - a) // 64)), device=DEV)
            tgt = torch.zeros(n, device=DEV)
            t = ops.ce_stats(h, W[a:b], labels, a, stats, tgt)
            ops.ce_merge(stats, t, tgt, parts[i])
        lse = torch.empty(n, device=DEV)
        loss = torch.empty(n, device=DEV)
        ops.ce_finalize(parts, labels, lse, loss)
        torch.testing.assert_close(lse, lse_r, rtol=1e-5, atol=2e-4)
        torch.testing.assert_close(loss, loss_r, rtol=1e-4, atol=2e-4)
    for c0, c1 in ((0, 1999), (1999, V)):
        dlog = torch.empty(n, c1 - c0, dtype=torch.bfloat16, device=DEV)
        ops.ce_grad(h, W[c0:c1], labels, c0, lse, 1.0 / n_valid, dlog)
        torch.testing.assert_close(dlog.float(), g_r[:, c0:c1], rtol=2e-2, atol=1e-6)
    assert ops.check_device_error() == 0


class _OneRank:
    size, rank = 1, 0

    def all_gather_object(self, obj):
        return [obj]

    def barrier(self):
        pass


@pytest.mark.parametrize("M,K,D", [(300, 192, 512), (1000, 640, 4096)])
def test_push_reduce_norm_one_rank(M, K, D):
    """The backward's row push + owner reduce + RMSNorm backward on one rank:
    the gathered bf16 rows and the fp32 rows equal
    rmsnorm_bwd(x, a @ b + add_push) + add_norm."""
    from deltaserve_vllm_b200.parallel.peer import BwdPeerWorkspace
    ws = BwdPeerWorkspace(_OneRank(), M + 8, D)
    try:
        a, b = rnd(M, K, seed=71), rnd(K, D, scale=0.05, seed=72)
        x, w = rnd(M, D, seed=73), rnd(D, scale=0.2, seed=74) + 1.0
        add_push = rnd(M, D, dtype=torch.float32, seed=75)
        add_norm = rnd(M, D, dtype=torch.float32, seed=76)
        for it in range(2):                      # twice: the counters reset themselves
            out = torch.zeros(M, D, device=DEV)
            ops.gemm_push(a, b, ws, add=add_push)
            got = ops.tp_reduce_rows(ws, M, it % 2, out, x=x, w=w, eps=1e-5, add=add_norm)
            torch.cuda.synchronize()
            dy = (a.float() @ b.float() + add_push).bfloat16().float()   # the partial travels in bf16
            exp = ref.rms_norm_bwd(x.float().cpu(), dy.cpu(), w.float().cpu(), 1e-5, add=add_norm.cpu()).to(DEV)
            # dy crosses the wire in bf16: a last-bit rounding difference of
            # the fp32 sum (tensor-core vs torch summation order) is allowed.
            torch.testing.assert_close(out, exp, rtol=2e-2, atol=3e-2)
            torch.testing.assert_close(got.float(), exp, rtol=2e-2, atol=3e-2)
        assert ops.check_device_error() == 0
    finally:
        ws.close()


class _DoubleComm:
    """Stand-in for a 2-rank communicator whose all-reduce doubles in place."""
    size, rank = 2, 0

    def all_reduce(self, t):
        t.mul_(2.0)
        return t


def test_bwd_comm_delay_exposes_a_missing_wait(monkeypatch):
    """DSERVE_BWD_COMM_DELAY spins the backward's side stream before each
    collective: a reader that skips reduce_end sees the old values every
    time, one that joins sees the reduced ones; DSERVE_BWD_COMM_SYNC joins
    at once."""
    from deltaserve_vllm_b200.models.configs import PRESETS
    from deltaserve_vllm_b200.models.lora_backward import LoraBackward, LoraMasters
    from deltaserve_vllm_b200.models.weights import init_weights
    arch = PRESETS["llama3-test"]
    w = init_weights(arch, seed=1, device=DEV)
    m = LoraMasters(arch, w.tp, 16, DEV)
    for env, joined in (({"DSERVE_BWD_COMM_DELAY": str(int(2e8))}, False), ({"DSERVE_BWD_COMM_SYNC": "1"}, True)):
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        bwd = LoraBackward(w, m, 2.0, comm=_DoubleComm())
        t = torch.ones(1 << 20, device=DEV)
        h = bwd.reduce_begin(t)
        early = t.clone()                      # no reduce_end: races the side stream
        LoraBackward.reduce_end(h, t.device)
        late = t.clone()
        torch.cuda.synchronize()
        assert float(late.min()) == 2.0
        assert float(early.max()) == (2.0 if joined else 1.0)
        for k in env:
            monkeypatch.delenv(k)


@pytest.mark.parametrize("T,M,PR,R,mode", [(4096, 4096, 48, 16, "qkv"), (1000, 3584, 32, 16, "gate_up"),
                                          (777, 512, 16, 16, "o"), (2048, 1792, 192, 64, "qkv")])
def test_gemm_wgrad_vs_fp32(T, M, PR, R, mode):
    """LoRA factor-gradient GEMMs over the token dimension: dA^T written
    transposed, and every projection's scaled dB^T scattered by output
    feature, against fp32 references."""
    a = rnd(T, M, seed=81)
    b = rnd(T, PR, seed=82)
    out = torch.zeros(PR, M, device=DEV)
    ops.gemm_wgrad(a, b, out, kind="t", n_valid=PR)
    prod = a.float().t() @ b.float()                       # [M, PR]
    torch.testing.assert_close(out, prod.t(), rtol=1e-3, atol=1e-2)
    interleave = mode == "gate_up"
    b1, b2 = (M // 2, 3 * M // 4) if mode == "qkv" else (M, M)
    bt = torch.zeros(R, M, device=DEV)
    ops.gemm_wgrad(a, b, bt, kind="bt", n_valid=PR, R=R, b1=b1, b2=b2, interleave=interleave, scale=0.5)
    exp = torch.zeros(R, M)
    ref.gemm_wgrad(a.cpu(), b.cpu(), exp, 1, PR, R, b1, b2, interleave, 0.5)
    torch.testing.assert_close(bt.cpu(), exp, rtol=1e-3, atol=1e-2)
    assert ops.check_device_error() == 0
