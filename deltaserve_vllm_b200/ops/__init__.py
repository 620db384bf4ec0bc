"""Hot ops of the engine.

Every function takes preallocated outputs (so the engine can keep persistent
buffers and capture CUDA graphs) and routes on the device of its first input:
CUDA tensors run the sm_100a kernels of ``ops/csrc`` (module ``_C``), CPU
tensors run the fp32 restatement in :mod:`.reference` — the oracle the tests
compare against. On a CUDA tensor a missing extension is an error, never a
silent fallback.
"""

from __future__ import annotations

import os

import torch

from . import reference as ref
from .reference import EPI_BF16, EPI_F32, EPI_SWIGLU, EPI_F32_ACCUM, EPI_SWIGLU_BWD  # noqa: F401

_EXT = None
_C_ERR: Exception | None = None
try:  # the in-tree build (python setup.py build_ext --inplace)
    import importlib as _il
    _EXT = _il.import_module(".ops._C", __name__.rsplit(".", 1)[0])
except Exception as e:  # pragma: no cover - depends on the build
    _C_ERR = e


def native_available() -> bool:
    return _EXT is not None


def native_ext():
    """The loaded extension module (None when it is not built)."""
    return _EXT


LAUNCHES = [0]  # kernels of this package launched so far (bench accounting)


def _native(kernels: int = 1):
    if _EXT is None:
        raise RuntimeError(
            "deltaserve_vllm_b200 CUDA extension is not built or failed to load "
            f"({_C_ERR!r}); run `python setup.py build_ext --inplace`")
    LAUNCHES[0] += kernels
    return _EXT


def check_device_error(clear: bool = True) -> int:
    """Error code written by a kernel whose bounded wait gave up (0 = none)."""
    if _EXT is None or not torch.cuda.is_available():
        return 0
    return int(_EXT.read_error(clear))


# ----------------------------------------------------------------- GEMM

def gemm(a, b, out, *, b_mn=False, epi=EPI_BF16, z=None, b2=None, tile_slots=None,
         lora_seg=0, save=None, save_lo=0, save_hi=0, save_dst=0, force_bn=0, max_ctas=0,
         aux=None, aux_out=None, after_shrink=False):
    """``out = a @ b.T`` (``b`` is [N, K]) or ``a @ b`` (``b_mn``: ``b`` is [K, N]),
    plus the segmented LoRA expand ``z @ b2.T`` and the epilogue ``epi``:
    bf16 / fp32 store, fp32 accumulate, SwiGLU over 64-interleaved gate/up
    columns, or (``EPI_SWIGLU_BWD``, MN-major ``b``) the SwiGLU backward: the
    product is d(act), ``aux`` the saved interleaved gate/up [M, 2N], ``out``
    receives their gradient [M, 2N] and ``aux_out`` (optional) the activation.
    ``save`` receives raw accumulator rows [save_lo, save_hi).
    ``max_ctas`` > number of SMs launches one CTA per tile (non-persistent).
    ``after_shrink``: the kernel right before this call in the stream is the
    :func:`lora_shrink` that wrote ``z`` (and nothing this GEMM reads came from
    a later-pending kernel): the GEMM is then launched to overlap it, streaming
    its base K blocks while the shrink runs and waiting for it only before the
    LoRA blocks (programmatic dependent launch)."""
    if a.is_cuda:
        _native().gemm(a, b, out, b_mn, epi, z, b2, tile_slots, lora_seg, save,
                       save_lo, save_hi, save_dst, force_bn, max_ctas, aux, aux_out,
                       bool(after_shrink and z is not None))
        return out
    return ref.gemm(a, b, out, b_mn, epi, z, b2, tile_slots, lora_seg, save, save_lo, save_hi,
                    save_dst, aux=aux, aux_out=aux_out)


def gemm_ag(ws, rows_per_rank, b, out, *, epi=EPI_BF16, z=None, b2=None, tile_slots=None, lora_seg=0,
            fresh=True, copy_once=True):
    """All-gather -> column-parallel GEMM over the ranks of ``ws`` (an
    :class:`~..parallel.peer.AGPeerWorkspace`): ``out[M, N] = A_all @ b.T``
    (+ the segmented LoRA expand ``z @ b2.T``; SwiGLU with ``EPI_SWIGLU``)
    where rank ``r``'s rows ``ws.local[:rows_per_rank]`` are rows
    ``[r * rows_per_rank, (r + 1) * rows_per_rank)`` of ``A_all``
    (``rows_per_rank`` a multiple of 128). Every rank's shard must be written
    before any rank calls this, and a shard rewritten only after every rank's
    call over it has finished. ``fresh``: the shards hold new rows since the
    last call (the copy-once gather starts over; ``False`` reuses the rows an
    earlier call of the same shards gathered)."""
    if copy_once:
        if fresh:
            ws.cnt.zero_()
        _native().gemm_ag(ws.maps, rows_per_rank, ws.world, ws.local, b, out, epi, z, b2, tile_slots, lora_seg,
                          ws.gathered, ws.cnt, ws.src, ws.rank)
    else:
        _native().gemm_ag(ws.maps, rows_per_rank, ws.world, ws.local, b, out, epi, z, b2, tile_slots, lora_seg,
                          None, None, None, ws.rank)
    return out


def lora_shrink_ag(ws, rows_per_rank, A, slot_ids, Z, seg, fresh=True, copy_once=True):
    """The LoRA shrink of the all-gathered input of :func:`gemm_ag`:
    ``Z[M, slots * seg]``, each row's own slot segment (``fresh`` and
    ``copy_once`` as for :func:`gemm_ag`; a following ``gemm_ag`` with
    ``fresh=False`` reuses the rows this call gathered)."""
    slots, pr, K = A.shape
    if copy_once:
        if fresh:
            ws.cnt.zero_()
        _native().lora_shrink_ag(ws.maps, rows_per_rank, ws.world, ws.local, A.reshape(slots * pr, K), slot_ids, Z,
                                 pr, seg, ws.gathered, ws.cnt, ws.src, ws.rank)
    else:
        _native().lora_shrink_ag(ws.maps, rows_per_rank, ws.world, ws.local, A.reshape(slots * pr, K), slot_ids, Z,
                                 pr, seg, None, None, None, ws.rank)
    return Z


def gemm_ar(a, b, ws, *, z=None, b2=None, tile_slots=None, lora_seg=0, force_splits=0, force_reducers=-1):
    """All-reduce over the ranks of ``ws`` (a :class:`~..parallel.peer.PeerWorkspace`)
    of ``a @ b.T`` (+ the segmented LoRA expand), in ONE kernel: the GEMM
    epilogue pushes bf16 partial tiles to their owner rank over peer memory,
    owners reduce and broadcast, every rank waits for its full result.
    Returns a [M, N] view of the workspace's output buffer (valid until the
    next call on the same workspace)."""
    if not a.is_cuda:
        raise RuntimeError("gemm_ar runs on CUDA tensors only")
    if not ws.fits(a.shape[0], b.shape[0]):
        raise ValueError(f"gemm_ar: [{a.shape[0]}, {b.shape[0]}] does not fit the workspace "
                         f"([{ws.max_rows}, {ws.n_cols}])")
    ws.calls += 1
    return _native().gemm_ar(a, b, z, b2, tile_slots, lora_seg, ws.table, ws.tile_cnt, ws.rank,
                             ws.world, ws.owned_cap, ws.max_rows, force_splits, force_reducers)


def linear(x, w, out=None, epi=EPI_BF16, **kw):
    if out is None:
        n = w.shape[0]
        if epi == EPI_SWIGLU:
            n //= 2
        dt = torch.float32 if epi in (EPI_F32, EPI_F32_ACCUM) else x.dtype
        out = torch.empty(x.shape[0], n, dtype=dt, device=x.device)
    return gemm(x, w, out, epi=epi, **kw)


# ----------------------------------------------------------------- norms / rope

def rms_norm(x, w, out, eps, *, residual=None, save=None, save_lo=0, save_hi=0, save_dst=0):
    """``out = rmsnorm(x [+ residual]) * w``; with ``residual`` the sum is written
    back into ``residual`` (the residual stream). ``save`` captures rows
    [save_lo, save_hi) of the (updated) stream."""
    if x.is_cuda:
        _native().rms_norm(x, residual, w, out, eps, save, save_lo, save_hi, save_dst)
        return out
    return ref.rms_norm(x, residual, w, out, eps, save, save_lo, save_hi, save_dst)


def qk_norm_rope_cache(qkv, positions, cos_sin, q_norm, k_norm, eps, num_heads, num_kv_heads,
                       k_cache=None, v_cache=None, slot_mapping=None):
    if qkv.is_cuda:
        _native().qk_norm_rope_cache(qkv, positions, cos_sin, q_norm, k_norm, eps, num_heads,
                                     num_kv_heads, k_cache, v_cache, slot_mapping)
        return
    ref.qk_norm_rope_cache(qkv, positions, cos_sin, q_norm, k_norm, eps, num_heads, num_kv_heads,
                           k_cache, v_cache, slot_mapping)


# ----------------------------------------------------------------- attention

PREFILL_TILE = 128      # queries per prefill tile (the tcgen05 kernel's M)
ATTN_TC = os.environ.get("DSV_ATTN_TC", "1") != "0"


def prefill_tiles(cu_q: list[int], bm: int = PREFILL_TILE) -> list[tuple[int, int]]:
    """(sequence, first query) of every ``bm``-query tile of a varlen batch,
    later queries first: under the causal mask they see the most keys, so
    the longest CTAs start first."""
    out = []
    for s in range(len(cu_q) - 1):
        n = cu_q[s + 1] - cu_q[s]
        for q0 in range(0, n, bm):
            out.append((s, q0))
    out.sort(key=lambda t: -t[1])
    return out


def prefill_uses_tc(block_size: int) -> bool:
    """The tcgen05 prefill kernel loads 128-key tiles as whole page boxes:
    the page size must divide 128 or be a multiple of it."""
    return ATTN_TC and (128 % block_size == 0 or block_size % 128 == 0) and block_size % 8 == 0


def paged_prefill(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, tile_info, out, num_heads,
                  scale):
    """Causal varlen attention of the new queries over their paged context;
    ``tile_info`` from :func:`prefill_tiles` (128-query tiles)."""
    if q.is_cuda:
        if prefill_uses_tc(k_cache.shape[2]):
            _native().paged_prefill_tc(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, tile_info,
                                       out, num_heads, scale)
        else:
            _native().paged_prefill(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, tile_info, out,
                                    num_heads, scale, PREFILL_TILE)
        return out
    return ref.paged_prefill(q, k_cache, v_cache, block_tables, cu_q, ctx_lens, out, num_heads, scale)


def decode_splits(batch: int, num_kv_heads: int, max_ctx: int, num_sms: int = 148) -> tuple[int, int]:
    """Split-KV factor so that batch x kv_heads x splits gives every SM about
    four CTAs (two resident at a time, 100 KB of shared memory each)."""
    want = max(1, (4 * num_sms) // max(1, batch * num_kv_heads))
    keys = max(64, -(-max_ctx // want))
    keys = -(-keys // 64) * 64
    return max(1, -(-max_ctx // keys)), keys


def paged_decode(q, k_cache, v_cache, block_tables, ctx_lens, out, num_heads, scale,
                 part_o=None, part_ml=None, splits=1, keys_per_split=0):
    if q.is_cuda:
        _native(2).paged_decode(q, k_cache, v_cache, block_tables, ctx_lens, out, part_o, part_ml,
                               num_heads, scale, splits, keys_per_split)
        return out
    return ref.paged_decode(q, k_cache, v_cache, block_tables, ctx_lens, out, num_heads, scale)


# ----------------------------------------------------------------- trainer attention

def dense_attn_tiles(starts, lens, device, bm: int = 64) -> torch.Tensor:
    """int32 [T, 3] = (first row, length, tile row) of every ``bm``-row tile of
    packed causal samples, ordered by tile row: the attention-backward kernels
    use that order to start their heaviest CTAs first."""
    rows = [(int(st), int(ln), t0) for t0 in range(0, max([int(x) for x in lens], default=0), bm)
            for st, ln in zip(starts, lens) if t0 < int(ln)]
    return torch.tensor(rows, dtype=torch.int32).reshape(-1, 3).to(device)


def attn_bwd(q, k, v, d_o, tiles, scale, *, rope=None, dqkv=None, bf16_mask=0, o=None, lse=None,
             tiles128=None, dd=None):
    """Gradients of causal varlen GQA attention over packed samples.

    ``q`` [n, Hq, 128] / ``k``, ``v`` [n, Hkv, 128] (bf16 on CUDA; row strides
    free, heads adjacent), ``d_o`` [n, Hq * 128], ``tiles`` from
    :func:`dense_attn_tiles`. ``rope = (cos, sin)`` ([n, 64] fp32) rotates dq
    and dk back through RoPE (gradients w.r.t. the pre-RoPE q / k). Bits of
    ``bf16_mask`` (1: dq, 2: dk, 4: dv) store those gradients as bf16 into the
    fused ``dqkv`` [n, (Hq + 2 Hkv) * 128] (q, k, v column blocks) instead of
    returning them. Returns (dq, dk, dv): fp32 [n, H, 128], or None for the
    ones written into ``dqkv``; rows outside every sample are zero in the fp32
    outputs and untouched in ``dqkv``.

    With ``tiles128`` (128-row tiles) the tcgen05 kernels run on CUDA. They
    take the forward output ``o`` [n, Hq*128] bf16 and its base-2 row
    log-sum-exp ``lse`` [Hq, >= n] (from :func:`attn_fwd_dense`); without
    them the tcgen05 forward recomputes both first. ``dd`` is optional
    scratch shaped like ``lse``."""
    n, hq, hd = q.shape
    hkv = k.shape[1]
    dev = q.device
    if bf16_mask and dqkv is None:
        raise ValueError("attn_bwd: bf16_mask needs dqkv")
    outs = [None if bf16_mask & (1 << i) else torch.zeros(n, h, hd, dtype=torch.float32, device=dev)
            for i, h in enumerate((hq, hkv, hkv))]
    cos, sin = rope if rope is not None else (None, None)
    if q.is_cuda and ATTN_TC and tiles128 is not None:
        g = d_o.reshape(n, hq * hd)
        if g.dtype != torch.bfloat16:
            g = g.to(torch.bfloat16)
        if o is None or lse is None:
            o = torch.empty(n, hq * hd, dtype=torch.bfloat16, device=dev)
            lse = torch.empty_like(dd) if dd is not None else torch.empty(hq, n, dtype=torch.float32, device=dev)
            _native().attn_fwd_dense_tc(q, k, v, tiles128, o, hq, hkv, scale, lse, None, None)
        if dd is None:
            dd = torch.empty_like(lse)
        _native(2).attn_bwd_tc(q, k, v, o, g, tiles128, lse, dd, outs[0], outs[1], outs[2], scale, cos, sin,
                               dqkv, bf16_mask)
        return tuple(outs)
    if q.is_cuda:
        lse = torch.empty(hq, n, dtype=torch.float32, device=dev)
        dd = torch.empty(hq, n, dtype=torch.float32, device=dev)
        do_bf = torch.empty(n, hq * hd, dtype=torch.bfloat16, device=dev)
        _native(2).attn_bwd(q, k, v, d_o.reshape(n, hq * hd).float(), tiles, lse, dd, do_bf, outs[0], outs[1],
                            outs[2], scale, cos, sin, dqkv, bf16_mask)
        return tuple(outs)
    full = [torch.zeros(n, h, hd, dtype=torch.float32) for h in (hq, hkv, hkv)]
    ref.dense_attn_bwd(q, k, v, d_o.reshape(n, hq, hd), tiles, scale, *full)
    if rope is not None:
        full[0] = ref.rope_bwd(full[0], *rope)
        full[1] = ref.rope_bwd(full[1], *rope)
    cols = (0, hq * hd, (hq + hkv) * hd)
    samples = ref._tile_samples(tiles)
    for i, t in enumerate(full):
        if bf16_mask & (1 << i):
            w = t.shape[1] * hd
            for st, ln in samples:
                dqkv[st:st + ln, cols[i]:cols[i] + w] = t[st:st + ln].reshape(ln, w).to(dqkv.dtype)
        else:
            outs[i].copy_(t.to(dev))
    return tuple(outs)


def attn_fwd_dense(q, k, v, tiles, scale, out, tiles128=None, lse=None, d_o=None, dd=None):
    """Causal varlen GQA attention over packed samples into ``out`` [n, >= Hq*128]
    (bf16 on CUDA); rows outside every sample are left untouched.

    With ``tiles128`` (:func:`dense_attn_tiles` with ``bm=128``) the tcgen05
    kernel runs, and can also write the base-2 row log-sum-exp into ``lse``
    and rowsum(dO * O) into ``dd`` (fp32 [Hq, >= n]; ``d_o`` fp32 [n, Hq*128])."""
    if q.is_cuda:
        if ATTN_TC and tiles128 is not None:
            _native().attn_fwd_dense_tc(q, k, v, tiles128, out, q.shape[1], k.shape[1], scale, lse, d_o, dd)
        else:
            if lse is not None or dd is not None:
                raise ValueError("attn_fwd_dense: statistics need the tcgen05 kernel (tiles128)")
            _native().attn_fwd_dense(q, k, v, tiles, out, scale)
        return out
    ref.dense_attn_fwd(q, k, v, tiles if tiles is not None else tiles128, scale, out)
    if lse is not None or dd is not None:
        ref.dense_attn_stats(q, k, v, tiles if tiles is not None else tiles128, scale, lse, d_o, dd)
    return out


# ----------------------------------------------------------------- LoRA / misc

def lora_shrink(x, A, slot_ids, Z, seg):
    if x.is_cuda:
        _native().lora_shrink(x, A, slot_ids, Z, seg)
        return Z
    return ref.lora_shrink(x, A, slot_ids, Z, seg)


def embedding(ids, table, out, v0=0):
    if ids.is_cuda:
        _native().embedding(ids, table, out, v0)
        return out
    return ref.embedding(ids, table, out, v0)


def embedding_peer(ids, ptable, out):
    """Full embedding rows on every rank from the vocabulary shards of all
    ranks (``ptable``: a :class:`~..parallel.peer.PeerTable`), read over peer
    memory; replaces ``embedding`` + the all-reduce of the partial rows."""
    _native().embedding_peer(ids, ptable.table, ptable.rows, ptable.vocab, out)
    return out


def ce_fwd_bwd(logits, targets, loss, grad=None, gscale=1.0):
    if logits.is_cuda:
        _native().ce_fwd_bwd(logits, targets, loss, grad, gscale)
        return
    ref.ce_fwd_bwd(logits, targets, loss, grad, gscale)


def seg_sumsq(g, seg_len, out):
    if g.is_cuda:
        _native(2).seg_sumsq(g, seg_len, out)
        return out
    ref.seg_sumsq(g, seg_len, out)
    return out


def adamw(p, g, m, v, *, seg_len, seg_sumsq_t=None, max_norm=0.0, grad_scale=1.0, lr=1e-4,
          b1=0.9, b2=0.999, eps=1e-8, wd=0.0, step=1):
    if p.is_cuda:
        _native(1).adamw(p, g, m, v, seg_len, seg_sumsq_t, max_norm, grad_scale, lr, b1, b2, eps, wd,
                        step)
        return
    ref.adamw(p, g, m, v, seg_len, seg_sumsq_t, max_norm, grad_scale, lr, b1, b2, eps, wd, step)


def lora_publish(A_src, A_dst, Bt_src, B2_dst, col0, b1, b2, interleave, scale):
    if A_src.is_cuda:
        _native().lora_publish(A_src, A_dst, Bt_src, B2_dst, col0, b1, b2, interleave, scale)
        return
    ref.lora_publish(A_src, A_dst, Bt_src, B2_dst, col0, b1, b2, interleave, scale)


def rms_norm_bwd(x, dy, w, eps, *, add=None, out=None, out_bf16=None):
    """fp32 gradient of ``rmsnorm(x) * w`` w.r.t. ``x`` given fp32 ``dy``
    (+ ``add``); optionally also written as bf16 into ``out_bf16``."""
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    if x.is_cuda:
        _native().rms_norm_bwd(x, dy.contiguous(), w, add, out, out_bf16, eps)
        return out
    ref.rms_norm_bwd(x, dy, w, eps, add, out, out_bf16)
    return out


def swiglu_bwd(gu, dact, dgu, act=None):
    """From saved interleaved gate/up (``gu``) and fp32 ``dact``: ``dgu`` (same
    interleave) and, optionally, the activation ``silu(g) * u``."""
    if gu.is_cuda:
        _native().swiglu_bwd(gu, dact.contiguous(), dgu, act)
        return
    ref.swiglu_bwd(gu, dact, dgu, act)


def sample(logits, temps, seeds, out, top_k=None, top_p=None, logprobs=None):
    """One token per row of fp32 ``logits``: greedy where ``temps`` <= 0, else
    Gumbel-max at the row's temperature (counter-based noise from ``seeds``),
    optionally restricted to the ``top_k`` largest logits (int32 per row, 0 =
    off) and then to the top-``top_p`` probability mass (fp32 per row, 1 =
    off). ``logprobs`` (fp32 per row) receives the chosen token's raw
    log-softmax."""
    if logits.is_cuda:
        _native().sample(logits, temps, seeds, out, top_k, top_p, logprobs)
        return out
    ref.sample(logits, temps, seeds, out, top_k, top_p, logprobs)
    return out


# ----------------------------------------------------------------- LM head + CE (vocabulary slices)

def ce_stats(h, w, labels, v0, stats, tgt, max_ctas=0) -> int:
    """Softmax statistics of ``logits = h @ w.T`` (``w``: vocabulary rows
    ``[v0, v0 + N)``) without storing the logits: per row and N tile
    (max, sum exp(logit - max)) into ``stats`` (fp32 [M, >= 2 * ceil(N / 64)],
    float pairs) and the label's logit into ``tgt`` (rows whose label is
    outside the slice keep their value). Returns the tiles per row."""
    if h.is_cuda:
        return int(_native().gemm_ce_stats(h, w, labels, int(v0), stats, tgt, int(max_ctas)))
    return ref.ce_stats(h, w, labels, int(v0), stats, tgt)


def ce_merge(stats, n_tiles, tgt, part):
    """part [M, 3] = (max, sum exp, label logit) of this vocabulary slice."""
    if part.is_cuda:
        _native().ce_merge(stats, int(n_tiles), tgt, part)
        return part
    return ref.ce_merge(stats, int(n_tiles), tgt, part)


def ce_finalize(parts, labels, lse, loss):
    """Across slices (``parts`` [slices, M, 3]): log-sum-exp per row and the
    loss ``lse - logit[label]`` (0 on rows without a label)."""
    if parts.is_cuda:
        _native().ce_finalize(parts, labels, lse, loss)
        return lse, loss
    return ref.ce_finalize(parts, labels, lse, loss)


def ce_grad(h, w, labels, v0, lse, scale, dlog, max_ctas=0):
    """bf16 ``dlog = (softmax - onehot) * scale`` for ``logits = h @ w.T``
    (``w``: vocabulary rows ``[v0, v0 + N)``), recomputed from ``lse``; zero
    rows where the label is -1."""
    if h.is_cuda:
        _native().gemm_ce_grad(h, w, labels, int(v0), lse, float(scale), dlog, int(max_ctas))
        return dlog
    return ref.ce_grad(h, w, labels, int(v0), lse, float(scale), dlog)


# ----------------------------------------------------------------- tensor-parallel backward over peer memory

def gemm_push(a, b, ws, *, z=None, b2=None, tile_slots=None, lora_seg=0, add=None, max_ctas=0):
    """``a @ b`` (``b`` MN-major [K, N]) plus the LoRA term, pushed as bf16
    partial rows to each 128-row block's owner rank in ``ws`` (a
    :class:`~..parallel.peer.BwdPeerWorkspace`); ``add`` (fp32 [M, N]) is
    added first. Nothing waits here: :func:`tp_reduce_rows` completes it."""
    _native().gemm_push(a, b, z, b2, tile_slots, lora_seg, ws.push_table, ws.rank, ws.world, ws.blocks_cap,
                        ws.ld, add, int(max_ctas))


def tp_reduce_rows(ws, M, buf, out, *, x=None, w=None, eps=0.0, add=None):
    """Finish a push: wait for this rank's owned row blocks, sum them, apply
    the RMSNorm backward of ``x`` / ``w`` (when given) plus ``add``, write the
    fp32 rows into ``out`` (owned rows only) and the bf16 rows into gather
    buffer ``buf`` (0 or 1) of every rank, then wait for the other ranks'
    rows. Returns this rank's gather buffer [M, N] (every row)."""
    ext = _native(3)
    D = ws.ld
    n_blocks = -(-M // 128)
    n_owned = -(-(n_blocks - ws.rank) // ws.world)
    ext.wait_counts(ws.cnt_addr, n_owned, ws.world * D, 0, 0, 0)
    ext.reduce_norm_bcast(ws.recv_addr, ws.rank, ws.world, ws.blocks_cap, D, M, D, x, w, float(eps), add, out,
                          ws.gather_tables[buf])
    ext.wait_counts(ws.gcnt_addr, n_blocks, 0, M, ws.world, ws.rank)
    return ws.gather_view(buf, M)


def gemm_wgrad(a, b, out, *, kind, n_valid, R=0, b1=0, b2=0, interleave=False, scale=1.0, max_ctas=0):
    """LoRA factor-gradient GEMM reducing over the token dimension (``a``
    [T, M], ``b`` [T, >= n_valid] bf16, both token-major). ``kind="t"``:
    ``out[N, M] = b^T a`` (fp32) for the first ``n_valid`` columns of ``b``;
    ``kind="bt"``: ``out[j, m] = scale * (a^T b)[m, p(m) * R + j]`` with the
    projection p(m) of output feature m (bounds ``b1`` / ``b2`` or 64-column
    interleave) — every projection's B gradient of a group in one pass."""
    k = {"t": 0, "bt": 1}[kind]
    if a.is_cuda:
        _native().gemm_wgrad(a, b, out, k, int(n_valid), int(R), int(b1), int(b2), bool(interleave), float(scale),
                             int(max_ctas))
        return out
    return ref.gemm_wgrad(a, b, out, k, int(n_valid), int(R), int(b1), int(b2), bool(interleave), float(scale))


# ----------------------------------------------------------------- fused optimizer of the replicated factors

def push_slices(g, lo, hi, ws):
    """Send elements [lo, hi) of the replicated gradient block ``g`` to their
    slice owners (``ws``: :class:`~..parallel.peer.OptPeerWorkspace`)."""
    _native().push_slices(g, int(lo), int(hi), ws.slice, ws.rank, ws.world, ws.push_table)


def fused_replicated_adamw(ws, params, grads, exp_avg, exp_avg_sq, seg_len, shard_sumsq, *, max_norm, lr, wd,
                           step, b1=0.9, b2=0.999, eps=1e-8, coef=None, total=None, sq=None):
    """Finish the replicated block's optimizer step once every rank pushed all
    of its gradients: sum the owned slice, exchange per-layer sums of squares
    (plus ``shard_sumsq``, this rank's unreplicated part), AdamW with
    per-layer clipping on the owned slice, updated values to every rank, then
    wait for the other owners' slices and copy them in. Returns the per-layer
    squared norms (for the unreplicated part's own AdamW)."""
    ext = _native(7)
    L = ws.layers
    ext.wait_counts(ws.cnt_push, 1, ws.world * ws.len, 0, 0, 0)
    sq = sq if sq is not None else torch.zeros(L, dtype=torch.float32, device=params.device)
    sq.zero_()
    ext.reduce_slice_sumsq(ws.recv_addr, ws.world, ws.slice, ws.first, ws.len, seg_len, grads, sq)
    ext.exchange_rows(sq, shard_sumsq, ws.rank, ws.world, ws.row_table)
    ext.wait_counts(ws.cnt_rows, 1, ws.world, 0, 0, 0)
    coef = coef if coef is not None else torch.empty(L, dtype=torch.float32, device=params.device)
    total = total if total is not None else torch.empty(L, dtype=torch.float32, device=params.device)
    ext.clip_coef(ws.rows, float(max_norm), coef, total)
    ext.adamw_slice_bcast(params, grads, exp_avg, exp_avg_sq, ws.first, ws.len, seg_len, coef, lr, b1, b2, eps,
                          wd, int(step), ws.rank, ws.world, ws.param_table)
    return total


def fused_replicated_finish(ws, params):
    """Wait for the other owners' updated slices and copy them into ``params``."""
    _native().wait_counts(ws.cnt_param, 1, ws.total - ws.len, 0, 0, 0)
    if ws.first > 0:
        params[:ws.first].copy_(ws.pstage[:ws.first])
    end = ws.first + ws.len
    if end < ws.total:
        params[end:ws.total].copy_(ws.pstage[end:ws.total])
