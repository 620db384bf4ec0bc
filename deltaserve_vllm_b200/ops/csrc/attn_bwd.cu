// Varlen causal GQA attention for the LoRA trainer: the backward (dQ, dK,
// dV) and a forward that recomputes the attention context, on packed dense
// q / k / v rows (head dim 128), bf16 operands, fp32 accumulation.
//
// Two kernels, both deterministic (no atomics):
//
// * q-side: one CTA = (64-query tile, query head). Pass 1 is a flash forward
//   over the tile's visible keys: online softmax -> the row log-sum-exp (log2
//   domain) and O, then D = rowsum(dO * O) in fp32. Pass 2 recomputes
//   P = exp2(S - lse), dP = dO V^T, dS = P * (dP - D) and accumulates
//   dQ = scale * dS K. It also leaves a bf16 copy of the dO tile for the
//   kv-side kernel. With kFwdOnly it stops after pass 1 and writes O.
// * kv-side: one CTA = (64-key tile, KV head). For every query head of the
//   GQA group and every query tile at or after the key tile it recomputes
//   S^T = K Q^T and P^T, forms dP^T = V dO^T and dS^T, and accumulates
//   dV += P^T dO and dK += scale * dS^T Q in registers; the group's heads are
//   summed inside the CTA.
//
// 4 warps per CTA, 16 rows each; K/V (q-side) and Q/dO (kv-side) tiles are
// double-buffered through cp.async into XOR-swizzled shared memory; every MMA
// is the warp-level m16n8k16 bf16 instruction. The algorithm is the standard
// two-pass flash-attention backward (Dao, "FlashAttention-2", 2023, Alg. 2)
// with dQ computed by its own pass instead of atomics.
//
// Reference behaviour: the reference trainer's attention backward
// (deltaserve-plugin/deltaserve/bwd_services/common/graph.py, padded
// [bn_max, l_max] attention) computes the same gradients; this kernel handles
// unpadded variable-length samples.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "attn_common.cuh"

namespace dsv {

constexpr int AB_BM = 64;        // rows (queries or keys) per CTA
constexpr int AB_BN = 64;        // keys (q-side) / queries (kv-side) per inner tile
constexpr int AB_THREADS = 128;  // 4 warps x 16 rows
constexpr int AB_Q_SMEM = (2 * AB_BM * HD + 4 * AB_BN * HD) * 2;             // 96 KB
constexpr int AB_KV_SMEM = (2 * AB_BM * HD + 4 * AB_BN * HD) * 2 + 4 * AB_BN * 4;  // 97 KB

struct AttnBwdArgs {
  const __nv_bfloat16* q;  // [n, ...] row stride q_stride; head h at h * 128
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int q_stride, k_stride, v_stride;
  const float* d_o;        // [n, Hq * 128] fp32, row stride do_stride
  int do_stride;
  const int* tiles;        // [num_tiles, 3] = (first row of the sample, sample length, tile row in sample)
  int n_total;             // rows of every row-indexed tensor
  int num_heads, group;    // Hq, Hq / Hkv
  int stat_stride;         // row stride of lse / dd ([Hq, stat_stride])
  float scale, scale_log2; // softmax scale, scale * log2(e)
  float* lse;              // [Hq, stat_stride] row log-sum-exp, log2 domain
  float* dd;               // [Hq, stat_stride] rowsum(dO * O)
  __nv_bfloat16* do_bf;    // [n, Hq * 128] bf16 copy of dO
  float* dq;               // [n, Hq * 128]
  float* dk;               // [n, Hkv * 128]
  float* dv;               // [n, Hkv * 128]
  __nv_bfloat16* o;        // forward-only: [n, ...] row stride o_stride
  int o_stride;
  // Optional epilogue work: rotate dq / dk back through RoPE (cos / sin
  // [n, 64] fp32, row stride rope_stride; nullptr = off) and store any of
  // dq / dk / dv (bf16_mask bits 1 / 2 / 4) as bf16 straight into the fused
  // d(qkv) rows (row stride dqkv_stride, head h of each part at its column
  // offset + h * 128) instead of fp32 into dq / dk / dv.
  const float* rope_cos;
  const float* rope_sin;
  int rope_stride;
  __nv_bfloat16* dqkv;
  int dqkv_stride, dq_col, dk_col, dv_col, bf16_mask;
};

// Row epilogue shared by both kernels: `acc` holds this thread's two rows
// (h = 0: row g, h = 1: row g + 8) x columns j * 8 + 2t + {0, 1}. Scales,
// optionally applies the inverse RoPE rotation (column c < 64 pairs with
// c + 64, which the same thread holds in acc[j + 8]), and stores fp32 or bf16.
__device__ __forceinline__ void store_grad_row(const AttnBwdArgs& a, const float (&acc)[16][4], int h, int grow,
                                               float scale, bool rope, float* f32_row, __nv_bfloat16* bf_row,
                                               int tq) {
  float v[16][2];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    v[j][0] = acc[j][2 * h] * scale;
    v[j][1] = acc[j][2 * h + 1] * scale;
  }
  if (rope) {
    const float* cr = a.rope_cos + (size_t)grow * a.rope_stride;
    const float* sr = a.rope_sin + (size_t)grow * a.rope_stride;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 cs = *reinterpret_cast<const float2*>(cr + j * 8 + 2 * tq);
      const float2 sn = *reinterpret_cast<const float2*>(sr + j * 8 + 2 * tq);
      const float x0 = v[j][0], y0 = v[j + 8][0], x1 = v[j][1], y1 = v[j + 8][1];
      v[j][0] = x0 * cs.x + y0 * sn.x;
      v[j + 8][0] = y0 * cs.x - x0 * sn.x;
      v[j][1] = x1 * cs.y + y1 * sn.y;
      v[j + 8][1] = y1 * cs.y - x1 * sn.y;
    }
  }
  if (bf_row != nullptr) {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<uint32_t*>(bf_row + j * 8 + 2 * tq) = pack_bf16(v[j][0], v[j][1]);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<float2*>(f32_row + j * 8 + 2 * tq) = make_float2(v[j][0], v[j][1]);
  }
}

// Tile of 64 rows x 128 bf16 from global rows (row0 + r) of `src` (row stride
// `stride`, column offset `col`) into swizzled smem; rows at or past `limit`
// are zero-filled.
__device__ __forceinline__ void load_rows_async(__nv_bfloat16* dst, const __nv_bfloat16* src, int stride, int col,
                                                int base, int r0, int limit, int tid) {
  for (int i = tid; i < 64 * 16; i += AB_THREADS) {
    const int r = i >> 4, c = i & 15;
    const int rr = r0 + r;
    const bool ok = rr < limit;
    cp_async16(dst + swz(r, c), src + (size_t)(base + (ok ? rr : 0)) * stride + col + c * 8, ok);
  }
}

// acc[16 x 64] += A[16 x 128] (rows arow0.. of a swizzled tile) * B^T, where B
// is a swizzled [64 x 128] tile whose rows are the 64 output columns.
__device__ __forceinline__ void mma_rows_x_rows(float (&acc)[8][4], const __nv_bfloat16* A, int arow0,
                                                const __nv_bfloat16* B, int lane) {
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t af[4];
    ldsm_x4(af, A + swz(arow0 + (lane & 15), ks * 2 + (lane >> 4)));
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {
      uint32_t b[4];
      ldsm_x4(b, B + swz(jp * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 2 + ((lane >> 3) & 1)));
      mma_bf16(acc[2 * jp], af, b[0], b[1]);
      mma_bf16(acc[2 * jp + 1], af, b[2], b[3]);
    }
  }
}

// out[16 x 128] += P[16 x 64] (accumulator layout, packed per 16-column step)
// * T[64 x 128] where T is a swizzled tile whose rows are P's columns.
__device__ __forceinline__ void mma_acc_x_tile(float (&out)[16][4], const uint32_t (&pa)[4], int kk,
                                               const __nv_bfloat16* T, int lane) {
#pragma unroll
  for (int dp = 0; dp < 8; ++dp) {
    uint32_t b[4];
    ldsm_x4_t(b, T + swz(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), dp * 2 + (lane >> 4)));
    mma_bf16(out[2 * dp], pa, b[0], b[1]);
    mma_bf16(out[2 * dp + 1], pa, b[2], b[3]);
  }
}

__device__ __forceinline__ void pack_a(uint32_t (&pa)[4], const float (&s)[8][4], int kk) {
  pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
  pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
  pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
  pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
}

template <bool kFwdOnly>
__global__ void __launch_bounds__(AB_THREADS) attn_bwd_q_kernel(AttnBwdArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [64 x 128]
  __nv_bfloat16* sdO = sQ + AB_BM * HD;                              // [64 x 128]
  __nv_bfloat16* sK = sdO + AB_BM * HD;                              // [2][64 x 128]
  __nv_bfloat16* sV = sK + 2 * AB_BN * HD;                           // [2][64 x 128]

  // Tiles are listed in increasing tile row; the q-side work grows with the
  // tile row, so run them last-first (heaviest CTAs start first).
  const int tile = gridDim.x - 1 - blockIdx.x;
  const int head = blockIdx.y;
  const int kvh = head / a.group;
  const int st = a.tiles[3 * tile], len = a.tiles[3 * tile + 1], qt0 = a.tiles[3 * tile + 2];
  if (st < 0 || len <= 0 || st + len > a.n_total || qt0 < 0 || qt0 >= len) {
    if (threadIdx.x == 0) set_error(kErrShape);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int row0 = warp * 16;
  const int kv_end = min(qt0 + AB_BM, len);  // keys visible to the tile's last query
  const int n_kb = (kv_end + AB_BN - 1) / AB_BN;

  load_rows_async(sQ, a.q, a.q_stride, head * HD, st, qt0, len, tid);
  load_rows_async(sK, a.k, a.k_stride, kvh * HD, st, 0, kv_end, tid);
  load_rows_async(sV, a.v, a.v_stride, kvh * HD, st, 0, kv_end, tid);
  cp_async_commit();
  if (!kFwdOnly) {
    // dO tile: fp32 -> bf16 into smem, plus the bf16 copy the kv-side kernel reads.
    const int ld = a.num_heads * HD;
    for (int i = tid; i < AB_BM * 32; i += AB_THREADS) {
      const int r = i >> 5, c4 = i & 31;
      const int qi = qt0 + r;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (qi < len) x = *reinterpret_cast<const float4*>(a.d_o + (size_t)(st + qi) * a.do_stride + head * HD + c4 * 4);
      uint2 pk;
      pk.x = pack_bf16(x.x, x.y);
      pk.y = pack_bf16(x.z, x.w);
      *reinterpret_cast<uint2*>(sdO + swz(r, c4 >> 1) + (c4 & 1) * 4) = pk;
      if (qi < len) *reinterpret_cast<uint2*>(a.do_bf + (size_t)(st + qi) * ld + head * HD + c4 * 4) = pk;
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[8][4];
  const int my_row = qt0 + row0;  // first query of this warp (within the sample)
  // A key tile needs masking if it reaches past this warp's first query or
  // the warp has rows past the sample end.
  auto need_mask = [&](int kb) { return (kb + 1) * AB_BN - 1 > my_row || my_row + 16 > len; };

  // ---------------- pass 1: online softmax -> lse, O
  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) {
      load_rows_async(sK + (buf ^ 1) * AB_BN * HD, a.k, a.k_stride, kvh * HD, st, (kb + 1) * AB_BN, kv_end, tid);
      load_rows_async(sV + (buf ^ 1) * AB_BN * HD, a.v, a.v_stride, kvh * HD, st, (kb + 1) * AB_BN, kv_end, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) ldsm_x4(qf[ks], sQ + swz(row0 + (lane & 15), ks * 2 + (lane >> 4)));
    }
    const __nv_bfloat16* k_t = sK + buf * AB_BN * HD;
    const __nv_bfloat16* v_t = sV + buf * AB_BN * HD;
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t b[4];
        ldsm_x4(b, k_t + swz(jp * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 2 + ((lane >> 3) & 1)));
        mma_bf16(s[2 * jp], qf[ks], b[0], b[1]);
        mma_bf16(s[2 * jp + 1], qf[ks], b[2], b[3]);
      }
    }
    const bool msk = need_mask(kb);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * a.scale_log2;
        if (msk) {
          const int qrow = my_row + g + ((e >> 1) << 3);
          const int kpos = kb * AB_BN + j * 8 + 2 * tq + (e & 1);
          if (kpos > qrow || qrow >= len) x = -INFINITY;
        }
        s[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float m_new = fmaxf(m_r[h], mx[h]);
      corr[h] = (m_new == -INFINITY) ? 1.f : exp2f(m_r[h] - m_new);
      m_r[h] = m_new;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        const float p = (mm == -INFINITY) ? 0.f : exp2f(s[j][e] - mm);
        s[j][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
      rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
      l_r[h] = l_r[h] * corr[h] + rs[h];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pack_a(pa, s, kk);
      mma_acc_x_tile(o, pa, kk, v_t, lane);
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  float inv[2], lse2[2], dsum[2] = {0.f, 0.f};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    inv[h] = l_r[h] > 0.f ? 1.f / l_r[h] : 0.f;
    lse2[h] = l_r[h] > 0.f ? m_r[h] + log2f(l_r[h]) : 0.f;
  }
  if (kFwdOnly) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int qi = my_row + g + h * 8;
      if (qi >= len) continue;
      __nv_bfloat16* dst = a.o + (size_t)(st + qi) * a.o_stride + head * HD;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<uint32_t*>(dst + j * 8 + 2 * tq) = pack_bf16(o[j][2 * h] * inv[h], o[j][2 * h + 1] * inv[h]);
    }
    return;
  }
  // D = rowsum(dO * O) from the fp32 dO rows.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int qi = my_row + g + h * 8;
    if (qi < len) {
      const float* src = a.d_o + (size_t)(st + qi) * a.do_stride + head * HD;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float2 d = *reinterpret_cast<const float2*>(src + j * 8 + 2 * tq);
        dsum[h] += d.x * o[j][2 * h] * inv[h] + d.y * o[j][2 * h + 1] * inv[h];
      }
    }
    dsum[h] += __shfl_xor_sync(0xffffffffu, dsum[h], 1);
    dsum[h] += __shfl_xor_sync(0xffffffffu, dsum[h], 2);
    if (tq == 0 && qi < len) {
      a.lse[(size_t)head * a.stat_stride + st + qi] = lse2[h];
      a.dd[(size_t)head * a.stat_stride + st + qi] = dsum[h];
    }
  }

  // ---------------- pass 2: dQ = scale * sum_j P (dP - D) K
  // (the last pass-1 iteration ended with a barrier: both K/V buffers are free)
  load_rows_async(sK, a.k, a.k_stride, kvh * HD, st, 0, kv_end, tid);
  load_rows_async(sV, a.v, a.v_stride, kvh * HD, st, 0, kv_end, tid);
  cp_async_commit();
  float (&dq)[16][4] = o;  // O is no longer needed: reuse its registers
#pragma unroll
  for (int j = 0; j < 16; ++j) dq[j][0] = dq[j][1] = dq[j][2] = dq[j][3] = 0.f;
  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) {
      load_rows_async(sK + (buf ^ 1) * AB_BN * HD, a.k, a.k_stride, kvh * HD, st, (kb + 1) * AB_BN, kv_end, tid);
      load_rows_async(sV + (buf ^ 1) * AB_BN * HD, a.v, a.v_stride, kvh * HD, st, (kb + 1) * AB_BN, kv_end, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const __nv_bfloat16* k_t = sK + buf * AB_BN * HD;
    const __nv_bfloat16* v_t = sV + buf * AB_BN * HD;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      dp[j][0] = dp[j][1] = dp[j][2] = dp[j][3] = 0.f;
    }
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t b[4];
        ldsm_x4(b, k_t + swz(jp * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 2 + ((lane >> 3) & 1)));
        mma_bf16(s[2 * jp], qf[ks], b[0], b[1]);
        mma_bf16(s[2 * jp + 1], qf[ks], b[2], b[3]);
      }
    }
    mma_rows_x_rows(dp, sdO, row0, v_t, lane);  // dP = dO V^T
    const bool msk = need_mask(kb);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        float p = exp2f(s[j][e] * a.scale_log2 - lse2[h]);
        if (msk) {
          const int qrow = my_row + g + (h << 3);
          const int kpos = kb * AB_BN + j * 8 + 2 * tq + (e & 1);
          if (kpos > qrow || qrow >= len) p = 0.f;
        }
        s[j][e] = p * (dp[j][e] - dsum[h]);  // dS
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pack_a(pa, s, kk);
      mma_acc_x_tile(dq, pa, kk, k_t, lane);
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  const bool rope = a.rope_cos != nullptr;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int qi = my_row + g + h * 8;
    if (qi >= len) continue;
    const size_t grow = (size_t)(st + qi);
    float* f32 = (a.bf16_mask & 1) ? nullptr : a.dq + grow * (a.num_heads * HD) + head * HD;
    __nv_bfloat16* bf = (a.bf16_mask & 1) ? a.dqkv + grow * a.dqkv_stride + a.dq_col + head * HD : nullptr;
    store_grad_row(a, dq, h, (int)grow, a.scale, rope, f32, bf, tq);
  }
}

__global__ void __launch_bounds__(AB_THREADS) attn_bwd_kv_kernel(AttnBwdArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [64 x 128]
  __nv_bfloat16* sV = sK + AB_BM * HD;                               // [64 x 128]
  __nv_bfloat16* sQ = sV + AB_BM * HD;                               // [2][64 x 128]
  __nv_bfloat16* sdO = sQ + 2 * AB_BN * HD;                          // [2][64 x 128]
  float* sL = reinterpret_cast<float*>(sdO + 2 * AB_BN * HD);        // [2][64]
  float* sD = sL + 2 * AB_BN;                                        // [2][64]

  const int tile = blockIdx.x;  // increasing tile row: the heaviest kv-side CTAs first
  const int kvh = blockIdx.y;
  const int st = a.tiles[3 * tile], len = a.tiles[3 * tile + 1], kt0 = a.tiles[3 * tile + 2];
  if (st < 0 || len <= 0 || st + len > a.n_total || kt0 < 0 || kt0 >= len) {
    if (threadIdx.x == 0) set_error(kErrShape);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int row0 = warp * 16;
  const int ld = a.num_heads * HD;
  const int n_qt = (len - kt0 + AB_BN - 1) / AB_BN;  // query tiles at or after this key tile
  const int iters = a.group * n_qt;

  load_rows_async(sK, a.k, a.k_stride, kvh * HD, st, kt0, len, tid);
  load_rows_async(sV, a.v, a.v_stride, kvh * HD, st, kt0, len, tid);
  auto load_q = [&](int it, int buf) {
    const int h = kvh * a.group + it / n_qt;
    const int qi0 = kt0 + (it % n_qt) * AB_BN;
    load_rows_async(sQ + buf * AB_BN * HD, a.q, a.q_stride, h * HD, st, qi0, len, tid);
    load_rows_async(sdO + buf * AB_BN * HD, a.do_bf, ld, h * HD, st, qi0, len, tid);
    for (int r = tid; r < AB_BN; r += AB_THREADS) {
      const int qi = qi0 + r;
      const bool ok = qi < len;
      sL[buf * AB_BN + r] = ok ? a.lse[(size_t)h * a.stat_stride + st + qi] : 0.f;
      sD[buf * AB_BN + r] = ok ? a.dd[(size_t)h * a.stat_stride + st + qi] : 0.f;
    }
  };
  load_q(0, 0);
  cp_async_commit();

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    dk[j][0] = dk[j][1] = dk[j][2] = dk[j][3] = 0.f;
    dv[j][0] = dv[j][1] = dv[j][2] = dv[j][3] = 0.f;
  }
  const int my_key = kt0 + row0;  // first key of this warp (within the sample)
  for (int it = 0; it < iters; ++it) {
    const int buf = it & 1;
    if (it + 1 < iters) load_q(it + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int qi0 = kt0 + (it % n_qt) * AB_BN;
    const __nv_bfloat16* q_t = sQ + buf * AB_BN * HD;
    const __nv_bfloat16* do_t = sdO + buf * AB_BN * HD;
    const float* l_t = sL + buf * AB_BN;
    const float* d_t = sD + buf * AB_BN;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      dp[j][0] = dp[j][1] = dp[j][2] = dp[j][3] = 0.f;
    }
    mma_rows_x_rows(s, sK, row0, q_t, lane);    // S^T = K Q^T  (16 keys x 64 queries)
    mma_rows_x_rows(dp, sV, row0, do_t, lane);  // dP^T = V dO^T
    // Masking is needed on the diagonal tile and where queries run past the sample.
    const bool msk = qi0 < my_key + 16 || qi0 + AB_BN > len;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = j * 8 + 2 * tq + (e & 1);  // query within the tile
        float p = exp2f(s[j][e] * a.scale_log2 - l_t[ql]);
        if (msk) {
          const int key = my_key + g + ((e >> 1) << 3);
          const int qi = qi0 + ql;
          if (qi < key || qi >= len) p = 0.f;
        }
        s[j][e] = p;                          // P^T
        dp[j][e] = p * (dp[j][e] - d_t[ql]);  // dS^T
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4], da[4];
      pack_a(pa, s, kk);
      pack_a(da, dp, kk);
      mma_acc_x_tile(dv, pa, kk, do_t, lane);  // dV += P^T dO
      mma_acc_x_tile(dk, da, kk, q_t, lane);   // dK += dS^T Q
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  const int ldkv = (a.num_heads / a.group) * HD;
  const bool rope = a.rope_cos != nullptr;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int kj = my_key + g + h * 8;
    if (kj >= len) continue;
    const size_t grow = (size_t)(st + kj);
    __nv_bfloat16* qkv_row = a.dqkv != nullptr ? a.dqkv + grow * a.dqkv_stride : nullptr;
    store_grad_row(a, dk, h, (int)grow, a.scale, rope,
                   (a.bf16_mask & 2) ? nullptr : a.dk + grow * ldkv + kvh * HD,
                   (a.bf16_mask & 2) ? qkv_row + a.dk_col + kvh * HD : nullptr, tq);
    store_grad_row(a, dv, h, (int)grow, 1.f, false,
                   (a.bf16_mask & 4) ? nullptr : a.dv + grow * ldkv + kvh * HD,
                   (a.bf16_mask & 4) ? qkv_row + a.dv_col + kvh * HD : nullptr, tq);
  }
}

}  // namespace dsv

// ---------------------------------------------------------------- bindings

namespace {

void check_rows(const torch::Tensor& t, const char* name, at::ScalarType dt, int64_t heads) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == dt, "attn_bwd: ", name, " has the wrong dtype/device");
  TORCH_CHECK(t.dim() == 3 && t.size(1) == heads && t.size(2) == dsv::HD, "attn_bwd: ", name, " must be [n, ",
              heads, ", 128]");
  TORCH_CHECK(t.stride(2) == 1 && t.stride(1) == dsv::HD, "attn_bwd: ", name, " heads must be adjacent rows of 128");
  const int64_t esz = t.element_size();
  TORCH_CHECK((t.stride(0) * esz) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "attn_bwd: ", name, " rows must be 16-byte aligned");
}

dsv::AttnBwdArgs make_args(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                           const torch::Tensor& tiles, double scale) {
  dsv::AttnBwdArgs a{};
  const int64_t hq = q.size(1), hkv = k.size(1);
  check_rows(q, "q", at::kBFloat16, hq);
  check_rows(k, "k", at::kBFloat16, hkv);
  check_rows(v, "v", at::kBFloat16, hkv);
  TORCH_CHECK(hq % hkv == 0, "attn_bwd: query heads must be a multiple of KV heads");
  TORCH_CHECK(k.size(0) == q.size(0) && v.size(0) == q.size(0), "attn_bwd: q/k/v row counts differ");
  TORCH_CHECK(tiles.is_cuda() && tiles.scalar_type() == at::kInt && tiles.dim() == 2 && tiles.size(1) == 3 &&
                  tiles.is_contiguous(), "attn_bwd: tiles must be int32 [T, 3]");
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.q_stride = (int)q.stride(0);
  a.k_stride = (int)k.stride(0);
  a.v_stride = (int)v.stride(0);
  a.tiles = tiles.data_ptr<int>();
  a.n_total = (int)q.size(0);
  a.num_heads = (int)hq;
  a.group = (int)(hq / hkv);
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  return a;
}

}  // namespace

// dq [n, Hq, 128], dk / dv [n, Hkv, 128] fp32 (rows outside every sample are
// left untouched); lse / dd [Hq, >= n] fp32 and do_bf [n, Hq*128] bf16 are
// scratch.
void dsv_attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor d_o, torch::Tensor tiles,
                  torch::Tensor lse, torch::Tensor dd, torch::Tensor do_bf, c10::optional<torch::Tensor> dq,
                  c10::optional<torch::Tensor> dk, c10::optional<torch::Tensor> dv, double scale,
                  c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin,
                  c10::optional<torch::Tensor> dqkv, int64_t bf16_mask) {
  using namespace dsv;
  if (tiles.size(0) == 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  AttnBwdArgs a = make_args(q, k, v, tiles, scale);
  const int64_t n = q.size(0), hq = q.size(1), hkv = k.size(1);
  TORCH_CHECK(d_o.scalar_type() == at::kFloat && d_o.dim() == 2 && d_o.size(0) == n && d_o.size(1) == hq * HD &&
                  d_o.stride(1) == 1 && d_o.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(d_o.data_ptr()) % 16 == 0,
              "attn_bwd: d_o must be fp32 [n, Hq*128] with 16-byte aligned rows");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && dd.scalar_type() == at::kFloat && lse.is_contiguous() &&
                  dd.is_contiguous() && lse.dim() == 2 && lse.size(0) == hq && lse.size(1) >= n &&
                  dd.sizes() == lse.sizes(), "attn_bwd: lse / dd must be fp32 [Hq, >= n]");
  TORCH_CHECK(do_bf.scalar_type() == at::kBFloat16 && do_bf.is_contiguous() && do_bf.numel() == n * hq * HD,
              "attn_bwd: do_bf must be bf16 [n, Hq*128]");
  TORCH_CHECK(bf16_mask >= 0 && bf16_mask <= 7, "attn_bwd: bf16_mask is a 3-bit mask");
  const int64_t want[3] = {hq, hkv, hkv};
  const c10::optional<torch::Tensor>* outs[3] = {&dq, &dk, &dv};
  for (int i = 0; i < 3; ++i) {
    if (bf16_mask & (1 << i)) continue;
    const auto& t = *outs[i];
    TORCH_CHECK(t.has_value() && t->scalar_type() == at::kFloat && t->is_contiguous() &&
                    t->numel() == n * want[i] * HD, "attn_bwd: fp32 output ", i, " must be [n, H, 128]");
  }
  if (bf16_mask != 0) {
    TORCH_CHECK(dqkv.has_value() && dqkv->scalar_type() == at::kBFloat16 && dqkv->dim() == 2 &&
                    dqkv->size(0) == n && dqkv->stride(1) == 1 && dqkv->stride(0) % 2 == 0 &&
                    dqkv->size(1) >= (hq + 2 * hkv) * HD, "attn_bwd: dqkv must be bf16 [n, (Hq+2Hkv)*128]");
    a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv->data_ptr());
    a.dqkv_stride = (int)dqkv->stride(0);
    a.dq_col = 0;
    a.dk_col = (int)(hq * HD);
    a.dv_col = (int)((hq + hkv) * HD);
  }
  a.bf16_mask = (int)bf16_mask;
  if (rope_cos.has_value()) {
    TORCH_CHECK(rope_sin.has_value() && rope_cos->scalar_type() == at::kFloat && rope_sin->scalar_type() == at::kFloat &&
                    rope_cos->dim() == 2 && rope_cos->size(0) >= n && rope_cos->size(1) == HD / 2 &&
                    rope_cos->stride(1) == 1 && rope_sin->sizes() == rope_cos->sizes() &&
                    rope_sin->strides() == rope_cos->strides() && rope_cos->stride(0) % 2 == 0,
                "attn_bwd: rope cos / sin must be fp32 [>= n, 64]");
    a.rope_cos = rope_cos->data_ptr<float>();
    a.rope_sin = rope_sin->data_ptr<float>();
    a.rope_stride = (int)rope_cos->stride(0);
  }
  a.d_o = d_o.data_ptr<float>();
  a.do_stride = (int)d_o.stride(0);
  a.stat_stride = (int)lse.size(1);
  a.lse = lse.data_ptr<float>();
  a.dd = dd.data_ptr<float>();
  a.do_bf = reinterpret_cast<__nv_bfloat16*>(do_bf.data_ptr());
  a.dq = (bf16_mask & 1) ? nullptr : dq->data_ptr<float>();
  a.dk = (bf16_mask & 2) ? nullptr : dk->data_ptr<float>();
  a.dv = (bf16_mask & 4) ? nullptr : dv->data_ptr<float>();
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn_bwd_q_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, AB_Q_SMEM);
    cudaFuncSetAttribute(attn_bwd_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AB_KV_SMEM);
    attr = true;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  const unsigned T = (unsigned)tiles.size(0);
  attn_bwd_q_kernel<false><<<dim3(T, (unsigned)hq), AB_THREADS, AB_Q_SMEM, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  attn_bwd_kv_kernel<<<dim3(T, (unsigned)hkv), AB_THREADS, AB_KV_SMEM, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Causal varlen attention forward on packed rows: o [n, Hq*128] bf16 (row
// stride o.stride(0)); rows outside every sample are left untouched.
void dsv_attn_fwd_dense(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor tiles, torch::Tensor o,
                        double scale) {
  using namespace dsv;
  if (tiles.size(0) == 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  AttnBwdArgs a = make_args(q, k, v, tiles, scale);
  TORCH_CHECK(o.scalar_type() == at::kBFloat16 && o.dim() == 2 && o.size(0) == q.size(0) &&
                  o.size(1) >= q.size(1) * HD && o.stride(1) == 1 && o.stride(0) % 8 == 0,
              "attn_fwd_dense: o must be bf16 [n, >= Hq*128]");
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.o_stride = (int)o.stride(0);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn_bwd_q_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, AB_Q_SMEM);
    attr = true;
  }
  attn_bwd_q_kernel<true><<<dim3((unsigned)tiles.size(0), (unsigned)q.size(1)), AB_THREADS, AB_Q_SMEM,
                            at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

DSV_ERROR_ACCESSOR(dsv_read_error_attn_bwd)
