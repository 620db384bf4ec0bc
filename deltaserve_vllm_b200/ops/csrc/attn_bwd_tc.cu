// Causal varlen GQA attention backward on the 5th-generation tensor cores
// (sm_100a), for the LoRA trainer's packed samples (head dim 128).
//
// Inputs per row: q / k / v (bf16, the RoPE'd projections), the forward
// output O and its gradient dO (bf16), and the forward's base-2 row
// log-sum-exp (from the tcgen05 forward's statistics output). Two kernels,
// deterministic (no atomics), each CTA = 192 threads: warp 0 TMA producer,
// warp 1 MMA issuer + TMEM owner, warps 2-5 one accumulator row per thread.
//
// * q-side (dQ): one CTA = 128 queries x one query head. Its threads first
//   form D = rowsum(dO * O) for their rows (stored for the kv-side). Per
//   64-key tile: S = Q K^T and dP = dO V^T into double-buffered TMEM, then
//   dS = P * (dP - D) with P = exp2(S * scale * log2 e - lse), written bf16
//   to shared memory, then dQ += dS K (K read MN-major from the same tile).
// * kv-side (dK, dV): one CTA = 128 keys x one KV head, looping over the
//   GQA group's query heads and the 64-query tiles at or after the key
//   tile: S^T = K Q^T and dP^T = V dO^T, then P^T and dS^T (bf16, shared
//   memory), then dV += P^T dO and dK += dS^T Q (dO and Q MN-major). The
//   group's heads accumulate in the same TMEM columns. When there are fewer
//   (key tile, KV head) pairs than SMs (high TP degrees), each CTA takes one
//   query head of the group instead and writes fp32 partials that a small
//   finish kernel sums (then scale, RoPE, store) in a fixed order.
//
// TMEM: q-side S[2] 0/64, dP[2] 128/192, dQ 256-383; kv-side S^T[2] 0/64,
// dP^T[2] 128/192, dV 256-383, dK 384-511 (512 allocated; 192 KB of shared
// memory per CTA keeps one CTA per SM). Epilogues scale dQ / dK by the
// softmax scale, undo RoPE on dQ / dK (pairs c, c + 64) and store fp32
// [n, H*128] rows or bf16 into the fused d(qkv) rows, the same contract as
// the warp-level kernels in attn_bwd.cu.
//
// Algorithm: FlashAttention-2 backward (Dao, 2023, Alg. 2), with dQ
// computed by its own pass instead of atomics. Reference behaviour: the
// reference trainer's attention backward
// (deltaserve-plugin/deltaserve/bwd_services/common/attention.py:48-112).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_tc.cuh"
#include "tmap.h"

namespace dsv {

constexpr int AT_THREADS = 192;
constexpr int AT_T128 = 2 * 128 * 128;   // bf16 [128 x 128] tile (two 64-col chunks of 16 KB)
constexpr int AT_T64 = 2 * 64 * 128;     // bf16 [64 x 128] tile (two 64-col chunks of 8 KB)
constexpr int AT_C128 = 128 * 128;       // one chunk of a 128-row tile
constexpr int AT_C64 = 64 * 128;         // one chunk of a 64-row tile
constexpr int AQ_SMEM = 2 * AT_T128 + 3 * AT_T64 + 3 * AT_T64 + 2 * AT_C128 + 1024 + 256;
constexpr int AKV_SMEM = 2 * AT_T128 + 2 * AT_T64 + 2 * AT_T64 + 4 * AT_C128 + 2 * 128 * 4 + 1024 + 256;

enum : int {
  kErrAtQ = 0x4201,
  kErrAtKv = 0x4202,
  kErrAtS = 0x4203,
  kErrAtDs = 0x4204,
  kErrAtDone = 0x4205,
  kErrAtEmpty = 0x4206,
  kErrAtSEmpty = 0x4207,
  kErrAtDsEmpty = 0x4208,
  kErrAtDrain = 0x4209,
  kErrAtStat = 0x420a,
};

struct FaBwdArgs {
  const int* tiles;         // [T, 3] = (first row of the sample, sample length, tile row), 128-row tiles
  int num_tiles;
  int num_heads, num_kv_heads, group;
  const __nv_bfloat16* o;   // [n, Hq*128] forward output, row stride o_stride
  int o_stride;
  const __nv_bfloat16* d_o; // [n, Hq*128] bf16 gradient, row stride do_stride
  int do_stride;
  const float* lse;         // [Hq, stat_stride] base-2 log-sum-exp of the scaled scores
  float* dd;                // [Hq, stat_stride] rowsum(dO * O), written by the q-side
  int stat_stride;
  float scale, scale_log2;
  float* dq;                // fp32 [n, Hq*128] or null (bf16 into dqkv)
  float* dk;                // fp32 [n, Hkv*128] or null
  float* dv;
  __nv_bfloat16* dqkv;
  int dqkv_stride, dq_col, dk_col, dv_col, bf16_mask;
  const float* rope_cos;    // [n, 64] fp32 (row stride rope_stride) or null
  const float* rope_sin;
  int rope_stride;
  // Head split of the dK/dV pass (few key tiles x KV heads for the SMs): one
  // CTA per (key tile, query head of the group) writes raw fp32 dK / dV
  // partials [group][n][Hkv*128]; kv_split_finish_kernel sums the group.
  int split_heads;
  float* part_dk;
  float* part_dv;
  int n_rows;
};

// Bounded wait that the whole warp agrees on (tcgen05.ld / st that follow are
// warp-collective).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, code));
}

// Epilogue of one accumulator row (128 fp32 TMEM columns at `taddr`): scale,
// optional inverse RoPE rotation, store fp32 or bf16. Warp-collective.
__device__ __forceinline__ void store_acc_row(uint32_t taddr, float scale, const float* cr, const float* sr,
                                              float* f32_row, __nv_bfloat16* bf_row, bool row_ok) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t x[32], y[32];
    tmem_ld_32x32b_x32(taddr + h * 32, x);
    tmem_ld_32x32b_x32(taddr + 64 + h * 32, y);
    tmem_ld_wait();
    if (!row_ok) continue;
    float a[32], b[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      a[i] = __uint_as_float(x[i]) * scale;
      b[i] = __uint_as_float(y[i]) * scale;
    }
    if (cr != nullptr) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 c4 = *reinterpret_cast<const float4*>(cr + h * 32 + i);
        const float4 s4 = *reinterpret_cast<const float4*>(sr + h * 32 + i);
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float xa = a[i + e], yb = b[i + e];
          a[i + e] = xa * cc[e] + yb * ss[e];
          b[i + e] = yb * cc[e] - xa * ss[e];
        }
      }
    }
    if (bf_row != nullptr) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint4 wa, wb;
        wa.x = pack2_bf16(a[u * 8 + 0], a[u * 8 + 1]);
        wa.y = pack2_bf16(a[u * 8 + 2], a[u * 8 + 3]);
        wa.z = pack2_bf16(a[u * 8 + 4], a[u * 8 + 5]);
        wa.w = pack2_bf16(a[u * 8 + 6], a[u * 8 + 7]);
        wb.x = pack2_bf16(b[u * 8 + 0], b[u * 8 + 1]);
        wb.y = pack2_bf16(b[u * 8 + 2], b[u * 8 + 3]);
        wb.z = pack2_bf16(b[u * 8 + 4], b[u * 8 + 5]);
        wb.w = pack2_bf16(b[u * 8 + 6], b[u * 8 + 7]);
        *reinterpret_cast<uint4*>(bf_row + h * 32 + u * 8) = wa;
        *reinterpret_cast<uint4*>(bf_row + 64 + h * 32 + u * 8) = wb;
      }
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        *reinterpret_cast<float4*>(f32_row + h * 32 + u * 4) = make_float4(a[u * 4], a[u * 4 + 1], a[u * 4 + 2], a[u * 4 + 3]);
        *reinterpret_cast<float4*>(f32_row + 64 + h * 32 + u * 4) =
            make_float4(b[u * 4], b[u * 4 + 1], b[u * 4 + 2], b[u * 4 + 3]);
      }
    }
  }
}

// Wait until the TMA loads of a ring slot issued `issued` times have landed.
__device__ __forceinline__ void drain_slot(uint64_t* bar, int issued) {
  if (issued == 0) return;
  const uint32_t par = (uint32_t)(issued - 1) & 1u;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, par)) {
    if (globaltimer_ns() - t0 > kWaitNs) { set_error(kErrAtDrain); break; }
  }
}

// ---------------------------------------------------------------- q-side
__global__ void __launch_bounds__(AT_THREADS, 1)
    fa_bwd_q_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       FaBwdArgs a) {
  extern __shared__ uint8_t aq_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(aq_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + AT_T128;
  uint8_t* sK = sDO + AT_T128;      // [3][T64]
  uint8_t* sV = sK + 3 * AT_T64;    // [3][T64]
  uint8_t* sDS = sV + 3 * AT_T64;   // [2][C128]: dS [128 q x 64 keys]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + 2 * AT_C128);
  uint64_t* qo_full = bars + 0;
  uint64_t* k_full = bars + 1;      // [3]
  uint64_t* v_full = bars + 4;      // [3]
  uint64_t* kv_empty = bars + 7;    // [3]
  uint64_t* s_full = bars + 10;     // [2]
  uint64_t* s_empty = bars + 12;    // [2]
  uint64_t* ds_full = bars + 14;    // [2]
  uint64_t* ds_empty = bars + 16;   // [2]
  uint64_t* dq_done = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tile = a.num_tiles - 1 - (int)blockIdx.x;   // later tile rows (more keys) first
  const int head = blockIdx.y;
  const int kvh = head / a.group;
  const int s0 = a.tiles[3 * tile], len = a.tiles[3 * tile + 1], qt0 = a.tiles[3 * tile + 2];
  const int rows_valid = min(128, len - qt0);
  const int kv_end = qt0 + rows_valid;
  const int n_kt = (kv_end + 63) / 64;

  if (threadIdx.x == 0) {
    mbar_init(qo_full, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&ds_full[i], 128);
      mbar_init(&ds_empty[i], 1);
    }
    mbar_init(dq_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(qo_full, 2 * AT_T128);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(sQ + c * AT_C128, &tmQ, qo_full, head * 128 + c * 64, s0 + qt0);
        tma_load_2d(sDO + c * AT_C128, &tmDO, qo_full, head * 128 + c * 64, s0 + qt0);
      }
      int issued[3] = {0, 0, 0};
      for (int j = 0; j < n_kt; ++j) {
        const int st = j % 3;
        if (!mbar_wait(&kv_empty[st], (uint32_t)((j / 3) & 1) ^ 1u, kErrAtEmpty)) break;
        mbar_arrive_expect_tx(&k_full[st], AT_T64);
        for (int c = 0; c < 2; ++c) tma_load_2d(sK + st * AT_T64 + c * AT_C64, &tmK, &k_full[st], kvh * 128 + c * 64, s0 + j * 64);
        mbar_arrive_expect_tx(&v_full[st], AT_T64);
        for (int c = 0; c < 2; ++c) tma_load_2d(sV + st * AT_T64 + c * AT_C64, &tmV, &v_full[st], kvh * 128 + c * 64, s0 + j * 64);
        issued[st]++;
      }
      drain_slot(qo_full, 1);
      for (int st = 0; st < 3; ++st) {
        drain_slot(&k_full[st], issued[st]);
        drain_slot(&v_full[st], issued[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 64, false, false);
      constexpr uint32_t IDESC_Q = idesc_bf16_f32(128, 128, false, true);
      const uint32_t q_addr = smem_u32(sQ), do_addr = smem_u32(sDO);
      bool ok = mbar_wait(qo_full, 0, kErrAtQ);
      auto issue_sdp = [&](int j) -> bool {
        const int st = j % 3, b = j & 1;
        const uint32_t use = (uint32_t)(j / 3) & 1u;
        if (!mbar_wait(&k_full[st], use, kErrAtKv) || !mbar_wait(&v_full[st], use, kErrAtKv)) return false;
        if (!mbar_wait(&s_empty[b], ((uint32_t)(j >> 1) & 1u) ^ 1u, kErrAtSEmpty)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * AT_T64), v_addr = smem_u32(sV + st * AT_T64);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tmem + b * 64, desc_kmajor(q_addr, kk, AT_C128), desc_kmajor(k_addr, kk, AT_C64), IDESC_S,
                     kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tmem + 128 + b * 64, desc_kmajor(do_addr, kk, AT_C128), desc_kmajor(v_addr, kk, AT_C64),
                     IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[b]);
        return true;
      };
      if (ok) {
        tc_fence_after();
        ok = issue_sdp(0);
      }
      for (int j = 0; j < n_kt && ok; ++j) {
        if (j + 1 < n_kt && !issue_sdp(j + 1)) { ok = false; break; }
        const int st = j % 3, b = j & 1;
        if (!mbar_wait(&ds_full[b], (uint32_t)(j >> 1) & 1u, kErrAtDs)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ds_addr = smem_u32(sDS + b * AT_C128), k_addr = smem_u32(sK + st * AT_T64);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_f16(tmem + 256, desc_kmajor(ds_addr, kk, AT_C128), desc_mnmajor(k_addr, kk, AT_C64), IDESC_Q,
                     (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&ds_empty[b]);
        tc_commit(&kv_empty[st]);
      }
      if (ok) {
        tc_commit(dq_done);
        mbar_wait(dq_done, 0, kErrAtDone);   // every commit of this thread has landed
      }
    }
  } else {
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(q4 * 32) << 16);
    const bool row_ok = r < rows_valid;
    const int qi = qt0 + r;                     // query index within the sample
    const size_t grow = (size_t)s0 + qi;
    float lse_r = INFINITY, d_r = 0.f;
    if (row_ok) {
      lse_r = a.lse[(size_t)head * a.stat_stride + grow];
      const __nv_bfloat16* orow = a.o + grow * a.o_stride + head * 128;
      const __nv_bfloat16* grow_p = a.d_o + grow * a.do_stride + head * 128;
#pragma unroll 4
      for (int u = 0; u < 16; ++u) {
        const uint4 ov = *reinterpret_cast<const uint4*>(orow + u * 8);
        const uint4 gv = *reinterpret_cast<const uint4*>(grow_p + u * 8);
        const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
        const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 of = __bfloat1622float2(o2[e]), gf = __bfloat1622float2(g2[e]);
          d_r += of.x * gf.x + of.y * gf.y;
        }
      }
      a.dd[(size_t)head * a.stat_stride + grow] = d_r;
    }
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      const int b = j & 1;
      const uint32_t use = (uint32_t)(j >> 1) & 1u;
      if (!warp_wait(&s_full[b], use, kErrAtS) || !warp_wait(&ds_empty[b], use ^ 1u, kErrAtDsEmpty)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int lim = min(qi + 1, len) - j * 64;  // keys [j*64, j*64 + lim) are visible to this row
      uint8_t* ds_tile = sDS + b * AT_C128;
      uint32_t x[2][32], y[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld_32x32b_x32(t_lane + b * 64 + c * 32, x[c]);
        tmem_ld_32x32b_x32(t_lane + 128 + b * 64 + c * 32, y[c]);
      }
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float ds[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p = (c * 32 + i < lim) ? fast_exp2(fmaf(__uint_as_float(x[c][i]), a.scale_log2, -lse_r)) : 0.f;
          ds[i] = p * (__uint_as_float(y[c][i]) - d_r);
        }
        store_row_units(ds_tile, r, c * 4, ds);
      }
      tc_fence_before();
      mbar_arrive(&s_empty[b]);
      fence_proxy_async_smem();
      mbar_arrive(&ds_full[b]);
    }
    if (ok && warp_wait(dq_done, 0, kErrAtDone)) {
      tc_fence_after();
      const bool rope = a.rope_cos != nullptr;
      const float* cr = rope && row_ok ? a.rope_cos + grow * a.rope_stride : nullptr;
      const float* sr = rope && row_ok ? a.rope_sin + grow * a.rope_stride : nullptr;
      float* f32 = (a.bf16_mask & 1) ? nullptr : a.dq + grow * (size_t)(a.num_heads * 128) + head * 128;
      __nv_bfloat16* bf = (a.bf16_mask & 1) ? a.dqkv + grow * a.dqkv_stride + a.dq_col + head * 128 : nullptr;
      store_acc_row(t_lane + 256, a.scale, cr, sr, f32, bf, row_ok);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- kv-side
__global__ void __launch_bounds__(AT_THREADS, 1)
    fa_bwd_kv_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        FaBwdArgs a) {
  extern __shared__ uint8_t akv_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(akv_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + AT_T128;
  uint8_t* sQ = sV + AT_T128;        // [2][T64]
  uint8_t* sDO = sQ + 2 * AT_T64;    // [2][T64]
  uint8_t* sPt = sDO + 2 * AT_T64;   // [2][C128]: P^T [128 keys x 64 q]
  uint8_t* sDSt = sPt + 2 * AT_C128; // [2][C128]
  float* stats = reinterpret_cast<float*>(sDSt + 2 * AT_C128);   // [2][128]: lse[64], D[64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(stats + 2 * 128);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;      // [2]
  uint64_t* stat_full = bars + 3;    // [2]
  uint64_t* qd_empty = bars + 5;     // [2]
  uint64_t* s_full = bars + 7;       // [2]
  uint64_t* s_empty = bars + 9;      // [2]
  uint64_t* ds_full = bars + 11;     // [2]
  uint64_t* pds_empty = bars + 13;   // [2]
  uint64_t* dkv_done = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tile = blockIdx.x;       // earlier key tiles (more queries) first
  const int g = a.split_heads ? (int)blockIdx.y / a.group : (int)blockIdx.y;
  const int h_first = a.split_heads ? (int)blockIdx.y % a.group : 0;   // first query head of the group
  const int h_count = a.split_heads ? 1 : a.group;
  const int s0 = a.tiles[3 * tile], len = a.tiles[3 * tile + 1], k0 = a.tiles[3 * tile + 2];
  const int rows_valid = min(128, len - k0);
  const int nq = (len + 63) / 64 - k0 / 64;   // 64-query tiles at or after the key tile
  const int n_it = h_count * nq;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&stat_full[i], 32);
      mbar_init(&qd_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&ds_full[i], 128);
      mbar_init(&pds_empty[i], 1);
    }
    mbar_init(dkv_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(kv_full, 2 * AT_T128);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(sK + c * AT_C128, &tmK, kv_full, g * 128 + c * 64, s0 + k0);
        tma_load_2d(sV + c * AT_C128, &tmV, kv_full, g * 128 + c * 64, s0 + k0);
      }
    }
    int issued[2] = {0, 0};
    for (int it = 0; it < n_it; ++it) {
      const int st = it & 1;
      const int head = g * a.group + h_first + it / nq;
      const int q0 = k0 + (it % nq) * 64;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&qd_empty[st], ((uint32_t)(it >> 1) & 1u) ^ 1u, kErrAtEmpty) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&qd_full[st], 2 * AT_T64);
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(sQ + st * AT_T64 + c * AT_C64, &tmQ, &qd_full[st], head * 128 + c * 64, s0 + q0);
          tma_load_2d(sDO + st * AT_T64 + c * AT_C64, &tmDO, &qd_full[st], head * 128 + c * 64, s0 + q0);
        }
      }
      issued[st]++;
      float* sl = stats + st * 128;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = lane + e * 32;
        const int q = q0 + i;
        const size_t off = (size_t)head * a.stat_stride + s0 + q;
        sl[i] = q < len ? a.lse[off] : INFINITY;       // rows past the sample: P = 0
        sl[64 + i] = q < len ? a.dd[off] : 0.f;
      }
      mbar_arrive(&stat_full[st]);
    }
    if (lane == 0) {
      drain_slot(kv_full, 1);
      for (int st = 0; st < 2; ++st) drain_slot(&qd_full[st], issued[st]);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 64, false, false);
      constexpr uint32_t IDESC_G = idesc_bf16_f32(128, 128, false, true);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(kv_full, 0, kErrAtQ);
      auto issue_sdp = [&](int it) -> bool {
        const int st = it & 1;
        const uint32_t use = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(&qd_full[st], use, kErrAtKv)) return false;
        if (!mbar_wait(&s_empty[st], use ^ 1u, kErrAtSEmpty)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + st * AT_T64), do_addr = smem_u32(sDO + st * AT_T64);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tmem + st * 64, desc_kmajor(k_addr, kk, AT_C128), desc_kmajor(q_addr, kk, AT_C64), IDESC_S,
                     kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tmem + 128 + st * 64, desc_kmajor(v_addr, kk, AT_C128), desc_kmajor(do_addr, kk, AT_C64),
                     IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[st]);
        return true;
      };
      if (ok) {
        tc_fence_after();
        ok = issue_sdp(0);
      }
      for (int it = 0; it < n_it && ok; ++it) {
        if (it + 1 < n_it && !issue_sdp(it + 1)) { ok = false; break; }
        const int st = it & 1;
        if (!mbar_wait(&ds_full[st], (uint32_t)(it >> 1) & 1u, kErrAtDs)) { ok = false; break; }
        tc_fence_after();
        const uint32_t pt = smem_u32(sPt + st * AT_C128), dst = smem_u32(sDSt + st * AT_C128);
        const uint32_t q_addr = smem_u32(sQ + st * AT_T64), do_addr = smem_u32(sDO + st * AT_T64);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_f16(tmem + 256, desc_kmajor(pt, kk, AT_C128), desc_mnmajor(do_addr, kk, AT_C64), IDESC_G,
                     (it > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_f16(tmem + 384, desc_kmajor(dst, kk, AT_C128), desc_mnmajor(q_addr, kk, AT_C64), IDESC_G,
                     (it > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&pds_empty[st]);
        tc_commit(&qd_empty[st]);
      }
      if (ok) {
        tc_commit(dkv_done);
        mbar_wait(dkv_done, 0, kErrAtDone);
      }
    }
  } else {
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(q4 * 32) << 16);
    const bool row_ok = r < rows_valid;
    const int kpos = k0 + r;                    // key index within the sample
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int st = it & 1;
      const uint32_t use = (uint32_t)(it >> 1) & 1u;
      if (!warp_wait(&s_full[st], use, kErrAtS) || !warp_wait(&stat_full[st], use, kErrAtStat) ||
          !warp_wait(&pds_empty[st], use ^ 1u, kErrAtDsEmpty)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int q0 = k0 + (it % nq) * 64;
      const int first = kpos - q0;              // queries q0 + i with i >= first see this key
      const float* sl = stats + st * 128;
      uint32_t x[2][32], y[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld_32x32b_x32(t_lane + st * 64 + c * 32, x[c]);
        tmem_ld_32x32b_x32(t_lane + 128 + st * 64 + c * 32, y[c]);
      }
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float p[32], ds[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int qq = c * 32 + i;
          const float pv = qq >= first ? fast_exp2(fmaf(__uint_as_float(x[c][i]), a.scale_log2, -sl[qq])) : 0.f;
          p[i] = pv;
          ds[i] = pv * (__uint_as_float(y[c][i]) - sl[64 + qq]);
        }
        store_row_units(sPt + st * AT_C128, r, c * 4, p);
        store_row_units(sDSt + st * AT_C128, r, c * 4, ds);
      }
      tc_fence_before();
      mbar_arrive(&s_empty[st]);
      fence_proxy_async_smem();
      mbar_arrive(&ds_full[st]);
    }
    if (ok && a.split_heads && warp_wait(dkv_done, 0, kErrAtDone)) {
      tc_fence_after();
      const size_t grow = (size_t)s0 + kpos;
      const size_t off = ((size_t)h_first * a.n_rows + grow) * (size_t)(a.num_kv_heads * 128) + g * 128;
      store_acc_row(t_lane + 256, 1.f, nullptr, nullptr, a.part_dv + off, nullptr, row_ok);
      store_acc_row(t_lane + 384, 1.f, nullptr, nullptr, a.part_dk + off, nullptr, row_ok);
    } else if (ok && warp_wait(dkv_done, 0, kErrAtDone)) {
      tc_fence_after();
      const size_t grow = (size_t)s0 + kpos;
      const int hkv128 = a.num_kv_heads * 128;
      float* fv = (a.bf16_mask & 4) ? nullptr : a.dv + grow * (size_t)hkv128 + g * 128;
      __nv_bfloat16* bv = (a.bf16_mask & 4) ? a.dqkv + grow * a.dqkv_stride + a.dv_col + g * 128 : nullptr;
      store_acc_row(t_lane + 256, 1.f, nullptr, nullptr, fv, bv, row_ok);
      const bool rope = a.rope_cos != nullptr;
      const float* cr = rope && row_ok ? a.rope_cos + grow * a.rope_stride : nullptr;
      const float* sr = rope && row_ok ? a.rope_sin + grow * a.rope_stride : nullptr;
      float* fk = (a.bf16_mask & 2) ? nullptr : a.dk + grow * (size_t)hkv128 + g * 128;
      __nv_bfloat16* bk = (a.bf16_mask & 2) ? a.dqkv + grow * a.dqkv_stride + a.dk_col + g * 128 : nullptr;
      store_acc_row(t_lane + 384, a.scale, cr, sr, fk, bk, row_ok);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Head-split finish: per row of the tile and KV head, sum the group's fp32
// dK / dV partials, scale dK, undo RoPE on it and store both (fp32 rows or
// bf16 into d(qkv)), the same outputs as the single-pass epilogue.
__global__ void __launch_bounds__(128) kv_split_finish_kernel(FaBwdArgs a) {
  const int tile = blockIdx.x, g = blockIdx.y, r = threadIdx.x;
  const int s0 = a.tiles[3 * tile], len = a.tiles[3 * tile + 1], k0 = a.tiles[3 * tile + 2];
  if (k0 + r >= len) return;
  const size_t grow = (size_t)s0 + k0 + r;
  const int hkv128 = a.num_kv_heads * 128;
  const size_t plane = (size_t)a.n_rows * hkv128;
  for (int which = 0; which < 2; ++which) {   // 0: dV, 1: dK
    const float* src = (which == 0 ? a.part_dv : a.part_dk) + grow * hkv128 + g * 128;
    const bool bf = (a.bf16_mask & (which == 0 ? 4 : 2)) != 0;
    const float scale = which == 0 ? 1.f : a.scale;
    const bool rope = which == 1 && a.rope_cos != nullptr;
    for (int h = 0; h < 64; h += 32) {
      float x[32], y[32];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 u = make_float4(0.f, 0.f, 0.f, 0.f), v = u;
        for (int p = 0; p < a.group; ++p) {
          const float4 pu = *reinterpret_cast<const float4*>(src + p * plane + h + i);
          const float4 pv = *reinterpret_cast<const float4*>(src + p * plane + 64 + h + i);
          u.x += pu.x; u.y += pu.y; u.z += pu.z; u.w += pu.w;
          v.x += pv.x; v.y += pv.y; v.z += pv.z; v.w += pv.w;
        }
        x[i] = u.x * scale; x[i + 1] = u.y * scale; x[i + 2] = u.z * scale; x[i + 3] = u.w * scale;
        y[i] = v.x * scale; y[i + 1] = v.y * scale; y[i + 2] = v.z * scale; y[i + 3] = v.w * scale;
      }
      if (rope) {
        const float* cr = a.rope_cos + grow * a.rope_stride + h;
        const float* sr = a.rope_sin + grow * a.rope_stride + h;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float xa = x[i], yb = y[i];
          x[i] = xa * cr[i] + yb * sr[i];
          y[i] = yb * cr[i] - xa * sr[i];
        }
      }
      if (bf) {
        __nv_bfloat16* dst = a.dqkv + grow * a.dqkv_stride + (which == 0 ? a.dv_col : a.dk_col) + g * 128;
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          *reinterpret_cast<uint32_t*>(dst + h + i) = pack2_bf16(x[i], x[i + 1]);
          *reinterpret_cast<uint32_t*>(dst + 64 + h + i) = pack2_bf16(y[i], y[i + 1]);
        }
      } else {
        float* dst = (which == 0 ? a.dv : a.dk) + grow * hkv128 + g * 128;
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          *reinterpret_cast<float4*>(dst + h + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
          *reinterpret_cast<float4*>(dst + 64 + h + i) = make_float4(y[i], y[i + 1], y[i + 2], y[i + 3]);
        }
      }
    }
  }
}

static bool at_set_smem() {
  cudaFuncSetAttribute(fa_bwd_q_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AQ_SMEM);
  cudaFuncSetAttribute(fa_bwd_kv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AKV_SMEM);
  return true;
}

static void check_heads(const torch::Tensor& t, const char* name, int64_t heads) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, "attn_bwd_tc: ", name, " must be bf16 CUDA");
  TORCH_CHECK(t.dim() == 3 && t.size(1) == heads && t.size(2) == 128 && t.stride(2) == 1 && t.stride(1) == 128,
              "attn_bwd_tc: ", name, " must be [n, H, 128] with adjacent heads");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "attn_bwd_tc: ", name, " rows must be 16-byte aligned");
}

}  // namespace dsv

// dq [n, Hq, 128], dk / dv [n, Hkv, 128] fp32 (rows outside every sample are
// left untouched) or bf16 into dqkv per bf16_mask; o / d_o bf16 [n, Hq*128];
// lse [Hq, >= n] from the forward; dd [Hq, same stride] is written (scratch).
void dsv_attn_bwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor d_o,
                     torch::Tensor tiles, torch::Tensor lse, torch::Tensor dd, c10::optional<torch::Tensor> dq,
                     c10::optional<torch::Tensor> dk, c10::optional<torch::Tensor> dv, double scale,
                     c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin,
                     c10::optional<torch::Tensor> dqkv, int64_t bf16_mask) {
  using namespace dsv;
  const int T = (int)tiles.size(0);
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  const int64_t n = q.size(0), hq = q.size(1), hkv = k.size(1);
  check_heads(q, "q", hq);
  check_heads(k, "k", hkv);
  check_heads(v, "v", hkv);
  TORCH_CHECK(hq % hkv == 0 && k.size(0) == n && v.size(0) == n, "attn_bwd_tc: q/k/v shapes");
  TORCH_CHECK(tiles.scalar_type() == at::kInt && tiles.dim() == 2 && tiles.size(1) == 3 && tiles.is_contiguous(),
              "attn_bwd_tc: tiles must be int32 [T, 3] (128-row tiles)");
  for (const torch::Tensor* t : {&o, &d_o}) {
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->size(0) == n && t->size(1) >= hq * 128 &&
                    t->stride(1) == 1 && (t->stride(0) * 2) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "attn_bwd_tc: o / d_o must be bf16 [n, >= Hq*128] with 16-byte aligned rows");
  }
  TORCH_CHECK(lse.scalar_type() == at::kFloat && dd.scalar_type() == at::kFloat && lse.dim() == 2 && dd.dim() == 2 &&
                  lse.size(0) >= hq && lse.size(1) >= n && lse.stride(1) == 1 && dd.strides() == lse.strides() &&
                  dd.size(0) >= hq && dd.size(1) >= n,
              "attn_bwd_tc: lse / dd must be fp32 [Hq, >= n] with the same strides");
  TORCH_CHECK(bf16_mask >= 0 && bf16_mask <= 7, "attn_bwd_tc: bf16_mask is a 3-bit mask");
  FaBwdArgs a{};
  const int64_t want[3] = {hq, hkv, hkv};
  const c10::optional<torch::Tensor>* outs[3] = {&dq, &dk, &dv};
  float* ptrs[3] = {nullptr, nullptr, nullptr};
  for (int i = 0; i < 3; ++i) {
    if (bf16_mask & (1 << i)) continue;
    const auto& t = *outs[i];
    TORCH_CHECK(t.has_value() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == n * want[i] * 128,
                "attn_bwd_tc: fp32 output ", i, " must be [n, H, 128]");
    ptrs[i] = t->data_ptr<float>();
  }
  if (bf16_mask != 0) {
    TORCH_CHECK(dqkv.has_value() && dqkv->scalar_type() == at::kBFloat16 && dqkv->dim() == 2 && dqkv->size(0) == n &&
                    dqkv->stride(1) == 1 && (dqkv->stride(0) * 2) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(dqkv->data_ptr()) % 16 == 0 && dqkv->size(1) >= (hq + 2 * hkv) * 128,
                "attn_bwd_tc: dqkv must be bf16 [n, (Hq+2Hkv)*128] with 16-byte aligned rows");
    a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv->data_ptr());
    a.dqkv_stride = (int)dqkv->stride(0);
    a.dq_col = 0;
    a.dk_col = (int)(hq * 128);
    a.dv_col = (int)((hq + hkv) * 128);
  }
  if (rope_cos.has_value()) {
    TORCH_CHECK(rope_sin.has_value() && rope_cos->scalar_type() == at::kFloat && rope_sin->scalar_type() == at::kFloat &&
                    rope_cos->dim() == 2 && rope_cos->size(0) >= n && rope_cos->size(1) == 64 &&
                    rope_cos->stride(1) == 1 && rope_sin->strides() == rope_cos->strides() &&
                    rope_cos->stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(rope_cos->data_ptr()) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(rope_sin->data_ptr()) % 16 == 0,
                "attn_bwd_tc: rope cos / sin must be fp32 [>= n, 64] with 16-byte aligned rows");
    a.rope_cos = rope_cos->data_ptr<float>();
    a.rope_sin = rope_sin->data_ptr<float>();
    a.rope_stride = (int)rope_cos->stride(0);
  }
  a.tiles = tiles.data_ptr<int>();
  a.num_tiles = T;
  a.num_heads = (int)hq;
  a.num_kv_heads = (int)hkv;
  a.group = (int)(hq / hkv);
  a.o = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  a.o_stride = (int)o.stride(0);
  a.d_o = reinterpret_cast<const __nv_bfloat16*>(d_o.data_ptr());
  a.do_stride = (int)d_o.stride(0);
  a.lse = lse.data_ptr<float>();
  a.dd = dd.data_ptr<float>();
  a.stat_stride = (int)lse.stride(0);
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.dq = ptrs[0];
  a.dk = ptrs[1];
  a.dv = ptrs[2];
  a.bf16_mask = (int)bf16_mask;
  static bool attr = at_set_smem();
  (void)attr;
  auto stream = at::cuda::getCurrentCUDAStream();
  {
    CUtensorMap tq = make_tmap_bf16(q.data_ptr(), n, (uint64_t)hq * 128, q.stride(0), 128);
    CUtensorMap tdo = make_tmap_bf16(d_o.data_ptr(), n, (uint64_t)hq * 128, d_o.stride(0), 128);
    CUtensorMap tk = make_tmap_bf16(k.data_ptr(), n, (uint64_t)hkv * 128, k.stride(0), 64);
    CUtensorMap tv = make_tmap_bf16(v.data_ptr(), n, (uint64_t)hkv * 128, v.stride(0), 64);
    fa_bwd_q_tc_kernel<<<dim3((unsigned)T, (unsigned)hq), AT_THREADS, AQ_SMEM, stream>>>(tq, tdo, tk, tv, a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  {
    CUtensorMap tq = make_tmap_bf16(q.data_ptr(), n, (uint64_t)hq * 128, q.stride(0), 64);
    CUtensorMap tdo = make_tmap_bf16(d_o.data_ptr(), n, (uint64_t)hq * 128, d_o.stride(0), 64);
    CUtensorMap tk = make_tmap_bf16(k.data_ptr(), n, (uint64_t)hkv * 128, k.stride(0), 128);
    CUtensorMap tv = make_tmap_bf16(v.data_ptr(), n, (uint64_t)hkv * 128, v.stride(0), 128);
    // Few (key tile, KV head) CTAs for the SMs (high TP): one CTA per query
    // head of the group instead, partials summed by a finish kernel.
    const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
    at::Tensor part;
    if (a.group > 1 && (int64_t)T * hkv < sms) {
      part = at::empty({2, (int64_t)a.group, n, hkv * 128}, q.options().dtype(at::kFloat));
      a.split_heads = 1;
      a.part_dk = part.data_ptr<float>();
      a.part_dv = a.part_dk + (size_t)a.group * n * hkv * 128;
      a.n_rows = (int)n;
    }
    fa_bwd_kv_tc_kernel<<<dim3((unsigned)T, (unsigned)(a.split_heads ? hkv * a.group : hkv)), AT_THREADS, AKV_SMEM,
                          stream>>>(tq, tdo, tk, tv, a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    if (a.split_heads) {
      kv_split_finish_kernel<<<dim3((unsigned)T, (unsigned)hkv), 128, 0, stream>>>(a);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
    }
  }
}

DSV_ERROR_ACCESSOR(dsv_read_error_attn_bwd_tc)
