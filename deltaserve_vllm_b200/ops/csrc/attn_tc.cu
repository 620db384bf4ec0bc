// Causal GQA flash attention on the 5th-generation tensor cores (sm_100a):
// the forward for paged-KV prefill (serving, chunked prefill included) and
// for packed dense samples (the trainer's recompute, with the row
// log-sum-exp and D = rowsum(dO * O) that the backward needs).
//
// One CTA = 128 queries x 1 query head, 192 threads in three roles:
//
//   warp 0      TMA producer: the Q tile once, then K and V tiles of 128
//               keys into a 2-stage ring (paged: one box per page segment).
//   warp 1      MMA issuer (one elected thread) and TMEM owner:
//               S_j = Q K_j^T into one of two TMEM score buffers, then
//               O += P_j V_j into the TMEM output accumulator. S_{j+1} is
//               issued before waiting for P_j, so the next scores are
//               computed while the softmax warps work on this tile.
//   warps 2-5   softmax: thread t owns query row t (TMEM lane t): reads its
//               128 scores with tcgen05.ld, masks, updates the running max
//               and sum (base-2 domain), writes bf16 P into shared memory in
//               the 128-byte-swizzled K-major layout the MMA reads, and
//               rescales its O row in TMEM (tcgen05.ld / st) when its max
//               grew by more than 2^8 (lazy rescaling: below that the old
//               reference max stays). After the last tile: O / l stored as
//               bf16, and the optional statistics.
//
// Shared memory (all tiles are two 64-column chunks of [128 rows x 128 B],
// 128-byte swizzle, i.e. the TMA box layout): Q, K[2], V[2], P = 192 KB, so
// one CTA per SM; this also keeps it from sharing an SM with the tcgen05
// GEMMs (> 190 KB each), whose TMEM it would otherwise compete for.
// TMEM: S[2] in columns 0-255, O in 256-383 (512 allocated).
//
// Operand forms (instruction descriptor bf16 x bf16 -> fp32, M = N = 128):
//   S = Q K^T : A = Q  K-major, B = K K-major (keys x d, d contiguous)
//   O += P V  : A = P  K-major, B = V MN-major (keys x d, d contiguous = N)
//
// Every wait is bounded (common.cuh); a timeout records an error code that
// the host reads with read_error() and the kernel returns.
//
// Reference behaviour: the reference serves through vLLM's FlashAttention /
// FlashInfer prefill kernels and computes the trainer's attention with
// deltaserve-plugin/deltaserve/bwd_services/common/attention.py; this is the
// same math (softmax(QK^T * scale) V, causal, GQA).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "attn_tc.cuh"
#include "tmap.h"

namespace dsv {

constexpr int FA_ROWS = 128;                 // queries per CTA = keys per tile
constexpr int FA_THREADS = 192;
constexpr int FA_CHUNK = 128 * 128;          // one [128 rows x 64 cols] bf16 chunk (bytes)
constexpr int FA_TILE = 2 * FA_CHUNK;        // a 128 x 128 bf16 tile
constexpr int FA_SMEM = 6 * FA_TILE + 1024 + 256;
constexpr uint32_t FA_TMEM_COLS = 512;
constexpr uint32_t FA_O_COL = 256;
constexpr float FA_RESCALE_LOG2 = 8.f;       // lazy-rescaling threshold (log2 units)

enum : int {
  kErrFaQ = 0x4101,
  kErrFaKv = 0x4102,
  kErrFaS = 0x4103,
  kErrFaP = 0x4104,
  kErrFaO = 0x4105,
  kErrFaEmpty = 0x4106,
  kErrFaSEmpty = 0x4107,
  kErrFaDrain = 0x4108,
};

struct FaFwdArgs {
  // paged: tile_info [tiles, 2] = (sequence, first query); dense: [tiles, 3]
  // = (first row of the sample, sample length, first query)
  const int* tile_info;
  const int* block_tables;  // paged [S, max_blocks]
  int max_blocks;
  const int* cu_q;          // paged [S+1]
  const int* ctx_lens;      // paged [S]
  int block_size, box_rows; // paged: page size, rows per K/V box (min(block_size, 128))
  int num_blocks;           // paged: pages in the cache (bounds-check build)
  int num_kv_heads, group;
  __nv_bfloat16* out;       // [T, ...] row stride out_stride, head h at h * 128
  int out_stride;
  float* lse;               // dense, optional: [Hq, stat_stride] log-sum-exp (base 2)
  const float* d_o;         // dense, optional: [n, Hq * 128] fp32, row stride do_stride
  int do_stride;
  float* dd;                // dense, optional: [Hq, stat_stride] rowsum(dO * O)
  int stat_stride;
  float scale_log2;
};

template <bool PAGED>
__global__ void __launch_bounds__(FA_THREADS, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, FaFwdArgs a) {
  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + FA_TILE;          // [2][tile]
  uint8_t* sV = sK + 2 * FA_TILE;      // [2][tile]
  uint8_t* sP = sV + 2 * FA_TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + FA_TILE);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2]
  uint64_t* s_empty = bars + 9;   // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* o_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tile = blockIdx.x, head = blockIdx.y;
  const int kvh = head / a.group;

  // Geometry of this query tile.
  int q_begin, q_len, pos0, qt0, seq = 0;
  if constexpr (PAGED) {
    seq = a.tile_info[2 * tile];
    qt0 = a.tile_info[2 * tile + 1];
    q_begin = a.cu_q[seq];
    q_len = a.cu_q[seq + 1] - q_begin;
    pos0 = a.ctx_lens[seq] - q_len;
  } else {
    q_begin = a.tile_info[3 * tile];
    q_len = a.tile_info[3 * tile + 1];
    qt0 = a.tile_info[3 * tile + 2];
    pos0 = 0;
  }
  const int rows_valid = min(FA_ROWS, q_len - qt0);
  const int kv_end = pos0 + qt0 + rows_valid;  // keys visible to the tile's last query
  const int n_kb = (kv_end + FA_ROWS - 1) / FA_ROWS;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, FA_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, FA_TILE);
      tma_load_2d(sQ, &tmQ, q_full, head * 128, q_begin + qt0);
      tma_load_2d(sQ + FA_CHUNK, &tmQ, q_full, head * 128 + 64, q_begin + qt0);
      const int* btab = PAGED ? a.block_tables + (size_t)seq * a.max_blocks : nullptr;
      int issued[2] = {0, 0};
      bool ok = true;
      for (int kb = 0; kb < n_kb && ok; ++kb) {
        const int st = kb & 1;
        const uint32_t ph = (uint32_t)(kb >> 1) & 1u;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, kErrFaEmpty)) { ok = false; break; }
        uint8_t* dk = sK + st * FA_TILE;
        uint8_t* dv = sV + st * FA_TILE;
        mbar_arrive_expect_tx(&k_full[st], FA_TILE);
        if constexpr (PAGED) {
          const int R = a.box_rows;
          for (int s = 0; s < FA_ROWS / R; ++s) {
            const int key0 = kb * FA_ROWS + s * R;
            const bool in = key0 < kv_end;
            int page = btab[in ? key0 / a.block_size : 0];
            if (!DSV_IN_BOUNDS(page, a.num_blocks)) page = 0;
            const int y = (page * a.num_kv_heads + kvh) * a.block_size + (in ? key0 % a.block_size : 0);
            tma_load_2d(dk + s * R * 128, &tmK, &k_full[st], 0, y);
            tma_load_2d(dk + FA_CHUNK + s * R * 128, &tmK, &k_full[st], 64, y);
          }
        } else {
          const int y = q_begin + kb * FA_ROWS;
          tma_load_2d(dk, &tmK, &k_full[st], kvh * 128, y);
          tma_load_2d(dk + FA_CHUNK, &tmK, &k_full[st], kvh * 128 + 64, y);
        }
        mbar_arrive_expect_tx(&v_full[st], FA_TILE);
        if constexpr (PAGED) {
          const int R = a.box_rows;
          for (int s = 0; s < FA_ROWS / R; ++s) {
            const int key0 = kb * FA_ROWS + s * R;
            const bool in = key0 < kv_end;
            int page = btab[in ? key0 / a.block_size : 0];
            if (!DSV_IN_BOUNDS(page, a.num_blocks)) page = 0;
            const int y = (page * a.num_kv_heads + kvh) * a.block_size + (in ? key0 % a.block_size : 0);
            tma_load_2d(dv + s * R * 128, &tmV, &v_full[st], 0, y);
            tma_load_2d(dv + FA_CHUNK + s * R * 128, &tmV, &v_full[st], 64, y);
          }
        } else {
          const int y = q_begin + kb * FA_ROWS;
          tma_load_2d(dv, &tmV, &v_full[st], kvh * 128, y);
          tma_load_2d(dv + FA_CHUNK, &tmV, &v_full[st], kvh * 128 + 64, y);
        }
        issued[st]++;
      }
      // Drain: the copies this thread issued have landed before the CTA exits.
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(q_full, 0)) {
        if (globaltimer_ns() - t0 > kWaitNs) { set_error(kErrFaDrain); break; }
      }
      for (int st = 0; st < 2; ++st) {
        if (issued[st] == 0) continue;
        const uint32_t par = (uint32_t)(issued[st] - 1) & 1u;
        t0 = globaltimer_ns();
        while (!mbar_try_wait(&k_full[st], par) || !mbar_try_wait(&v_full[st], par)) {
          if (globaltimer_ns() - t0 > kWaitNs) { set_error(kErrFaDrain); break; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(128, 128, false, true);
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, kErrFaQ);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t use = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&k_full[st], use, kErrFaKv)) return false;
        if (!mbar_wait(&s_empty[st], use ^ 1u, kErrFaSEmpty)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * FA_TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tmem + st * 128, desc_kmajor(q_addr, kk, FA_CHUNK), desc_kmajor(k_addr, kk, FA_CHUNK), IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[st]);
        return true;
      };
      if (ok) {
        tc_fence_after();
        ok = issue_s(0);
      }
      for (int j = 0; j < n_kb && ok; ++j) {
        if (j + 1 < n_kb && !issue_s(j + 1)) { ok = false; break; }
        const int st = j & 1;
        if (!mbar_wait(p_full, (uint32_t)j & 1u, kErrFaP)) { ok = false; break; }
        if (!mbar_wait(&v_full[st], (uint32_t)(j >> 1) & 1u, kErrFaKv)) { ok = false; break; }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * FA_TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(tmem + FA_O_COL, desc_kmajor(p_addr, kk, FA_CHUNK), desc_mnmajor(v_addr, kk, FA_CHUNK), IDESC_O,
                     (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(o_done);
        tc_commit(&kv_empty[st]);
      }
      // The stage-release commits land before the CTA exits.
      for (int st = 0; st < 2 && ok; ++st) {
        const int uses = (n_kb - st + 1) / 2;
        if (uses > 0) mbar_wait(&kv_empty[st], (uint32_t)(uses - 1) & 1u, kErrFaDrain);
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;                          // query row of this thread
    const uint32_t t_lane = tmem + ((uint32_t)(q4 * 32) << 16);
    const int qpos = pos0 + qt0 + r;                       // its position in the sequence
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    uint8_t* prow = sP + r * 128;
    for (int j = 0; j < n_kb; ++j) {
      const int st = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[st], (uint32_t)(j >> 1) & 1u, kErrFaS))) { ok = false; break; }
      tc_fence_after();
      // All four 32-column loads in flight before one wait; scores stay raw
      // (the scale is folded into the exponent's FMA below).
      float s[128];
      {
        uint32_t v0[32], v1[32], v2[32], v3[32];
        tmem_ld_32x32b_x32(t_lane + st * 128 + 0, v0);
        tmem_ld_32x32b_x32(t_lane + st * 128 + 32, v1);
        tmem_ld_32x32b_x32(t_lane + st * 128 + 64, v2);
        tmem_ld_32x32b_x32(t_lane + st * 128 + 96, v3);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(v0[i]);
          s[32 + i] = __uint_as_float(v1[i]);
          s[64 + i] = __uint_as_float(v2[i]);
          s[96 + i] = __uint_as_float(v3[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[st]);
      const int key0 = j * FA_ROWS;
      const int lim = min(qpos + 1, kv_end) - key0;        // keys [key0, key0 + lim) are visible
      if (lim < FA_ROWS) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= lim) s[i] = -INFINITY;
      }
      // Row max and sum as 8 independent chains (a single 128-long chain of
      // dependent max / add instructions dominated the loop).
      float red[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) red[c] = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) red[i & 7] = fmaxf(red[i & 7], s[i]);
      const float tile_max = fmaxf(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])),
                                   fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7])));
      // Lazy rescaling: the reference max m moves (and O, l are rescaled)
      // only when the row max exceeds it by more than FA_RESCALE_LOG2; below
      // that, P = exp2(s - m) stays under 2^FA_RESCALE_LOG2, exact enough in
      // bf16 / fp32, and O and l keep one consistent reference.
      const float row_max = tile_max * a.scale_log2;        // base-2 scaled domain
      const bool move = m == -INFINITY || row_max > m + FA_RESCALE_LOG2;
      const float mx = move ? fmaxf(m, row_max) : m;
      const float corr = (m == -INFINITY) ? 0.f : (move ? fast_exp2(m - mx) : 1.f);
      const float mref = (mx == -INFINITY) ? 0.f : mx;
#pragma unroll
      for (int c = 0; c < 8; ++c) red[c] = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        s[i] = fast_exp2(fmaf(s[i], a.scale_log2, -mref));
        red[i & 7] += s[i];
      }
      const float sum = ((red[0] + red[1]) + (red[2] + red[3])) + ((red[4] + red[5]) + (red[6] + red[7]));
      l = l * corr + sum;
      m = mx;
      if (j > 0) {
        // PV_{j-1} finished: P may be overwritten and O is stable.
        if (!__all_sync(0xffffffffu, mbar_wait(o_done, (uint32_t)(j - 1) & 1u, kErrFaO))) { ok = false; break; }
        tc_fence_after();
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        uint4 w;
        w.x = pack2_bf16(s[u * 8 + 0], s[u * 8 + 1]);
        w.y = pack2_bf16(s[u * 8 + 2], s[u * 8 + 3]);
        w.z = pack2_bf16(s[u * 8 + 4], s[u * 8 + 5]);
        w.w = pack2_bf16(s[u * 8 + 6], s[u * 8 + 7]);
        *reinterpret_cast<uint4*>(prow + (u >> 3) * FA_CHUNK + (((u & 7) ^ (r & 7)) << 4)) = w;
      }
      if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(t_lane + FA_O_COL + c * 32, v0);
          tmem_ld_32x32b_x32(t_lane + FA_O_COL + (c + 1) * 32, v1);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v0[i] = __float_as_uint(__uint_as_float(v0[i]) * corr);
            v1[i] = __float_as_uint(__uint_as_float(v1[i]) * corr);
          }
          tmem_st_32x32b_x32(t_lane + FA_O_COL + c * 32, v0);
          tmem_st_32x32b_x32(t_lane + FA_O_COL + (c + 1) * 32, v1);
        }
        tmem_st_wait();
      }
      fence_proxy_async_smem();   // P (generic-proxy stores) visible to the tensor core
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(o_done, (uint32_t)(n_kb - 1) & 1u, kErrFaO))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = r < rows_valid;
      const size_t grow = (size_t)q_begin + qt0 + r;
      __nv_bfloat16* dst = a.out + grow * a.out_stride + head * 128;
      const float* dor = (!PAGED && a.d_o != nullptr && row_ok) ? a.d_o + grow * a.do_stride + head * 128 : nullptr;
      float dsum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_lane + FA_O_COL + c * 32, v);
        tmem_ld_wait();
        if (row_ok) {
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(v[i]) * inv;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w;
            w.x = pack2_bf16(o[u * 8 + 0], o[u * 8 + 1]);
            w.y = pack2_bf16(o[u * 8 + 2], o[u * 8 + 3]);
            w.z = pack2_bf16(o[u * 8 + 4], o[u * 8 + 5]);
            w.w = pack2_bf16(o[u * 8 + 6], o[u * 8 + 7]);
            *reinterpret_cast<uint4*>(dst + c * 32 + u * 8) = w;
          }
          if (dor != nullptr) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const float4 g = *reinterpret_cast<const float4*>(dor + c * 32 + u * 4);
              dsum += g.x * o[u * 4] + g.y * o[u * 4 + 1] + g.z * o[u * 4 + 2] + g.w * o[u * 4 + 3];
            }
          }
        }
      }
      if (!PAGED && row_ok) {
        if (a.lse != nullptr) a.lse[(size_t)head * a.stat_stride + grow] = m + __log2f(l);
        if (a.dd != nullptr) a.dd[(size_t)head * a.stat_stride + grow] = dsum;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, FA_TMEM_COLS);
  }
}

static bool fa_set_smem() {
  cudaFuncSetAttribute(fa_fwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
  cudaFuncSetAttribute(fa_fwd_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
  return true;
}

}  // namespace dsv

// ---------------------------------------------------------------- bindings

// Same contract as dsv_paged_prefill, with tile_info built for 128-query tiles.
void dsv_paged_prefill_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                          torch::Tensor cu_q, torch::Tensor ctx_lens, torch::Tensor tile_info, torch::Tensor out,
                          int64_t num_heads, double scale) {
  using namespace dsv;
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16,
              "prefill_tc: bf16 CUDA tensors");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 128, "prefill_tc: cache [blocks, Hkv, BS, 128]");
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1, "prefill_tc: contiguous rows");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "prefill_tc: contiguous cache");
  const int num_tiles = (int)tile_info.size(0);
  if (num_tiles == 0) return;
  const int bs = (int)k_cache.size(2);
  const int box = bs < 128 ? bs : 128;
  TORCH_CHECK(box % 8 == 0 && 128 % box == 0 && bs % box == 0, "prefill_tc: block size must divide into 128-key tiles");
  c10::cuda::CUDAGuard guard(q.device());
  static bool attr = fa_set_smem();
  (void)attr;
  const int hkv = (int)k_cache.size(1);
  const uint64_t cache_rows = (uint64_t)k_cache.size(0) * hkv * bs;
  CUtensorMap tq = make_tmap_bf16(q.data_ptr(), q.size(0), (uint64_t)num_heads * 128, q.stride(0), 128);
  CUtensorMap tk = make_tmap_bf16(k_cache.data_ptr(), cache_rows, 128, 128, box);
  CUtensorMap tv = make_tmap_bf16(v_cache.data_ptr(), cache_rows, 128, 128, box);
  FaFwdArgs a{};
  a.tile_info = tile_info.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.max_blocks = (int)block_tables.size(1);
  a.cu_q = cu_q.data_ptr<int>();
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.block_size = bs;
  a.box_rows = box;
  a.num_blocks = (int)k_cache.size(0);
  a.num_kv_heads = hkv;
  a.group = (int)(num_heads / hkv);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_stride = (int)out.stride(0);
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  dim3 grid(num_tiles, (unsigned)num_heads);
  fa_fwd_tc_kernel<true><<<grid, FA_THREADS, FA_SMEM, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Dense varlen forward over packed samples: q [n, Hq*128 (row stride)], k / v
// [n, Hkv*128 (row stride)], tiles [num_tiles, 3] built for 128-row tiles.
// Writes out (bf16); with lse / dd given (fp32 [Hq, stat_stride]) also the
// base-2 row log-sum-exp and, from d_o (fp32 [n, Hq*128]), rowsum(dO * O).
void dsv_attn_fwd_dense_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor tiles, torch::Tensor out,
                           int64_t num_heads, int64_t num_kv_heads, double scale, c10::optional<torch::Tensor> lse,
                           c10::optional<torch::Tensor> d_o, c10::optional<torch::Tensor> dd) {
  using namespace dsv;
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16,
              "attn_fwd_dense_tc: bf16 CUDA tensors");
  TORCH_CHECK(q.stride(-1) == 1 && k.stride(-1) == 1 && v.stride(-1) == 1 && out.stride(-1) == 1,
              "attn_fwd_dense_tc: contiguous rows");
  const int num_tiles = (int)tiles.size(0);
  if (num_tiles == 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  static bool attr = fa_set_smem();
  (void)attr;
  const int64_t n = q.size(0);
  CUtensorMap tq = make_tmap_bf16(q.data_ptr(), n, (uint64_t)num_heads * 128, q.stride(0), 128);
  CUtensorMap tk = make_tmap_bf16(k.data_ptr(), n, (uint64_t)num_kv_heads * 128, k.stride(0), 128);
  CUtensorMap tv = make_tmap_bf16(v.data_ptr(), n, (uint64_t)num_kv_heads * 128, v.stride(0), 128);
  FaFwdArgs a{};
  a.tile_info = tiles.data_ptr<int>();
  a.num_kv_heads = (int)num_kv_heads;
  a.group = (int)(num_heads / num_kv_heads);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_stride = (int)out.stride(0);
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  if (lse.has_value()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->size(0) >= num_heads, "attn_fwd_dense_tc: lse [Hq, >= n]");
    a.lse = lse->data_ptr<float>();
    a.stat_stride = (int)lse->stride(0);
  }
  if (d_o.has_value() && dd.has_value()) {
    TORCH_CHECK(d_o->scalar_type() == at::kFloat && d_o->stride(-1) == 1, "attn_fwd_dense_tc: d_o fp32 rows");
    TORCH_CHECK(dd->scalar_type() == at::kFloat && dd->stride(0) == (lse.has_value() ? lse->stride(0) : dd->stride(0)),
                "attn_fwd_dense_tc: dd [Hq, stat_stride]");
    a.d_o = d_o->data_ptr<float>();
    a.do_stride = (int)d_o->stride(0);
    a.dd = dd->data_ptr<float>();
    a.stat_stride = (int)dd->stride(0);
  }
  dim3 grid(num_tiles, (unsigned)num_heads);
  fa_fwd_tc_kernel<false><<<grid, FA_THREADS, FA_SMEM, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

DSV_ERROR_ACCESSOR(dsv_read_error_attn_tc)
