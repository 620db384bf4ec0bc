// Paged-KV attention for sm_100a: varlen causal prefill (chunked prefill
// included) and split-KV GQA decode, bf16 in, fp32 softmax.
//
// KV cache layout per layer: k_cache / v_cache [num_blocks, Hkv, BS, 128] bf16,
// so one (page, head) is a contiguous BS x 128 tile. A sequence's pages come
// from block_tables[seq, :]. Query i of a sequence with q_len new tokens and
// total context ctx sits at position ctx - q_len + i and sees keys <= that.
//
// Prefill (the warp-level fallback of the tcgen05 kernel in attn_tc.cu, for
// page sizes that do not tile 128 keys): one CTA = 64 queries x 1 head, 4 warps x 16 rows, K/V tiles of 64
// keys double-buffered through cp.async into XOR-swizzled shared memory,
// QK^T and PV on the warp-level tensor-core path (m16n8k16), online softmax
// in fp32 registers.
// Decode: one CTA = (sequence, KV head, KV split): the GQA group's queries
// are the rows of one tensor-core tile and share every K/V byte read; with
// several splits, partial (max, sum, out) go to a workspace and a second
// kernel merges them.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "attn_common.cuh"

namespace dsv {

constexpr int PF_BM = 64;        // queries per CTA
constexpr int PF_BN = 64;        // keys per iteration
constexpr int PF_THREADS = 128;  // 4 warps

struct PrefillArgs {
  const __nv_bfloat16* q;   // [T, ...] row stride q_stride, head h at h*128
  int q_stride;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  const int* block_tables;  // [S, max_blocks]
  int max_blocks;
  const int* cu_q;          // [S+1] query offsets
  const int* ctx_lens;      // [S] total context after this step
  const int* tile_info;     // [num_tiles, 2] = (seq, first query of the tile)
  __nv_bfloat16* out;       // [T, Hq*128] row stride out_stride
  int out_stride;
  int num_kv_heads, group, block_size;
  int num_blocks;           // pages in the cache (the bounds-check build checks page ids against it)
  float scale_log2;         // softmax scale * log2(e)
};

__global__ void __launch_bounds__(PF_THREADS) paged_prefill_kernel(PrefillArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sK = sQ + PF_BM * HD;      // [2][64*128]
  __nv_bfloat16* sV = sK + 2 * PF_BN * HD;  // [2][64*128]

  const int tile = blockIdx.x;
  const int head = blockIdx.y;
  const int kvh = head / a.group;
  const int seq = a.tile_info[2 * tile];
  // first query index within the sequence: tiles list 128-query spans, each
  // covered by gridDim.z CTAs of 64 queries
  const int qt0 = a.tile_info[2 * tile + 1] + (int)blockIdx.z * PF_BM;
  const int q_begin = a.cu_q[seq];
  const int q_len = a.cu_q[seq + 1] - q_begin;
  if (qt0 >= q_len) return;
  const int ctx = a.ctx_lens[seq];
  const int pos0 = ctx - q_len;  // position of query 0
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int* btab = a.block_tables + (size_t)seq * a.max_blocks;

  // Q tile -> smem (rows past the sequence are zero).
  for (int i = tid; i < PF_BM * 16; i += PF_THREADS) {
    int r = i / 16, c = i % 16;
    int qi = qt0 + r;
    bool ok = qi < q_len;
    const __nv_bfloat16* src = a.q + (size_t)(q_begin + (ok ? qi : 0)) * a.q_stride + head * HD + c * 8;
    cp_async16(sQ + swz(r, c), src, ok);
  }
  // Keys visible to the last query of this tile.
  const int last_q = min(qt0 + PF_BM, q_len) - 1;
  const int kv_end = pos0 + last_q + 1;
  const int n_kb = (kv_end + PF_BN - 1) / PF_BN;

  auto load_kv = [&](int kb, int buf) {
    for (int i = tid; i < PF_BN * 16; i += PF_THREADS) {
      int r = i / 16, c = i % 16;
      int kpos = kb * PF_BN + r;
      bool ok = kpos < kv_end;
      int kp = ok ? kpos : 0;
      int page = btab[kp / a.block_size];
      if (!DSV_IN_BOUNDS(page, a.num_blocks)) page = 0;
      size_t off = (((size_t)page * a.num_kv_heads + kvh) * a.block_size + (kp % a.block_size)) * HD + c * 8;
      cp_async16(sK + buf * PF_BN * HD + swz(r, c), a.k_cache + off, ok);
      cp_async16(sV + buf * PF_BN * HD + swz(r, c), a.v_cache + off, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[8][4];
  const int g = lane >> 2, tq = lane & 3;
  const int row0 = warp * 16;  // first row of this warp in the tile

  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) load_kv(kb + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        int r = row0 + (lane & 15), c = ks * 2 + (lane >> 4);
        ldsm_x4(qf[ks], sQ + swz(r, c));
      }
    }
    const __nv_bfloat16* k_t = sK + buf * PF_BN * HD;
    const __nv_bfloat16* v_t = sV + buf * PF_BN * HD;
    // S = Q K^T  (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t b[4];
        int key = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        int c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(b, k_t + swz(key, c));
        mma_bf16(s[2 * jp], qf[ks], b[0], b[1]);
        mma_bf16(s[2 * jp + 1], qf[ks], b[2], b[3]);
      }
    }
    // Mask + online softmax (rows g and g+8 of this warp).
    const bool need_mask = (kb + 1) * PF_BN > pos0 + qt0 + row0 + 1 || (kb + 1) * PF_BN > kv_end;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * a.scale_log2;
        if (need_mask) {
          int qrow = qt0 + row0 + g + ((e >> 1) << 3);
          int kpos = kb * PF_BN + j * 8 + 2 * tq + (e & 1);
          if (kpos > pos0 + qrow || kpos >= kv_end) v = -INFINITY;
        }
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      float m_new = fmaxf(m_r[h], mx[h]);
      corr[h] = (m_new == -INFINITY) ? 1.f : exp2f(m_r[h] - m_new);
      m_r[h] = m_new;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float mm = m_r[e >> 1];
        float p = (mm == -INFINITY) ? 0.f : exp2f(s[j][e] - mm);
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
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b[4];
        int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        int c = dp * 2 + (lane >> 4);
        ldsm_x4_t(b, v_t + swz(key, c));
        mma_bf16(o[2 * dp], pa, b[0], b[1]);
        mma_bf16(o[2 * dp + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  // Normalise and store.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int qi = qt0 + row0 + g + h * 8;
    if (qi >= q_len) continue;
    const float inv = l_r[h] > 0.f ? 1.f / l_r[h] : 0.f;
    __nv_bfloat16* dst = a.out + (size_t)(q_begin + qi) * a.out_stride + head * HD;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<uint32_t*>(dst + j * 8 + 2 * tq) = pack_bf16(o[j][2 * h] * inv, o[j][2 * h + 1] * inv);
    }
  }
}

// ------------------------------------------------------------------ decode

constexpr int DC_KEYS = 64;       // keys per chunk (16 per warp)
constexpr int DC_THREADS = 128;   // 4 warps
constexpr int DC_MAX_GROUP = 16;  // query heads per KV head: the rows of the m16 tile
constexpr int DC_STAGES = 3;      // cp.async ring depth
constexpr int DC_SMEM = (16 * HD + DC_STAGES * 2 * DC_KEYS * HD) * 2;  // 100 KB: two CTAs per SM

struct DecodeArgs {
  const __nv_bfloat16* q;  // [B, ...] row stride q_stride
  int q_stride;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  const int* block_tables;
  int max_blocks;
  const int* ctx_lens;     // [B]
  float* part_o;           // [B, Hq, splits, 128]
  float* part_ml;          // [B, Hq, splits, 2]
  __nv_bfloat16* out;      // [B, Hq*128] row stride out_stride
  int out_stride;
  int num_heads, num_kv_heads, group, block_size, splits, keys_per_split;
  int num_blocks;            // pages in the cache (bounds-check build); INT_MAX when unknown
  float scale_log2;
};

// One CTA = (sequence, KV head, KV split). The GQA group's G query heads are
// the rows of one 16 x 128 tensor-core tile (rows >= G are zero), so every
// K/V byte is read once for the whole group. The split's keys stream through a
// 3-stage cp.async ring of 64-key chunks; warp w scores keys [16w, 16w+16) of
// each chunk (QK^T and PV on m16n8k16), keeping its own online-softmax state;
// the four warps merge at the end. With one split the result is normalised
// and stored directly; otherwise (max, sum, out) partials go to the workspace
// for decode_combine_kernel.
__global__ void __launch_bounds__(DC_THREADS) paged_decode_kernel(DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t dc_smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(dc_smem);  // [16][128]
  __nv_bfloat16* sK = sQ + 16 * HD;                                 // [STAGES][64][128]
  __nv_bfloat16* sV = sK + DC_STAGES * DC_KEYS * HD;                // [STAGES][64][128]

  const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = a.group;
  const int ctx = a.ctx_lens[b];
  // keys_per_split 0: each sequence splits its own context evenly (64-key
  // granularity), so a launch whose arguments are fixed (a CUDA graph) works
  // for any context length.
  const int kps = a.keys_per_split > 0 ? a.keys_per_split
                                       : ((ctx + a.splits - 1) / a.splits + DC_KEYS - 1) / DC_KEYS * DC_KEYS;
  const int k_begin = split * kps;
  const int k_end = min(ctx, k_begin + kps);
  const int n_chunks = k_end > k_begin ? (k_end - k_begin + DC_KEYS - 1) / DC_KEYS : 0;
  const int* btab = a.block_tables + (size_t)b * a.max_blocks;

  for (int i = tid; i < 16 * 16; i += DC_THREADS) {
    const int r = i / 16, c = i % 16;
    const bool ok = r < G;
    const __nv_bfloat16* src = a.q + (size_t)b * a.q_stride + (size_t)(kvh * G + (ok ? r : 0)) * HD + c * 8;
    cp_async16(sQ + swz(r, c), src, ok);
  }
  auto load_chunk = [&](int ci, int buf) {
    for (int i = tid; i < DC_KEYS * 16; i += DC_THREADS) {
      const int r = i / 16, c = i % 16;
      const int kpos = k_begin + ci * DC_KEYS + r;
      const bool ok = kpos < k_end;
      const int kp = ok ? kpos : k_begin;
      int page = btab[kp / a.block_size];
      if (!DSV_IN_BOUNDS(page, a.num_blocks)) page = 0;
      const size_t off =
          (((size_t)page * a.num_kv_heads + kvh) * a.block_size + (kp % a.block_size)) * HD + c * 8;
      cp_async16(sK + buf * DC_KEYS * HD + swz(r, c), a.k_cache + off, ok);
      cp_async16(sV + buf * DC_KEYS * HD + swz(r, c), a.v_cache + off, ok);
    }
  };
#pragma unroll
  for (int st = 0; st < DC_STAGES - 1; ++st) {
    if (st < n_chunks) load_chunk(st, st);
    cp_async_commit();  // group st (the first also carries Q)
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[8][4];
  const int g = lane >> 2, tq = lane & 3;
  const int kw = warp * 16;  // this warp's keys within a chunk

  for (int ci = 0; ci < n_chunks; ++ci) {
    const int nxt = ci + DC_STAGES - 1;
    if (nxt < n_chunks) load_chunk(nxt, nxt % DC_STAGES);
    cp_async_commit();
    cp_async_wait<DC_STAGES - 1>();
    __syncthreads();
    if (ci == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) ldsm_x4(qf[ks], sQ + swz(lane & 15, ks * 2 + (lane >> 4)));
    }
    const int buf = ci % DC_STAGES;
    const __nv_bfloat16* k_t = sK + buf * DC_KEYS * HD;
    const __nv_bfloat16* v_t = sV + buf * DC_KEYS * HD;
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t bb[4];
      ldsm_x4(bb, k_t + swz(kw + (lane & 7) + ((lane >> 4) << 3), ks * 2 + ((lane >> 3) & 1)));
      mma_bf16(s[0], qf[ks], bb[0], bb[1]);
      mma_bf16(s[1], qf[ks], bb[2], bb[3]);
    }
    const int key0 = k_begin + ci * DC_KEYS + kw;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * a.scale_log2;
        if (key0 + j * 8 + 2 * tq + (e & 1) >= k_end) v = -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
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
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        const float pv = (mm == -INFINITY) ? 0.f : exp2f(s[j][e] - mm);
        s[j][e] = pv;
        rs[e >> 1] += pv;
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
    uint32_t pa[4];
    pa[0] = pack_bf16(s[0][0], s[0][1]);
    pa[1] = pack_bf16(s[0][2], s[0][3]);
    pa[2] = pack_bf16(s[1][0], s[1][1]);
    pa[3] = pack_bf16(s[1][2], s[1][3]);
#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {
      uint32_t bb[4];
      ldsm_x4_t(bb, v_t + swz(kw + (lane & 7) + (((lane >> 3) & 1) << 3), dp * 2 + (lane >> 4)));
      mma_bf16(o[2 * dp], pa, bb[0], bb[1]);
      mma_bf16(o[2 * dp + 1], pa, bb[2], bb[3]);
    }
    __syncthreads();  // the next prefetch overwrites this buffer
  }
  cp_async_wait<0>();
  __syncthreads();
  // Merge the four warps' (max, sum, out) in shared memory (the K ring is free now).
  float* red_m = reinterpret_cast<float*>(sK);  // [4][16]
  float* red_l = red_m + 4 * 16;                // [4][16]
  float* red_o = red_l + 4 * 16;                // [4][16][128]
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = g + h * 8;
    if (tq == 0) {
      red_m[warp * 16 + row] = m_r[h];
      red_l[warp * 16 + row] = l_r[h];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      red_o[(warp * 16 + row) * HD + j * 8 + 2 * tq] = o[j][2 * h];
      red_o[(warp * 16 + row) * HD + j * 8 + 2 * tq + 1] = o[j][2 * h + 1];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += DC_THREADS) {
    const int r = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red_m[w * 16 + r]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float mw = red_m[w * 16 + r];
        if (mw == -INFINITY) continue;
        const float sc = exp2f(mw - M);
        L += red_l[w * 16 + r] * sc;
        O += red_o[(w * 16 + r) * HD + d] * sc;
      }
    }
    const int h = kvh * G + r;
    if (a.splits == 1) {
      a.out[(size_t)b * a.out_stride + h * HD + d] = f2bf(L > 0.f ? O / L : 0.f);
    } else {
      const size_t idx = ((size_t)b * a.num_heads + h) * a.splits + split;
      a.part_o[idx * HD + d] = O;
      if (d == 0) {
        a.part_ml[idx * 2 + 0] = M;
        a.part_ml[idx * 2 + 1] = L;
      }
    }
  }
}

__global__ void decode_combine_kernel(DecodeArgs a) {
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  size_t base = ((size_t)b * a.num_heads + h) * a.splits;
  float m = -INFINITY;
  for (int s = 0; s < a.splits; ++s) m = fmaxf(m, a.part_ml[(base + s) * 2]);
  float l = 0.f, o = 0.f;
  for (int s = 0; s < a.splits; ++s) {
    float ms = a.part_ml[(base + s) * 2];
    if (ms == -INFINITY) continue;
    float w = exp2f(ms - m);
    l += a.part_ml[(base + s) * 2 + 1] * w;
    o += a.part_o[(base + s) * HD + d] * w;
  }
  a.out[(size_t)b * a.out_stride + h * HD + d] = f2bf(l > 0.f ? o / l : 0.f);
}

}  // namespace dsv

// ---------------------------------------------------------------- bindings

void dsv_paged_prefill(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                       torch::Tensor cu_q, torch::Tensor ctx_lens, torch::Tensor tile_info, torch::Tensor out,
                       int64_t num_heads, double scale, int64_t tile_rows) {
  using namespace dsv;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16, "prefill: bf16");
  TORCH_CHECK(tile_rows > 0 && tile_rows % PF_BM == 0, "prefill: tile_rows must be a multiple of 64");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == HD, "prefill: cache [blocks, Hkv, BS, 128]");
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1, "prefill: contiguous rows");
  const int num_tiles = (int)tile_info.size(0);
  if (num_tiles == 0) return;
  c10::cuda::CUDAGuard guard(q.device());
  PrefillArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_stride = (int)q.stride(0);
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.max_blocks = (int)block_tables.size(1);
  a.cu_q = cu_q.data_ptr<int>();
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.tile_info = tile_info.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_stride = (int)out.stride(0);
  a.num_kv_heads = (int)k_cache.size(1);
  a.block_size = (int)k_cache.size(2);
  a.num_blocks = (int)k_cache.size(0);
  a.group = (int)(num_heads / a.num_kv_heads);
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  const int smem = (PF_BM * HD + 4 * PF_BN * HD) * 2;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(paged_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr = true;
  }
  dim3 grid(num_tiles, (unsigned)num_heads, (unsigned)(tile_rows / PF_BM));
  paged_prefill_kernel<<<grid, PF_THREADS, smem, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// part_o / part_ml: caller-provided workspaces of at least B*Hq*splits*128 and
// B*Hq*splits*2 floats.
void dsv_paged_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                      torch::Tensor ctx_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml,
                      int64_t num_heads, double scale, int64_t splits, int64_t keys_per_split) {
  using namespace dsv;
  const int B = (int)ctx_lens.size(0);
  if (B == 0) return;
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == HD, "decode: cache [blocks, Hkv, BS, 128]");
  TORCH_CHECK(keys_per_split % DC_KEYS == 0, "decode: keys_per_split must be a multiple of 64");
  const int Hkv = (int)k_cache.size(1);
  const int G = (int)(num_heads / Hkv);
  TORCH_CHECK(G >= 1 && G <= DC_MAX_GROUP, "decode: GQA group must be 1..16");
  TORCH_CHECK(part_o.numel() >= (int64_t)B * num_heads * splits * HD && part_ml.numel() >= (int64_t)B * num_heads * splits * 2,
              "decode: workspace too small");
  c10::cuda::CUDAGuard guard(q.device());
  DecodeArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.q_stride = (int)q.stride(0);
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.max_blocks = (int)block_tables.size(1);
  a.ctx_lens = ctx_lens.data_ptr<int>();
  a.part_o = part_o.data_ptr<float>();
  a.part_ml = part_ml.data_ptr<float>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_stride = (int)out.stride(0);
  a.num_heads = (int)num_heads;
  a.num_kv_heads = Hkv;
  a.group = G;
  a.block_size = (int)k_cache.size(2);
  a.num_blocks = (int)k_cache.size(0);
  a.splits = (int)splits;
  a.keys_per_split = (int)keys_per_split;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  static bool dattr = false;
  if (!dattr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(paged_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DC_SMEM));
    dattr = true;
  }
  paged_decode_kernel<<<dim3(B, Hkv, (unsigned)splits), DC_THREADS, DC_SMEM, s>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (splits > 1) {
    decode_combine_kernel<<<dim3(B, (unsigned)num_heads), HD, 0, s>>>(a);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// ---------------------------------------------------------------- allocation-free entry point
// See noalloc.h for who calls this and the contract (no counterpart in the
// reference project).
#include "noalloc.h"

namespace dsv {
// The scratch of dsv_paged_decode_noalloc: split partials (128 floats of output
// and 2 of max/sum per (sequence, head, split)). Host code must not use this
// name as an address: it looks the device address up with cudaGetSymbolAddress.
static __device__ __align__(256) float g_noalloc_scratch[DSV_NOALLOC_SCRATCH_FLOATS];
constexpr int kMaxDevices = 64;
// Per-device cache of the array's device address. Written without a lock:
// threads making their first call on one device at the same time each look
// the address up and store the same value.
static float* g_noalloc_ptr[kMaxDevices] = {nullptr};
}  // namespace dsv

extern "C" int dsv_paged_decode_noalloc(const void* q, int q_stride, const void* k_cache, const void* v_cache,
                                        int num_kv_heads, int block_size, const int* block_tables, int max_blocks,
                                        const int* ctx_lens, int batch, void* out, int out_stride, int num_heads,
                                        float scale, int splits, int keys_per_split, cudaStream_t stream) {
  using namespace dsv;
  if (batch == 0) return DSV_NOALLOC_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !ctx_lens || !out || batch < 0 || num_kv_heads <= 0 ||
      num_heads % num_kv_heads != 0 || splits < 1 || keys_per_split < 0 || keys_per_split % DC_KEYS != 0 ||
      block_size <= 0)
    return DSV_NOALLOC_EINVAL;
  const int G = num_heads / num_kv_heads;
  if (G < 1 || G > DC_MAX_GROUP) return DSV_NOALLOC_EINVAL;
  const long long parts = (long long)batch * num_heads * splits;
  if (parts * (HD + 2) > DSV_NOALLOC_SCRATCH_FLOATS) return DSV_NOALLOC_ETOOBIG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSV_NOALLOC_ECUDA;
  if (g_noalloc_ptr[dev] == nullptr) {
    // One-time set-up on this device (the device is current here).
    float* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return DSV_NOALLOC_ECUDA;
    g_noalloc_ptr[dev] = p;
  }
  float* scratch = g_noalloc_ptr[dev];
  DecodeArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.ctx_lens = ctx_lens;
  a.part_o = scratch;
  a.part_ml = scratch + parts * HD;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.out_stride = out_stride;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = G;
  a.block_size = block_size;
  a.num_blocks = 0x7fffffff;   // the C entry point is not told the cache's page count
  a.splits = splits;
  a.keys_per_split = keys_per_split;
  a.scale_log2 = scale * 1.4426950408889634f;
  // An error already pending on this thread belongs to an earlier, unrelated
  // call: leave it in place for its owner and launch nothing.
  if (cudaPeekAtLastError() != cudaSuccess) return DSV_NOALLOC_ECUDA;
  if (cudaFuncSetAttribute(paged_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DC_SMEM) != cudaSuccess)
    return DSV_NOALLOC_ECUDA;
  paged_decode_kernel<<<dim3(batch, num_kv_heads, (unsigned)splits), DC_THREADS, DC_SMEM, stream>>>(a);
  if (cudaPeekAtLastError() != cudaSuccess) {
    (void)cudaGetLastError();  // this launch's own error: consumed and reported
    return DSV_NOALLOC_ECUDA;
  }
  if (splits > 1) {
    decode_combine_kernel<<<dim3(batch, (unsigned)num_heads), HD, 0, stream>>>(a);
    if (cudaPeekAtLastError() != cudaSuccess) {
      (void)cudaGetLastError();
      return DSV_NOALLOC_ECUDA;
    }
  }
  return DSV_NOALLOC_OK;
}
