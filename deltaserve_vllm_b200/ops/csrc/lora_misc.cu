// Segmented multi-LoRA shrink, embedding, fused cross-entropy, AdamW with
// per-layer clipping, LoRA publish, and sampling kernels.
//
// LoRA layout used by the engine (one group = projections sharing an input,
// e.g. q/k/v share the attention input):
//   A     [slots, P*R, K]  bf16   shrink weights, rank-padded to R
//   Z     [T, slots*SEG]   bf16   shrink output; row t is non-zero only in the
//                                 SEG columns of its own slot (SEG = P*R rounded
//                                 up to 64), so the expand can run as extra
//                                 K blocks of the base GEMM (gemm_tc.cu)
//   B2    [N, slots*SEG]   bf16   expand weights (scale folded in), row n only
//                                 uses the R columns of its own projection.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace dsv {

constexpr int SHR_ROWS = 16;
constexpr int SHR_KC = 1024;  // K chunk staged in smem
constexpr int SHR_THREADS = 256;
constexpr int SHR_OUT = SHR_THREADS / 32;  // outputs per CTA (one per warp)
constexpr int SHR_MAXPR = 192;  // 3 projections x rank 64

// grid = (row tiles of 16, output groups of 8). A warp owns one output column
// o of the group: it keeps the A row chunk of the current slot in registers and
// dots it with each staged x row (rows are sorted by slot, so the A chunk is
// reloaded only at slot changes). Output groups run on different CTAs, so a
// decode step (one row tile) still spreads over P*R/8 CTAs. The y == 0 CTA
// also writes the zero columns of every row (other slots and padding).
__global__ void __launch_bounds__(SHR_THREADS) lora_shrink_kernel(const __nv_bfloat16* __restrict__ x, int sx,
                                                                  const __nv_bfloat16* __restrict__ A,
                                                                  const int* __restrict__ slot_ids, __nv_bfloat16* Z,
                                                                  int sz, int T, int K, int PR, int SEG, int slots) {
  __shared__ __align__(16) __nv_bfloat16 xs[SHR_ROWS * SHR_KC];
  __shared__ int rslot[SHR_ROWS];
  const int r0 = blockIdx.x * SHR_ROWS;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int o = blockIdx.y * SHR_OUT + warp;
  if (threadIdx.x < SHR_ROWS) {
    const int r = r0 + threadIdx.x;
    rslot[threadIdx.x] = (r < T) ? slot_ids[r] : -1;
  }
  __syncthreads();
  float acc[SHR_ROWS];
#pragma unroll
  for (int r = 0; r < SHR_ROWS; ++r) acc[r] = 0.f;
  for (int k0 = 0; k0 < K; k0 += SHR_KC) {
    const int kc = min(SHR_KC, K - k0);
    for (int i = threadIdx.x; i < SHR_ROWS * (kc / 8); i += SHR_THREADS) {
      const int r = i / (kc / 8), c = (i % (kc / 8)) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r0 + r < T && rslot[r] >= 0) v = *reinterpret_cast<const uint4*>(x + (size_t)(r0 + r) * sx + k0 + c);
      *reinterpret_cast<uint4*>(xs + r * SHR_KC + c) = v;
    }
    __syncthreads();
    if (o < PR) {
      int cur = -2;
      float av[SHR_KC / 32];
#pragma unroll
      for (int r = 0; r < SHR_ROWS; ++r) {
        const int s = rslot[r];
        if (s < 0) continue;
        if (s != cur) {
          const __nv_bfloat16* ar = A + ((size_t)s * PR + o) * K + k0;
#pragma unroll
          for (int j = 0; j < SHR_KC / 32; j += 8) {
            const int c = lane * 8 + j * 32;
            if (c < kc) {
              uint4 raw = *reinterpret_cast<const uint4*>(ar + c);
              const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float2 f = __bfloat1622float2(h[e]);
                av[j + 2 * e] = f.x;
                av[j + 2 * e + 1] = f.y;
              }
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) av[j + e] = 0.f;
            }
          }
          cur = s;
        }
        float d = 0.f;
#pragma unroll
        for (int j = 0; j < SHR_KC / 32; j += 8) {
          const int c = lane * 8 + j * 32;
          if (c < kc) {
            uint4 raw = *reinterpret_cast<const uint4*>(xs + r * SHR_KC + c);
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 f = __bfloat1622float2(h[e]);
              d += f.x * av[j + 2 * e] + f.y * av[j + 2 * e + 1];
            }
          }
        }
        acc[r] += d;
      }
    }
    __syncthreads();
  }
  if (o < PR) {
#pragma unroll
    for (int r = 0; r < SHR_ROWS; ++r) {
      const int s = rslot[r];
      if (s < 0) continue;
      const float v = warp_sum(acc[r]);
      if (lane == 0) Z[(size_t)(r0 + r) * sz + s * SEG + o] = f2bf(v);
    }
  }
  if (blockIdx.y == 0) {
    const int W = slots * SEG;
    for (int i = threadIdx.x; i < SHR_ROWS * W; i += SHR_THREADS) {
      const int r = i / W, c = i % W;
      if (r0 + r >= T) continue;
      const int s = rslot[r];
      if (s >= 0 && c >= s * SEG && c < s * SEG + PR) continue;
      Z[(size_t)(r0 + r) * sz + c] = f2bf(0.f);
    }
  }
}

// Small-batch shrink (decode): one CTA per (row, block of 8 output columns).
// Its 8 warps split the K range; each warp loads its slice of the x row once
// per 256 elements and the 8 A rows of the block alongside it (9 independent
// 16-byte loads in flight per lane), keeping 8 running dot products; the 8
// warps' partials meet in shared memory and warp 0 writes the 8 outputs. The
// CTA of block 0 also writes the row's zero columns. (One warp per output with
// the whole K serial was latency-bound: ~16 us per call at decode sizes.)
constexpr int SHV_OUT = 8;
__global__ void __launch_bounds__(256) lora_shrink_gemv_kernel(const __nv_bfloat16* __restrict__ x, int sx,
                                                               const __nv_bfloat16* __restrict__ A,
                                                               const int* __restrict__ slot_ids, __nv_bfloat16* Z,
                                                               int sz, int T, int K, int PR, int SEG, int slots) {
  __shared__ float part[8][SHV_OUT];
  griddep_launch_dependents();   // the GEMM that reads Z may start its base K blocks now
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row = blockIdx.x;
  const int o0 = blockIdx.y * SHV_OUT;
  int s = slot_ids[row];
  if (s >= 0 && !DSV_IN_BOUNDS(s, slots)) s = -1;    // bounds-check build: an unknown slot reads nothing
  if (blockIdx.y == 0) {
    const int W = slots * SEG;
    for (int c = threadIdx.x; c < W; c += blockDim.x) {
      if (s >= 0 && c >= s * SEG && c < s * SEG + PR) continue;
      Z[(size_t)row * sz + c] = f2bf(0.f);
    }
  }
  if (s < 0) return;
  // K range of this warp: whole 256-element steps, split as evenly as possible.
  const int steps = (K + 255) / 256;
  const int per = (steps + 7) / 8;
  const int k_lo = warp * per * 256, k_hi = min(K, (warp + 1) * per * 256);
  const __nv_bfloat16* xr = x + (size_t)row * sx;
  const __nv_bfloat16* ab = A + ((size_t)s * PR + o0) * K;
  const int n_out = min(SHV_OUT, PR - o0);
  float d[SHV_OUT];
#pragma unroll
  for (int j = 0; j < SHV_OUT; ++j) d[j] = 0.f;
  for (int k = k_lo + lane * 8; k < k_hi; k += 256) {
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + k);
    uint4 av[SHV_OUT];
#pragma unroll
    for (int j = 0; j < SHV_OUT; ++j)
      av[j] = j < n_out ? *reinterpret_cast<const uint4*>(ab + (size_t)j * K + k) : make_uint4(0, 0, 0, 0);
    const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
    for (int j = 0; j < SHV_OUT; ++j) {
      const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&av[j]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 xf = __bfloat1622float2(xh[e]);
        const float2 af = __bfloat1622float2(ah[e]);
        d[j] += xf.x * af.x + xf.y * af.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < SHV_OUT; ++j) {
    const float v = warp_sum(d[j]);
    if (lane == 0) part[warp][j] = v;
  }
  __syncthreads();
  if (warp == 0 && lane < n_out) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) v += part[w][lane];
    Z[(size_t)row * sz + s * SEG + o0 + lane] = f2bf(v);
  }
}

// Vocab-parallel embedding: ids outside [v0, v0 + Vl) give zero rows (the TP
// all-reduce sums the shards).
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* out, int D, int64_t v0, int64_t Vl) {
  const int t = blockIdx.x;
  const int64_t id = ids[t] - v0;
  const bool ok = id >= 0 && id < Vl;
  for (int i = threadIdx.x * 8; i < D; i += blockDim.x * 8) {
    uint4 v = ok ? *reinterpret_cast<const uint4*>(table + id * D + i) : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(out + (size_t)t * D + i) = v;
  }
}

// Vocab-parallel embedding without a collective: every rank's shard of the
// table sits in peer-mapped memory (CUDA IPC, plain P2P mappings); each token's
// row is read straight from the shard that holds it (`tables[owner]`, a P2P
// load over NVLink when the owner is another GPU), so every rank gets the full
// rows and no all-reduce of the summed partial rows is needed.
__global__ void embedding_peer_kernel(const int64_t* __restrict__ ids, const int64_t* __restrict__ tables, int world,
                                      int64_t v_local, int64_t vocab, __nv_bfloat16* out, int D) {
  const int t = blockIdx.x;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  const int owner = ok ? (int)min((int64_t)(world - 1), id / v_local) : 0;
  const __nv_bfloat16* table = reinterpret_cast<const __nv_bfloat16*>(tables[owner]);
  const int64_t row = ok ? id - (int64_t)owner * v_local : 0;
  for (int i = threadIdx.x * 8; i < D; i += blockDim.x * 8) {
    uint4 v = ok ? *reinterpret_cast<const uint4*>(table + row * D + i) : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(out + (size_t)t * D + i) = v;
  }
}

// Cross-entropy over fp32 logits rows, forward and backward in one pass pair:
// loss[r] = lse - logit[target]; grad (bf16) = (softmax - onehot) * gscale.
// target < 0 rows produce zero loss and zero gradient.
__global__ void ce_fwd_bwd_kernel(const float* __restrict__ logits, int64_t sl, const int64_t* __restrict__ targets,
                                  float* loss, __nv_bfloat16* grad, int64_t sg, int V, float gscale) {
  __shared__ float red[32];
  const int r = blockIdx.x;
  const float* lr = logits + (size_t)r * sl;
  const int64_t tgt = targets[r];
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) mx = fmaxf(mx, lr[i]);
  mx = warp_max(mx);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
    t = warp_max(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float se = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) se += __expf(lr[i] - mx);
  se = warp_sum(se);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = se;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float lse = mx + __logf(red[0]);
  if (threadIdx.x == 0) loss[r] = (tgt >= 0) ? (lse - lr[tgt]) : 0.f;
  if (grad != nullptr) {
    __nv_bfloat16* gr = grad + (size_t)r * sg;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      float p = (tgt >= 0) ? __expf(lr[i] - lse) - (i == tgt ? 1.f : 0.f) : 0.f;
      gr[i] = f2bf(p * gscale);
    }
  }
}

// Sum of squares per segment of equal length (one segment per layer).
__global__ void seg_sumsq_kernel(const float* __restrict__ g, int64_t seg_len, float* out) {
  __shared__ float red[32];
  const int s = blockIdx.y;
  const float* p = g + (size_t)s * seg_len;
  float acc = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < seg_len; i += (int64_t)gridDim.x * blockDim.x)
    acc += p[i] * p[i];
  acc = warp_sum(acc);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) atomicAdd(&out[s], t);
  }
}

// AdamW over one flat fp32 buffer; the gradient of segment s is scaled by
// coef[s] = min(1, max_norm / (||g_s|| + 1e-6)) (per-layer clipping) and by
// grad_scale (loss scaling / TP averaging).
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, int64_t n, int64_t seg_len, const float* __restrict__ seg_sumsq,
                             float max_norm, float grad_scale, float lr, float b1, float b2, float eps, float wd,
                             float bc1, float bc2) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float coef = grad_scale;
    if (seg_sumsq != nullptr && max_norm > 0.f) {
      const float nrm = sqrtf(seg_sumsq[i / seg_len]) * grad_scale;
      coef *= fminf(1.f, max_norm / (nrm + 1e-6f));
    }
    const float gi = g[i] * coef;
    float pi = p[i];
    pi -= lr * wd * pi;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi / bc2) + eps;
    p[i] = pi - lr * (mi / bc1) / denom;
  }
}

// Publish one LoRA group of one layer into a served slot:
//   A_dst[r, k]               = bf16(A_src[r, k])
//   B2_dst[n, col0 + p(n)*R + j] = bf16(clamp(Bt_src[j, n] * scale))
// p(n): rows [0, b1) -> 0, [b1, b2) -> 1, [b2, N) -> 2, or (n / 64) % 2 when
// interleave64 (gate/up).
__global__ void lora_publish_kernel(const float* __restrict__ A_src, __nv_bfloat16* A_dst, int64_t a_numel,
                                    const float* __restrict__ Bt_src, __nv_bfloat16* B2_dst, int64_t ldb2, int col0,
                                    int N, int R, int b1, int b2, int interleave64, float scale) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < a_numel; i += stride) A_dst[i] = f2bf(A_src[i]);
  for (int64_t i = tid; i < (int64_t)N * R; i += stride) {
    const int n = (int)(i / R), j = (int)(i % R);
    const int p = interleave64 ? ((n >> 6) & 1) : (n < b1 ? 0 : (n < b2 ? 1 : 2));
    float v = Bt_src[(int64_t)j * N + n] * scale;
    v = fminf(fmaxf(v, -65504.f), 65504.f);
    B2_dst[(int64_t)n * ldb2 + col0 + p * R + j] = f2bf(v);
  }
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  // SplitMix64 finaliser (Steele, Lea, Flood 2014).
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Block-wide sum (1024 threads) through a 32-entry shared scratch; every
// thread gets the total.
template <typename T>
__device__ __forceinline__ T block_sum_1024(T v, T* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  T t = 0;
  for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += red[w];
  return t;
}

// One CTA (1024 threads) per row: greedy (temperature <= 0) or Gumbel-max
// sampling at the row's temperature, optionally restricted to the top-k
// tokens and then to the smallest top set whose renormalised probability
// reaches top-p (thresholds found by bisection on the scaled logits, one
// pass over the row per step). Optionally the chosen token's log-probability
// under the raw logits (log_softmax) is written to logprob_out.
__global__ void sample_kernel(const float* __restrict__ logits, int64_t sl, const float* __restrict__ temps,
                              const int64_t* __restrict__ seeds, int64_t* out, int V,
                              const int* __restrict__ topk, const float* __restrict__ topp,
                              float* __restrict__ logprob_out) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  __shared__ float redf[32];
  __shared__ int redi[32];
  const int r = blockIdx.x;
  const float* lr = logits + (size_t)r * sl;
  const float t = temps[r];
  const uint64_t seed = (uint64_t)seeds[r];
  const int k = topk != nullptr ? topk[r] : 0;
  const float p = topp != nullptr ? topp[r] : 1.f;
  const float inv_t = t > 0.f ? 1.f / t : 1.f;
  // Row max / min of the (scaled) logits: the bisection range and the softmax shift.
  float zmax, zmin;
  {
    float m = -INFINITY, n = INFINITY;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float z = lr[i] * inv_t;
      m = fmaxf(m, z);
      // Masked tokens (-inf, e.g. EOS under min_tokens) stay out of the
      // bisection range: a -inf lower bound would never move.
      if (z > -INFINITY) n = fminf(n, z);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      n = fminf(n, __shfl_xor_sync(0xffffffffu, n, o));
    }
    __syncthreads();
    if (threadIdx.x % 32 == 0) {
      bv[threadIdx.x / 32] = m;
      redf[threadIdx.x / 32] = n;
    }
    __syncthreads();
    m = -INFINITY;
    n = INFINITY;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) {
      m = fmaxf(m, bv[w]);
      n = fminf(n, redf[w]);
    }
    zmax = m;
    zmin = fminf(n, m);  // every token masked: an empty range at zmax
  }
  float thr = -INFINITY;  // keep tokens whose scaled logit >= thr
  if (t > 0.f && ((k > 0 && k < V) || p < 1.f)) {
    if (k > 0 && k < V) {
      float lo = zmin, hi = zmax;  // invariant: count(z >= lo) >= k
      for (int it = 0; it < 40; ++it) {
        const float mid = 0.5f * (lo + hi);
        int c = 0;
        for (int i = threadIdx.x; i < V; i += blockDim.x) c += (lr[i] * inv_t >= mid);
        c = block_sum_1024(c, redi);
        if (c >= k) lo = mid;
        else hi = mid;
      }
      thr = lo;
    }
    if (p < 1.f) {
      float zsum = 0.f;
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float z = lr[i] * inv_t;
        if (z >= thr) zsum += __expf(z - zmax);
      }
      zsum = block_sum_1024(zsum, redf);
      float lo = fmaxf(thr, zmin), hi = zmax;  // invariant: mass(z >= lo) >= p
      for (int it = 0; it < 40; ++it) {
        const float mid = 0.5f * (lo + hi);
        float m = 0.f;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
          const float z = lr[i] * inv_t;
          if (z >= mid && z >= thr) m += __expf(z - zmax);
        }
        m = block_sum_1024(m, redf);
        if (m >= p * zsum) lo = mid;
        else hi = mid;
      }
      thr = fmaxf(thr, lo);
    }
  }
  float best = -INFINITY;
  int arg = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float v = lr[i];
    if (t > 0.f) {
      if (v * inv_t < thr) continue;
      const uint64_t h = mix64(seed * 0x100000001B3ull + (uint64_t)i);
      // 23 random bits: (k + 0.5) / 2^23 is exact in fp32 and strictly inside
      // (0, 1), so -log(-log(u)) is finite for every token.
      const float u = ((float)(h >> 41) + 0.5f) * (1.0f / 8388608.0f);
      v = v * inv_t - logf(-logf(u));
    }
    if (v > best) {
      best = v;
      arg = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, arg, o);
    if (ov > best || (ov == best && oi < arg)) {
      best = ov;
      arg = oi;
    }
  }
  __syncthreads();
  if (threadIdx.x % 32 == 0) {
    bv[threadIdx.x / 32] = best;
    bi[threadIdx.x / 32] = arg;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x / 32); ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < arg)) {
        best = bv[w];
        arg = bi[w];
      }
    out[r] = arg;
    bi[0] = arg;
  }
  if (logprob_out != nullptr) {
    __syncthreads();
    const int chosen = bi[0];
    float mraw = -INFINITY;
    for (int i = threadIdx.x; i < V; i += blockDim.x) mraw = fmaxf(mraw, lr[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mraw = fmaxf(mraw, __shfl_xor_sync(0xffffffffu, mraw, o));
    __syncthreads();
    if (threadIdx.x % 32 == 0) bv[threadIdx.x / 32] = mraw;
    __syncthreads();
    mraw = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) mraw = fmaxf(mraw, bv[w]);
    float se = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) se += __expf(lr[i] - mraw);
    se = block_sum_1024(se, redf);
    if (threadIdx.x == 0) logprob_out[r] = lr[chosen] - mraw - __logf(se);
  }
}

}  // namespace dsv

void dsv_lora_shrink_tc(torch::Tensor x, torch::Tensor A, torch::Tensor slot_ids, torch::Tensor Z, int64_t pr,
                        int64_t seg);

void dsv_lora_shrink(torch::Tensor x, torch::Tensor A, torch::Tensor slot_ids, torch::Tensor Z, int64_t seg) {
  using namespace dsv;
  const int T = (int)x.size(0);
  if (T == 0) return;
  const int K = (int)x.size(1);
  const int slots = (int)A.size(0), PR = (int)A.size(1);
  TORCH_CHECK(A.size(2) == K && K % 8 == 0 && PR <= SHR_MAXPR && PR <= seg, "lora_shrink: shapes");
  TORCH_CHECK(Z.size(1) == slots * seg && Z.size(0) >= T, "lora_shrink: Z shape");
  c10::cuda::CUDAGuard guard(x.device());
  if (T * PR <= 64 * 192 && x.stride(0) % 8 == 0 && (uintptr_t)x.data_ptr() % 16 == 0 && A.is_contiguous()) {
    const dim3 blocks((unsigned)T, (unsigned)((PR + SHV_OUT - 1) / SHV_OUT));
    lora_shrink_gemv_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)x.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(A.data_ptr()), slot_ids.data_ptr<int>(),
        reinterpret_cast<__nv_bfloat16*>(Z.data_ptr()), (int)Z.stride(0), T, K, PR, (int)seg, slots);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  if (T >= 256 && x.stride(0) % 8 == 0 && A.is_contiguous() && (uintptr_t)x.data_ptr() % 16 == 0) {
    // Large batches: a tcgen05 GEMM over the stacked factors (x read once per
    // 64-column tile of slots * P * R, from L2 after the first).
    dsv_lora_shrink_tc(x, A.view({slots * PR, K}), slot_ids, Z, PR, seg);
    return;
  }
  dim3 grid((T + SHR_ROWS - 1) / SHR_ROWS, (PR + SHR_OUT - 1) / SHR_OUT);
  lora_shrink_kernel<<<grid, SHR_THREADS, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)x.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(A.data_ptr()), slot_ids.data_ptr<int>(),
      reinterpret_cast<__nv_bfloat16*>(Z.data_ptr()), (int)Z.stride(0), T, K, PR, (int)seg, slots);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_embedding_peer(torch::Tensor ids, torch::Tensor tables, int64_t v_local, int64_t vocab, torch::Tensor out) {
  using namespace dsv;
  const int T = (int)ids.size(0);
  if (T == 0) return;
  const int D = (int)out.size(1);
  TORCH_CHECK(tables.is_cuda() && tables.scalar_type() == at::kLong && tables.dim() == 1 && tables.numel() <= 8,
              "embedding_peer: tables must be an int64 CUDA tensor of <= 8 shard addresses");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && D % 8 == 0 && ids.scalar_type() == at::kLong,
              "embedding_peer: bf16 [T, D] output, int64 ids");
  c10::cuda::CUDAGuard guard(ids.device());
  embedding_peer_kernel<<<T, std::min(1024, std::max(32, D / 8)), 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), tables.data_ptr<int64_t>(), (int)tables.numel(), v_local, vocab,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, int64_t v0) {
  using namespace dsv;
  const int T = (int)ids.size(0);
  if (T == 0) return;
  const int D = (int)table.size(1);
  c10::cuda::CUDAGuard guard(ids.device());
  embedding_kernel<<<T, std::min(1024, std::max(32, D / 8)), 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), D, v0, table.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_ce_fwd_bwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss,
                    c10::optional<torch::Tensor> grad, double gscale) {
  using namespace dsv;
  const int R = (int)logits.size(0);
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  dsv::ce_fwd_bwd_kernel<<<R, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.stride(0), targets.data_ptr<int64_t>(), loss.data_ptr<float>(),
      grad.has_value() ? reinterpret_cast<__nv_bfloat16*>(grad->data_ptr()) : nullptr,
      grad.has_value() ? grad->stride(0) : 0, (int)logits.size(1), (float)gscale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_seg_sumsq(torch::Tensor g, int64_t seg_len, torch::Tensor out) {
  const int segs = (int)out.numel();
  if (segs == 0) return;
  c10::cuda::CUDAGuard guard(g.device());
  out.zero_();
  dim3 grid(std::max<int64_t>(1, std::min<int64_t>(64, seg_len / 4096 + 1)), segs);
  dsv::seg_sumsq_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(g.data_ptr<float>(), seg_len,
                                                                           out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_adamw(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, int64_t seg_len,
               c10::optional<torch::Tensor> seg_sumsq, double max_norm, double grad_scale, double lr, double b1,
               double b2, double eps, double wd, int64_t step) {
  const int64_t n = p.numel();
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(p.device());
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2 = 1.f - (float)std::pow(b2, (double)step);
  const int blocks = (int)std::min<int64_t>(4096, (n + 255) / 256);
  dsv::adamw_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), n, seg_len,
      seg_sumsq.has_value() ? seg_sumsq->data_ptr<float>() : nullptr, (float)max_norm, (float)grad_scale, (float)lr,
      (float)b1, (float)b2, (float)eps, (float)wd, bc1, bc2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_lora_publish(torch::Tensor A_src, torch::Tensor A_dst, torch::Tensor Bt_src, torch::Tensor B2_dst,
                      int64_t col0, int64_t b1, int64_t b2, bool interleave64, double scale) {
  c10::cuda::CUDAGuard guard(A_src.device());
  const int R = (int)Bt_src.size(0), N = (int)Bt_src.size(1);
  const int64_t work = std::max<int64_t>(A_src.numel(), (int64_t)N * R);
  const int blocks = (int)std::min<int64_t>(2048, (work + 255) / 256);
  dsv::lora_publish_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      A_src.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(A_dst.data_ptr()), A_src.numel(),
      Bt_src.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(B2_dst.data_ptr()), B2_dst.stride(0), (int)col0, N,
      R, (int)b1, (int)b2, interleave64 ? 1 : 0, (float)scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_sample(torch::Tensor logits, torch::Tensor temps, torch::Tensor seeds, torch::Tensor out,
                c10::optional<torch::Tensor> topk, c10::optional<torch::Tensor> topp,
                c10::optional<torch::Tensor> logprobs) {
  const int R = (int)logits.size(0);
  if (R == 0) return;
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "sample: fp32 logits rows");
  if (topk.has_value())
    TORCH_CHECK(topk->scalar_type() == at::kInt && topk->numel() >= R, "sample: top_k must be int32 [R]");
  if (topp.has_value())
    TORCH_CHECK(topp->scalar_type() == at::kFloat && topp->numel() >= R, "sample: top_p must be fp32 [R]");
  if (logprobs.has_value())
    TORCH_CHECK(logprobs->scalar_type() == at::kFloat && logprobs->numel() >= R, "sample: logprobs fp32 [R]");
  c10::cuda::CUDAGuard guard(logits.device());
  dsv::sample_kernel<<<R, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.stride(0), temps.data_ptr<float>(), seeds.data_ptr<int64_t>(),
      out.data_ptr<int64_t>(), (int)logits.size(1), topk.has_value() ? topk->data_ptr<int>() : nullptr,
      topp.has_value() ? topp->data_ptr<float>() : nullptr, logprobs.has_value() ? logprobs->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
