// Normalisation, RoPE and KV-cache write kernels (bandwidth-bound, CUDA cores).
//
// * rms_norm / fused_add_rms_norm: one CTA per token row, fp32 statistics,
//   bf16 in/out. The fused variant updates the residual stream in place and can
//   copy a row range of the new residual into an activation-capture buffer
//   (the finetuning rows' layer input) in the same pass.
// * qk_norm_rope_cache: one warp per (token, head) of the fused qkv row: optional
//   per-head RMSNorm (Qwen3 q_norm/k_norm), NeoX rotate-half RoPE from an fp32
//   cos/sin table, q/k written back in place, k and v scattered into the paged
//   cache at slot_mapping[token].
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace dsv {

template <int VEC>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* p, float (&v)[VEC]) {
#pragma unroll
  for (int i = 0; i < VEC; i += 2) {
    float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p + i));
    v[i] = f.x;
    v[i + 1] = f.y;
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < blockDim.x / 32) ? red[threadIdx.x] : 0.f;
  if (w == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

// x: [T, D] (row stride sx); residual: [T, D] updated in place (if ADD);
// out: [T, D]; save rows [save_lo, save_hi) of the residual to save[save_dst + r - save_lo].
template <bool ADD>
__global__ void rms_norm_kernel(const __nv_bfloat16* __restrict__ x, int sx, __nv_bfloat16* residual, int sr,
                                const __nv_bfloat16* __restrict__ w, __nv_bfloat16* out, int so, int D, float eps,
                                __nv_bfloat16* save, int ssave, int save_lo, int save_hi, int save_dst) {
  extern __shared__ float buf[];  // D floats + 32
  float* red = buf + D;
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)row * sx;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < D; i += blockDim.x * 8) {
    float v[8];
    load_bf16<8>(xr + i, v);
    if (ADD) {
      float r[8];
      load_bf16<8>(residual + (size_t)row * sr + i, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += r[j];
      // The residual stream is kept in bf16: round before the statistics so
      // the normalised value matches what the next layer reads back.
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = bf2f(f2bf(v[j]));
      uint4 pk;
      uint32_t* p = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        p[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(residual + (size_t)row * sr + i) = pk;
      if (save != nullptr && row >= save_lo && row < save_hi)
        *reinterpret_cast<uint4*>(save + (size_t)(row - save_lo + save_dst) * ssave + i) = pk;
    } else if (save != nullptr && row >= save_lo && row < save_hi) {
      *reinterpret_cast<uint4*>(save + (size_t)(row - save_lo + save_dst) * ssave + i) =
          *reinterpret_cast<const uint4*>(xr + i);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      buf[i + j] = v[j];
      ss += v[j] * v[j];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / D + eps);
  for (int i = threadIdx.x * 8; i < D; i += blockDim.x * 8) {
    float wv[8];
    load_bf16<8>(w + i, wv);
    uint4 pk;
    uint32_t* p = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(buf[i + 2 * j] * inv * wv[2 * j], buf[i + 2 * j + 1] * inv * wv[2 * j + 1]);
      p[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + (size_t)row * so + i) = pk;
  }
}

// One warp per (token, head). Lane l owns dims {2l, 2l+1} and {64+2l, 65+2l}:
// the rotate-half partners sit in the same lane.
__global__ void qk_norm_rope_cache_kernel(__nv_bfloat16* qkv, int sq, const int64_t* __restrict__ positions,
                                          const float* __restrict__ cos_sin, const __nv_bfloat16* __restrict__ qn_w,
                                          const __nv_bfloat16* __restrict__ kn_w, float eps, int Hq, int Hkv,
                                          __nv_bfloat16* k_cache, __nv_bfloat16* v_cache,
                                          const int64_t* __restrict__ slot_mapping, int block_size, int T,
                                          int64_t cache_slots) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  const int H = Hq + 2 * Hkv;
  if (gw >= T * H) return;
  const int tok = gw / H, h = gw % H;
  __nv_bfloat16* row = qkv + (size_t)tok * sq + h * 128;
  int64_t slot = slot_mapping != nullptr ? slot_mapping[tok] : -1;
  if (slot >= 0 && !DSV_IN_BOUNDS(slot, cache_slots)) slot = -1;   // bounds-check build: skip the write
  if (h >= Hq + Hkv) {
    // v: copy into the cache only.
    if (slot >= 0) {
      const int kvh = h - Hq - Hkv;
      const int64_t blk = slot / block_size, off = slot % block_size;
      __nv_bfloat16* dst = v_cache + ((blk * Hkv + kvh) * block_size + off) * 128;
      reinterpret_cast<uint32_t*>(dst)[lane] = reinterpret_cast<const uint32_t*>(row)[lane];
      reinterpret_cast<uint32_t*>(dst)[lane + 32] = reinterpret_cast<const uint32_t*>(row)[lane + 32];
    }
    return;
  }
  float2 a = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(row)[lane]);
  float2 b = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(row + 64)[lane]);
  const __nv_bfloat16* nw = (h < Hq) ? qn_w : kn_w;
  if (nw != nullptr) {
    float ss = warp_sum(a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y);
    float inv = rsqrtf(ss / 128.f + eps);
    float2 wa = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(nw)[lane]);
    float2 wb = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(nw + 64)[lane]);
    // Round to bf16 after the norm, as the served module's output would be.
    a.x = bf2f(f2bf(a.x * inv * wa.x));
    a.y = bf2f(f2bf(a.y * inv * wa.y));
    b.x = bf2f(f2bf(b.x * inv * wb.x));
    b.y = bf2f(f2bf(b.y * inv * wb.y));
  }
  const float* cs = cos_sin + positions[tok] * 128;  // [cos(64) | sin(64)]
  const float c0 = cs[2 * lane], c1 = cs[2 * lane + 1];
  const float s0 = cs[64 + 2 * lane], s1 = cs[64 + 2 * lane + 1];
  float2 ra = make_float2(a.x * c0 - b.x * s0, a.y * c1 - b.y * s1);
  float2 rb = make_float2(b.x * c0 + a.x * s0, b.y * c1 + a.y * s1);
  __nv_bfloat162 ha = __floats2bfloat162_rn(ra.x, ra.y), hb = __floats2bfloat162_rn(rb.x, rb.y);
  reinterpret_cast<__nv_bfloat162*>(row)[lane] = ha;
  reinterpret_cast<__nv_bfloat162*>(row + 64)[lane] = hb;
  if (h >= Hq && slot >= 0) {
    const int kvh = h - Hq;
    const int64_t blk = slot / block_size, off = slot % block_size;
    __nv_bfloat16* dst = k_cache + ((blk * Hkv + kvh) * block_size + off) * 128;
    reinterpret_cast<__nv_bfloat162*>(dst)[lane] = ha;
    reinterpret_cast<__nv_bfloat162*>(dst + 64)[lane] = hb;
  }
}

}  // namespace dsv

void dsv_rms_norm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w, torch::Tensor out,
                  double eps, c10::optional<torch::Tensor> save, int64_t save_lo, int64_t save_hi, int64_t save_dst) {
  using namespace dsv;
  const int T = (int)x.size(0), D = (int)x.size(1);
  if (T == 0) return;
  TORCH_CHECK(D % 8 == 0 && x.stride(1) == 1 && out.stride(1) == 1, "rms_norm: D % 8 == 0, contiguous rows");
  c10::cuda::CUDAGuard guard(x.device());
  const int threads = std::min(1024, std::max(32, ((D / 8 + 31) / 32) * 32));
  const size_t smem = (D + 32) * sizeof(float);
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  __nv_bfloat16* sv = save.has_value() ? reinterpret_cast<__nv_bfloat16*>(save->data_ptr()) : nullptr;
  const int ssv = save.has_value() ? (int)save->stride(0) : 0;
  auto X = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto W = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto O = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (residual.has_value()) {
    rms_norm_kernel<true><<<T, threads, smem, s>>>(X, (int)x.stride(0), reinterpret_cast<__nv_bfloat16*>(residual->data_ptr()),
                                                   (int)residual->stride(0), W, O, (int)out.stride(0), D, (float)eps, sv, ssv,
                                                   (int)save_lo, (int)save_hi, (int)save_dst);
  } else {
    rms_norm_kernel<false><<<T, threads, smem, s>>>(X, (int)x.stride(0), nullptr, 0, W, O, (int)out.stride(0), D, (float)eps,
                                                    sv, ssv, (int)save_lo, (int)save_hi, (int)save_dst);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_qk_norm_rope_cache(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                            c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, double eps,
                            int64_t num_heads, int64_t num_kv_heads, c10::optional<torch::Tensor> k_cache,
                            c10::optional<torch::Tensor> v_cache, c10::optional<torch::Tensor> slot_mapping) {
  using namespace dsv;
  const int T = (int)qkv.size(0);
  if (T == 0) return;
  TORCH_CHECK(qkv.stride(1) == 1 && positions.scalar_type() == at::kLong && cos_sin.scalar_type() == at::kFloat,
              "qk_norm_rope_cache: bad inputs");
  c10::cuda::CUDAGuard guard(qkv.device());
  const int H = (int)(num_heads + 2 * num_kv_heads);
  const int64_t warps = (int64_t)T * H;
  const int threads = 256;
  const int blocks = (int)((warps * 32 + threads - 1) / threads);
  int bs = 0;
  __nv_bfloat16 *kc = nullptr, *vc = nullptr;
  const int64_t* sm = nullptr;
  if (k_cache.has_value()) {
    kc = reinterpret_cast<__nv_bfloat16*>(k_cache->data_ptr());
    vc = reinterpret_cast<__nv_bfloat16*>(v_cache->data_ptr());
    bs = (int)k_cache->size(2);
    sm = slot_mapping->data_ptr<int64_t>();
  }
  qk_norm_rope_cache_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), (int)qkv.stride(0), positions.data_ptr<int64_t>(),
      cos_sin.data_ptr<float>(),
      q_norm.has_value() ? reinterpret_cast<const __nv_bfloat16*>(q_norm->data_ptr()) : nullptr,
      k_norm.has_value() ? reinterpret_cast<const __nv_bfloat16*>(k_norm->data_ptr()) : nullptr, (float)eps,
      (int)num_heads, (int)num_kv_heads, kc, vc, sm, bs, T,
      k_cache.has_value() ? (int64_t)k_cache->size(0) * bs : (int64_t)0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ backward
namespace dsv {

// dx = rmsnorm_backward(x, dy) [+ add]; fp32 out, optional bf16 copy.
// x bf16 (row stride sx), dy / add / dx fp32 [T, D], w bf16 [D].
// d/dx of x * inv * w = inv * (g - xhat * mean(g * xhat)), g = dy * w.
//
// Wide rows: one CTA of 256 threads per row, NCH chunks of 8 consecutive
// elements per thread held in registers between the reduction and the store
// (16-byte loads and stores).
template <int NCH>
__global__ void __launch_bounds__(256) rms_norm_bwd_vec_kernel(const __nv_bfloat16* __restrict__ x, int sx,
                                                               const float* __restrict__ dy,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               const float* __restrict__ add, float* dx,
                                                               __nv_bfloat16* dx_bf, int D, float eps) {
  __shared__ float2 red[8];
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)row * sx;
  const float* dyr = dy + (size_t)row * D;
  float xv[NCH][8], gv[NCH][8];
  float ss = 0.f, dot = 0.f;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int i = (threadIdx.x + k * 256) * 8;
    if (i < D) {
      const uint4 xq = *reinterpret_cast<const uint4*>(xr + i);
      const uint4 wq = *reinterpret_cast<const uint4*>(w + i);
      const float4 d0 = *reinterpret_cast<const float4*>(dyr + i);
      const float4 d1 = *reinterpret_cast<const float4*>(dyr + i + 4);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xq);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wq);
      const float d[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        xv[k][e] = bf2f(xb[e]);
        gv[k][e] = d[e] * bf2f(wb[e]);
        ss += xv[k][e] * xv[k][e];
        dot += gv[k][e] * xv[k][e];
      }
    }
  }
  ss = warp_sum(ss);
  dot = warp_sum(dot);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(ss, dot);
  __syncthreads();
  float2 t = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    t.x += red[i].x;
    t.y += red[i].y;
  }
  const float inv = rsqrtf(t.x / D + eps);
  const float c = t.y * inv * inv / D;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int i = (threadIdx.x + k * 256) * 8;
    if (i >= D) continue;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = inv * (gv[k][e] - xv[k][e] * c);
    if (add != nullptr) {
      const float4 a0 = *reinterpret_cast<const float4*>(add + (size_t)row * D + i);
      const float4 a1 = *reinterpret_cast<const float4*>(add + (size_t)row * D + i + 4);
      v[0] += a0.x; v[1] += a0.y; v[2] += a0.z; v[3] += a0.w;
      v[4] += a1.x; v[5] += a1.y; v[6] += a1.z; v[7] += a1.w;
    }
    float4* o = reinterpret_cast<float4*>(dx + (size_t)row * D + i);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
    if (dx_bf != nullptr) {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
        pk[e] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(dx_bf + (size_t)row * D + i) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
}

// Narrow rows (per-head q/k norms, D <= 256): one warp per row, D / 32
// consecutive elements per lane.
template <int PER>
__global__ void __launch_bounds__(256) rms_norm_bwd_warp_kernel(const __nv_bfloat16* __restrict__ x, int sx,
                                                                const float* __restrict__ dy,
                                                                const __nv_bfloat16* __restrict__ w,
                                                                const float* __restrict__ add, float* dx,
                                                                __nv_bfloat16* dx_bf, int T, int D, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= T) return;
  const int lane = threadIdx.x & 31;
  const int i0 = lane * PER;
  float xv[PER], gv[PER];
  float ss = 0.f, dot = 0.f;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    xv[e] = bf2f(x[(size_t)row * sx + i0 + e]);
    gv[e] = dy[(size_t)row * D + i0 + e] * bf2f(w[i0 + e]);
    ss += xv[e] * xv[e];
    dot += gv[e] * xv[e];
  }
  ss = warp_sum(ss);
  dot = warp_sum(dot);
  const float inv = rsqrtf(ss / D + eps);
  const float c = dot * inv * inv / D;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    float v = inv * (gv[e] - xv[e] * c);
    if (add != nullptr) v += add[(size_t)row * D + i0 + e];
    dx[(size_t)row * D + i0 + e] = v;
    if (dx_bf != nullptr) dx_bf[(size_t)row * D + i0 + e] = f2bf(v);
  }
}

// General fallback (any D): one CTA per row, scalar loads.
__global__ void rms_norm_bwd_kernel(const __nv_bfloat16* __restrict__ x, int sx, const float* __restrict__ dy,
                                    const __nv_bfloat16* __restrict__ w, const float* __restrict__ add,
                                    float* dx, __nv_bfloat16* dx_bf, int D, float eps) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)row * sx;
  const float* dyr = dy + (size_t)row * D;
  float ss = 0.f, dot = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float xv = bf2f(xr[i]);
    ss += xv * xv;
    dot += dyr[i] * bf2f(w[i]) * xv;
  }
  auto bsum = [&](float v) {
    v = warp_sum(v);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
    __syncthreads();
    float t = (threadIdx.x < blockDim.x / 32) ? red[threadIdx.x] : 0.f;
    if (threadIdx.x < 32) t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    float r = red[0];
    __syncthreads();
    return r;
  };
  ss = bsum(ss);
  dot = bsum(dot);
  const float inv = rsqrtf(ss / D + eps);
  const float c = dot * inv * inv / D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float xv = bf2f(xr[i]);
    float v = inv * (dyr[i] * bf2f(w[i]) - xv * c);
    if (add != nullptr) v += add[(size_t)row * D + i];
    dx[(size_t)row * D + i] = v;
    if (dx_bf != nullptr) dx_bf[(size_t)row * D + i] = f2bf(v);
  }
}

// SwiGLU backward over 64-interleaved gate/up: from the saved pre-activation
// gu (bf16) and d_act (fp32) produce d_gu (bf16, same interleave) and the
// activation silu(g)*u (bf16, the down projection's input). One thread per 8
// consecutive d_act columns (inside one 64-column block): 16-byte loads and
// stores throughout.
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, int sgu, const float* __restrict__ dact,
                                  __nv_bfloat16* dgu, __nv_bfloat16* act, int I, int64_t total8) {
  const int per_row = I / 8;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total8;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / per_row;
    const int j = (int)(idx % per_row) * 8;
    const int col_g = (j / 64) * 128 + (j % 64);
    const uint4 gq = *reinterpret_cast<const uint4*>(gu + row * sgu + col_g);
    const uint4 uq = *reinterpret_cast<const uint4*>(gu + row * sgu + col_g + 64);
    const float4 d0 = *reinterpret_cast<const float4*>(dact + row * I + j);
    const float4 d1 = *reinterpret_cast<const float4*>(dact + row * I + j + 4);
    const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gq);
    const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&uq);
    const float da[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
    uint32_t og[4], ou[4], oa[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      float rg[2], ru[2], ra[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const float g = bf2f(gb[e + t]), u = bf2f(ub[e + t]);
        const float sg = 1.f / (1.f + __expf(-g));
        const float silu = g * sg;
        rg[t] = da[e + t] * u * sg * (1.f + g * (1.f - sg));
        ru[t] = da[e + t] * silu;
        ra[t] = silu * u;
      }
      __nv_bfloat162 hg = __floats2bfloat162_rn(rg[0], rg[1]);
      __nv_bfloat162 hu = __floats2bfloat162_rn(ru[0], ru[1]);
      __nv_bfloat162 ha = __floats2bfloat162_rn(ra[0], ra[1]);
      og[e / 2] = *reinterpret_cast<uint32_t*>(&hg);
      ou[e / 2] = *reinterpret_cast<uint32_t*>(&hu);
      oa[e / 2] = *reinterpret_cast<uint32_t*>(&ha);
    }
    __nv_bfloat16* drow = dgu + row * (2 * (int64_t)I);
    *reinterpret_cast<uint4*>(drow + col_g) = make_uint4(og[0], og[1], og[2], og[3]);
    *reinterpret_cast<uint4*>(drow + col_g + 64) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
    if (act != nullptr) *reinterpret_cast<uint4*>(act + row * I + j) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
  }
}

}  // namespace dsv

void dsv_rms_norm_bwd(torch::Tensor x, torch::Tensor dy, torch::Tensor w, c10::optional<torch::Tensor> add,
                      torch::Tensor dx, c10::optional<torch::Tensor> dx_bf, double eps) {
  const int T = (int)x.size(0), D = (int)x.size(1);
  if (T == 0) return;
  TORCH_CHECK(dy.scalar_type() == at::kFloat && dx.scalar_type() == at::kFloat && dy.is_contiguous() &&
                  dx.is_contiguous(), "rms_norm_bwd: fp32 contiguous dy/dx");
  if (add.has_value())
    TORCH_CHECK(add->scalar_type() == at::kFloat && add->is_contiguous() && add->numel() == (int64_t)T * D,
                "rms_norm_bwd: add must be fp32 [T, D]");
  if (dx_bf.has_value())
    TORCH_CHECK(dx_bf->scalar_type() == at::kBFloat16 && dx_bf->is_contiguous() && dx_bf->numel() == (int64_t)T * D,
                "rms_norm_bwd: bf16 copy must be contiguous [T, D]");
  c10::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  const float* ap = add.has_value() ? add->data_ptr<float>() : nullptr;
  auto* bp = dx_bf.has_value() ? reinterpret_cast<__nv_bfloat16*>(dx_bf->data_ptr()) : nullptr;
  const int sx = (int)x.stride(0);
  auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const bool vec_ok = D % 8 == 0 && sx % 8 == 0 && al16(xp) && al16(wp) && al16(dy.data_ptr()) &&
                      al16(dx.data_ptr()) && (ap == nullptr || al16(ap)) && (bp == nullptr || al16(bp));
  if (vec_ok && D >= 512 && D <= 8192) {
    const int nch = (D + 2047) / 2048;
    if (nch == 1) dsv::rms_norm_bwd_vec_kernel<1><<<T, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, D, (float)eps);
    else if (nch == 2) dsv::rms_norm_bwd_vec_kernel<2><<<T, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, D, (float)eps);
    else if (nch == 3) dsv::rms_norm_bwd_vec_kernel<3><<<T, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, D, (float)eps);
    else dsv::rms_norm_bwd_vec_kernel<4><<<T, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, D, (float)eps);
  } else if (D % 32 == 0 && D <= 256) {
    const int per = D / 32;
    const int blocks = (T + 7) / 8;
    if (per == 1) dsv::rms_norm_bwd_warp_kernel<1><<<blocks, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, T, D, (float)eps);
    else if (per == 2) dsv::rms_norm_bwd_warp_kernel<2><<<blocks, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, T, D, (float)eps);
    else if (per == 4) dsv::rms_norm_bwd_warp_kernel<4><<<blocks, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, T, D, (float)eps);
    else if (per == 8) dsv::rms_norm_bwd_warp_kernel<8><<<blocks, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, T, D, (float)eps);
    else dsv::rms_norm_bwd_kernel<<<T, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, D, (float)eps);
  } else {
    dsv::rms_norm_bwd_kernel<<<T, 256, 0, st>>>(xp, sx, dy.data_ptr<float>(), wp, ap, dx.data_ptr<float>(), bp, D, (float)eps);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_swiglu_bwd(torch::Tensor gu, torch::Tensor dact, torch::Tensor dgu, c10::optional<torch::Tensor> act) {
  const int64_t T = gu.size(0);
  const int I = (int)dact.size(1);
  if (T == 0) return;
  TORCH_CHECK(I % 64 == 0 && gu.size(1) == 2 * I && dact.is_contiguous() && dgu.is_contiguous(), "swiglu_bwd");
  TORCH_CHECK(gu.stride(1) == 1 && gu.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(gu.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(dact.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(dgu.data_ptr()) % 16 == 0,
              "swiglu_bwd: 16-byte aligned rows");
  if (act.has_value())
    TORCH_CHECK(act->is_contiguous() && reinterpret_cast<uintptr_t>(act->data_ptr()) % 16 == 0,
                "swiglu_bwd: act must be contiguous and 16-byte aligned");
  c10::cuda::CUDAGuard guard(gu.device());
  const int64_t total = T * I / 8;
  const int blocks = (int)std::min<int64_t>(148 * 16, (total + 255) / 256);
  dsv::swiglu_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), (int)gu.stride(0), dact.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()),
      act.has_value() ? reinterpret_cast<__nv_bfloat16*>(act->data_ptr()) : nullptr, I, total);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
