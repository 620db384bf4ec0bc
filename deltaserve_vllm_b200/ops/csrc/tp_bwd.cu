// Tensor-parallel LoRA backward: the residual-gradient reductions as
// GEMM -> reduce-scatter -> RMSNorm backward -> all-gather over NVLink peer
// memory, and the vocabulary-parallel LM head's cross-entropy statistics.
//
// Reduction of one residual-stream gradient (a dX GEMM whose output is a
// per-rank partial sum over the rank's shard of the reduction dimension):
//
//   1. the dX GEMM's epilogue (gemm_tc.cu, kEpiPushRows) stores each 128-row
//      block's bf16 partial into the receive rows of the block's owner rank
//      (block mt -> rank mt % world) and adds its column count to the owner's
//      block counter (release, system scope); nothing waits there;
//   2. wait_counts_kernel (one CTA): waits until every owned block counted
//      world * N columns, then resets the counters;
//   3. reduce_norm_bcast_kernel (no waits): for each owned row, sums the world
//      partials in fp32, applies the RMSNorm backward (+ the residual
//      gradient, fp32, owned rows only) and writes the fp32 result locally and
//      the bf16 result into every rank's gather buffer (P2P stores), then adds
//      1 to the block's row counter on every peer;
//   4. wait_counts_kernel (one CTA): waits until every block owned by another
//      rank has all its rows, then resets those counters.
//
// Only the two one-CTA kernels wait, and only on work that never waits (the
// peers' GEMM epilogues and reduce kernels), so the waits cannot form a
// cycle with each other or with the forward stream's fused all-reduce
// (whose grid leaves the SMs these need). Every wait is bounded (2 s): on
// timeout it records kErrWaitPeer and returns.
//
// Buffer reuse needs no epochs: a rank pushes the partials of the next
// reduction only after its step 4 of this one, which needs every owner's
// step 3, which comes after that owner's reads of this reduction's partials.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace dsv {

constexpr int kTpMaxPeers = 8;

// ---------------------------------------------------------------- waits
// One CTA of 32 threads: counter i (for i in [0, n), skipping the ones with
// i % skip_mod == skip_rem when skip_mod > 0) must reach target(i), where
// target(i) = per_block when rows == 0, else the number of rows of 128-row
// block i of an M-row matrix. Each counter is reset once reached.
__global__ void wait_counts_kernel(uint32_t* cnt, int n, uint32_t per_block, int rows, int skip_mod, int skip_rem) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (skip_mod > 0 && i % skip_mod == skip_rem) continue;
    const uint32_t target = rows > 0 ? (uint32_t)min(128, rows - i * 128) : per_block;
    if (wait_flag_geq(cnt + i, target)) st_relaxed_sys(cnt + i, 0u);
  }
}

// ---------------------------------------------------------------- reduce + norm + broadcast
struct ReduceNormArgs {
  const __nv_bfloat16* recv;   // this rank's receive rows: [world][blocks_cap][128][ld]
  int world, rank, blocks_cap, ld, M, D;
  const __nv_bfloat16* x;      // norm input rows [M, sx] (bf16), or null: no norm
  int sx;
  const __nv_bfloat16* w;      // norm weight [D]
  float eps;
  const float* add;            // optional residual gradient [M, ld_add] (owned rows read)
  int ld_add;
  float* out;                  // fp32 result [M, ld_out] (owned rows written)
  int ld_out;
  __nv_bfloat16* gather[kTpMaxPeers];   // every rank's bf16 gather buffer [M, ld]
  uint32_t* gcnt[kTpMaxPeers];          // every rank's per-block row counters
};

// One CTA (256 threads) per owned row, NCH x 8 columns per thread.
template <int NCH>
__global__ void __launch_bounds__(256) reduce_norm_bcast_kernel(ReduceNormArgs a) {
  __shared__ float2 red[8];
  const int n_blocks = (a.M + 127) / 128;
  const int n_owned_blocks = (n_blocks - a.rank + a.world - 1) / a.world;
  const int owned_rows = n_owned_blocks * 128;
  for (int o = blockIdx.x; o < owned_rows; o += gridDim.x) {
    const int j = o / 128, i = o % 128;
    const int mt = j * a.world + a.rank;
    const int row = mt * 128 + i;
    if (row >= a.M) continue;  // uniform across the CTA
    float acc[NCH][8], xv[NCH][8];
    float ss = 0.f, dot = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = (threadIdx.x + k * 256) * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[k][e] = 0.f;
      if (c >= a.D) continue;
      for (int s = 0; s < a.world; ++s) {
        const __nv_bfloat16* src = a.recv + ((size_t)(s * a.blocks_cap + j) * 128 + i) * a.ld + c;
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(src));
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[k][2 * e] += f.x;
          acc[k][2 * e + 1] += f.y;
        }
      }
      if (a.x != nullptr) {
        const uint4 xq = *reinterpret_cast<const uint4*>(a.x + (size_t)row * a.sx + c);
        const uint4 wq = *reinterpret_cast<const uint4*>(a.w + c);
        const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xq);
        const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wq);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xv[k][e] = bf2f(xb[e]);
          acc[k][e] *= bf2f(wb[e]);   // g = dy * w
          ss += xv[k][e] * xv[k][e];
          dot += acc[k][e] * xv[k][e];
        }
      }
    }
    float inv = 1.f, cc = 0.f;
    if (a.x != nullptr) {
      ss = warp_sum(ss);
      dot = warp_sum(dot);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_float2(ss, dot);
      __syncthreads();
      float2 t = red[0];
#pragma unroll
      for (int q = 1; q < 8; ++q) {
        t.x += red[q].x;
        t.y += red[q].y;
      }
      __syncthreads();  // red is rewritten by the next row
      inv = rsqrtf(t.x / a.D + a.eps);
      cc = t.y * inv * inv / a.D;
    }
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = (threadIdx.x + k * 256) * 8;
      if (c >= a.D) continue;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = a.x != nullptr ? inv * (acc[k][e] - xv[k][e] * cc) : acc[k][e];
      if (a.add != nullptr) {
        const float4 a0 = *reinterpret_cast<const float4*>(a.add + (size_t)row * a.ld_add + c);
        const float4 a1 = *reinterpret_cast<const float4*>(a.add + (size_t)row * a.ld_add + c + 4);
        v[0] += a0.x; v[1] += a0.y; v[2] += a0.z; v[3] += a0.w;
        v[4] += a1.x; v[5] += a1.y; v[6] += a1.z; v[7] += a1.w;
      }
      float4* op = reinterpret_cast<float4*>(a.out + (size_t)row * a.ld_out + c);
      op[0] = make_float4(v[0], v[1], v[2], v[3]);
      op[1] = make_float4(v[4], v[5], v[6], v[7]);
      uint4 pk;
      uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
        pw[e] = *reinterpret_cast<uint32_t*>(&h2);
      }
      for (int d = 0; d < a.world; ++d) {
        const int dr = (a.rank + d) % a.world;  // stagger the peers
        *reinterpret_cast<uint4*>(a.gather[dr] + (size_t)row * a.ld + c) = pk;
      }
    }
    __syncthreads();  // every thread's stores of this row are issued
    if (threadIdx.x < a.world && threadIdx.x != a.rank) {
      __threadfence_system();
      red_release_sys_add(a.gcnt[threadIdx.x] + mt, 1u);
    }
  }
}

// ---------------------------------------------------------------- LM head statistics
// Merge the per-tile (max, sum exp) pairs of one row (one warp per row) and
// append the label's logit: part[row] = (max, sum exp(logit - max), tgt).
__global__ void ce_merge_kernel(const float2* __restrict__ stats, int ld, int n_tiles, int M,
                                const float* __restrict__ tgt, float* __restrict__ part) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float m = -INFINITY, s = 0.f;
  for (int t = lane; t < n_tiles; t += 32) {
    const float2 p = stats[(size_t)row * ld + t];
    if (p.y <= 0.f) continue;
    const float mn = fmaxf(m, p.x);
    s = s * __expf(m - mn) + p.y * __expf(p.x - mn);
    m = mn;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = fmaxf(m, om);
    if (mn == -INFINITY) continue;  // both empty
    s = s * __expf(m - mn) + os * __expf(om - mn);
    m = mn;
  }
  if (lane == 0) {
    part[(size_t)row * 3] = m;
    part[(size_t)row * 3 + 1] = s;
    part[(size_t)row * 3 + 2] = tgt[row];
  }
}

// Across the ranks' vocabulary slices: lse = log(sum_r s_r exp(m_r - M)) + M,
// loss = lse - (the label's logit, from the one slice that holds it; the
// others contributed 0). Rows without a label get loss 0.
__global__ void ce_finalize_kernel(const float* __restrict__ parts, int world, int M,
                                   const int64_t* __restrict__ labels, float* __restrict__ lse,
                                   float* __restrict__ loss) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= M) return;
  float mx = -INFINITY;
  for (int r = 0; r < world; ++r) mx = fmaxf(mx, parts[((size_t)r * M + row) * 3]);
  float s = 0.f, t = 0.f;
  for (int r = 0; r < world; ++r) {
    const float* p = parts + ((size_t)r * M + row) * 3;
    if (p[1] > 0.f) s += p[1] * __expf(p[0] - mx);
    t += p[2];
  }
  const float l = mx + logf(s);
  lse[row] = l;
  loss[row] = labels[row] >= 0 ? l - t : 0.f;
}

}  // namespace dsv

// ------------------------------------------------------------------ host side

// Wait (one CTA) for counters of this rank's workspace; see wait_counts_kernel.
void dsv_wait_counts(int64_t cnt, int64_t n, int64_t per_block, int64_t rows, int64_t skip_mod, int64_t skip_rem) {
  using namespace dsv;
  if (n <= 0) return;
  wait_counts_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<uint32_t*>(cnt), (int)n,
                                                                     (uint32_t)per_block, (int)rows, (int)skip_mod,
                                                                     (int)skip_rem);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Sum this rank's owned rows over the world partials in `recv`, apply the
// RMSNorm backward (when x is given) plus `add`, write fp32 rows into `out`
// and bf16 rows into every rank's gather buffer; `table` is an int64 CPU
// tensor [2, world] (gather buffers, row counters).
void dsv_reduce_norm_bcast(int64_t recv, int64_t rank, int64_t world, int64_t blocks_cap, int64_t ld, int64_t M,
                           int64_t D, c10::optional<torch::Tensor> x, c10::optional<torch::Tensor> w, double eps,
                           c10::optional<torch::Tensor> add, torch::Tensor out, torch::Tensor table) {
  using namespace dsv;
  TORCH_CHECK(world >= 1 && world <= kTpMaxPeers && rank >= 0 && rank < world, "reduce_norm: rank/world");
  TORCH_CHECK(D % 8 == 0 && ld % 8 == 0 && D <= ld && D <= 4 * 256 * 8, "reduce_norm: D % 8 == 0, D <= 8192");
  TORCH_CHECK(table.device().is_cpu() && table.scalar_type() == at::kLong && table.size(0) == 2 &&
                  table.size(1) == world, "reduce_norm: table must be int64 [2, world] on the CPU");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.size(0) >= M && out.size(1) >= D && out.stride(1) == 1 &&
                  out.stride(0) % 4 == 0, "reduce_norm: out must be fp32 [M, >= D] with 16-byte rows");
  if (M <= 0) return;
  c10::cuda::CUDAGuard guard(out.device());
  ReduceNormArgs a{};
  a.recv = reinterpret_cast<const __nv_bfloat16*>(recv);
  a.world = (int)world;
  a.rank = (int)rank;
  a.blocks_cap = (int)blocks_cap;
  a.ld = (int)ld;
  a.M = (int)M;
  a.D = (int)D;
  if (x.has_value()) {
    TORCH_CHECK(w.has_value() && x->scalar_type() == at::kBFloat16 && x->stride(1) == 1 && x->stride(0) % 8 == 0 &&
                    x->size(0) >= M && x->size(1) == D && w->scalar_type() == at::kBFloat16 && w->numel() == D,
                "reduce_norm: x bf16 [M, D] with 16-byte rows and w bf16 [D]");
    a.x = reinterpret_cast<const __nv_bfloat16*>(x->data_ptr());
    a.sx = (int)x->stride(0);
    a.w = reinterpret_cast<const __nv_bfloat16*>(w->data_ptr());
  }
  a.eps = (float)eps;
  if (add.has_value()) {
    TORCH_CHECK(add->scalar_type() == at::kFloat && add->stride(1) == 1 && add->stride(0) % 4 == 0 &&
                    add->size(0) >= M && add->size(1) >= D, "reduce_norm: add must be fp32 [M, >= D]");
    a.add = add->data_ptr<float>();
    a.ld_add = (int)add->stride(0);
  }
  a.out = out.data_ptr<float>();
  a.ld_out = (int)out.stride(0);
  auto* tab = table.data_ptr<int64_t>();
  for (int r = 0; r < world; ++r) {
    a.gather[r] = reinterpret_cast<__nv_bfloat16*>(tab[r]);
    a.gcnt[r] = reinterpret_cast<uint32_t*>(tab[world + r]);
  }
  const int n_blocks = (int)((M + 127) / 128);
  const int owned = ((n_blocks - (int)rank + (int)world - 1) / (int)world) * 128;
  const int grid = std::max(1, std::min(owned, 4 * 148));
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const int nch = (int)((D / 8 + 255) / 256);
  if (nch <= 1) reduce_norm_bcast_kernel<1><<<grid, 256, 0, s>>>(a);
  else if (nch == 2) reduce_norm_bcast_kernel<2><<<grid, 256, 0, s>>>(a);
  else if (nch == 3) reduce_norm_bcast_kernel<3><<<grid, 256, 0, s>>>(a);
  else reduce_norm_bcast_kernel<4><<<grid, 256, 0, s>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// part [M, 3] = per-row (max, sum exp, label logit) of this rank's slice.
void dsv_ce_merge(torch::Tensor stats, int64_t n_tiles, torch::Tensor tgt, torch::Tensor part) {
  using namespace dsv;
  const int M = (int)part.size(0);
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.stride(1) == 1 && stats.stride(0) % 2 == 0 &&
                  stats.size(1) >= 2 * n_tiles, "ce_merge: stats");
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.is_contiguous() && part.size(1) == 3, "ce_merge: part [M, 3]");
  TORCH_CHECK(tgt.scalar_type() == at::kFloat && tgt.numel() >= M, "ce_merge: tgt");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(part.device());
  ce_merge_kernel<<<(M + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float2*>(stats.data_ptr<float>()), (int)(stats.stride(0) / 2), (int)n_tiles, M,
      tgt.data_ptr<float>(), part.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// parts [world, M, 3] -> lse [M], loss [M].
void dsv_ce_finalize(torch::Tensor parts, torch::Tensor labels, torch::Tensor lse, torch::Tensor loss) {
  using namespace dsv;
  TORCH_CHECK(parts.scalar_type() == at::kFloat && parts.is_contiguous() && parts.dim() == 3 && parts.size(2) == 3,
              "ce_finalize: parts [world, M, 3]");
  const int world = (int)parts.size(0), M = (int)parts.size(1);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.numel() >= M, "ce_finalize: labels");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(parts.device());
  ce_finalize_kernel<<<(M + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      parts.data_ptr<float>(), world, M, labels.data_ptr<int64_t>(), lse.data_ptr<float>(), loss.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

DSV_ERROR_ACCESSOR(dsv_read_error_tp_bwd)

// ================================================================ fused optimizer
// Replicated LoRA factors (column-parallel A, row-parallel B) hold the same
// values on every rank but each rank's gradient is a partial. Instead of an
// all-reduce of the gradients followed by AdamW on every rank, each rank owns
// a contiguous slice of the replicated block:
//   1. push_slices_kernel (during the backward, per finished bucket of layers):
//      the rank's partial gradient of every element goes to the element's
//      owner (recv[owner][rank][i - owner's first element], P2P stores); the
//      owner's counter grows by the elements stored (release);
//   2. wait_counts_kernel: every rank's elements of the owned slice arrived;
//   3. reduce_slice_sumsq_kernel: the owned slice is summed over the ranks
//      (into this rank's gradient buffer) and its per-layer sums of squares
//      accumulated;
//   4. exchange_rows_kernel + wait: every rank's per-layer sums of squares
//      (replicated slice + own shard) are written into every rank's table, so
//      each rank has the same per-layer gradient norm for clipping;
//   5. adamw_slice_bcast_kernel: AdamW with per-layer clipping on the owned
//      slice, the updated parameters stored into every rank's parameter
//      staging buffer (P2P) with the element count added to its counter;
//   6. wait: the other owners' slices arrived; they are copied into the
//      parameters (local), and the per-rank shard runs the plain AdamW.
// Only the one-CTA waits wait; reuse across cycles is ordered as in the
// residual reductions (a rank pushes cycle k+1 only after its step 6 of k).

namespace dsv {

struct SliceTable {
  float* recv[kTpMaxPeers];
  uint32_t* cnt[kTpMaxPeers];
};

// Elements [lo, hi) of the replicated block: element e goes to owner e / slice.
// One CTA stores a chunk of `chunk` elements (split where it crosses an
// owner's slice boundary) and bumps each owner's count by what it stored.
__global__ void push_slices_kernel(const float* __restrict__ g, int64_t lo, int64_t hi, int64_t slice, int rank,
                                   int64_t chunk, SliceTable t) {
  const int64_t c0 = lo + (int64_t)blockIdx.x * chunk;
  const int64_t cend = min(hi, c0 + chunk);
  for (int64_t a = c0; a < cend;) {
    const int owner = (int)(a / slice);
    const int64_t b = min(cend, (int64_t)(owner + 1) * slice);
    float* dst = t.recv[owner] + (int64_t)rank * slice - (int64_t)owner * slice;
    for (int64_t e = a + threadIdx.x; e < b; e += blockDim.x) dst[e] = g[e];
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      red_release_sys_add(t.cnt[owner], (uint32_t)(b - a));
    }
    a = b;
  }
}

// Owned slice of the replicated block, cut at layer boundaries into pieces:
// piece q covers block elements [lo[q], hi[q]) of layer seg[q]. CTA (x, q)
// sums a chunk of piece q over the ranks' partials (recv row s holds rank s's
// values for the slice starting at `first`), writes the sums into g and adds
// the chunk's sum of squares to sq[seg[q]] (one atomic per CTA).
constexpr int kMaxPieces = 64;
struct SlicePieces {
  int64_t lo[kMaxPieces], hi[kMaxPieces];
  int seg[kMaxPieces];
};

__global__ void reduce_slice_sumsq_kernel(const float* __restrict__ recv, int world, int64_t slice, int64_t first,
                                          int64_t chunk, SlicePieces pc, float* __restrict__ g, float* sq) {
  __shared__ float red[8];
  const int q = blockIdx.y;
  const int64_t c0 = pc.lo[q] + (int64_t)blockIdx.x * chunk;
  if (c0 >= pc.hi[q]) return;                   // uniform per CTA
  const int64_t c1 = min(pc.hi[q], c0 + chunk);
  float acc = 0.f;
  for (int64_t e = c0 + threadIdx.x; e < c1; e += blockDim.x) {
    const int64_t i = e - first;
    float v = 0.f;
    for (int s = 0; s < world; ++s) v += __ldcg(recv + (int64_t)s * slice + i);
    g[e] = v;
    acc += v * v;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(sq + pc.seg[q], t);
  }
}

// One CTA: row[l] = a[l] (+ b[l]) written into every rank's table at row
// `rank` (table[d] + rank * n), then each rank's counter + 1.
__global__ void exchange_rows_kernel(const float* __restrict__ a, const float* __restrict__ b, int n, int rank,
                                     int world, SliceTable t) {
  for (int d = 0; d < world; ++d) {
    float* dst = t.recv[d] + (int64_t)rank * n;
    for (int l = threadIdx.x; l < n; l += blockDim.x) dst[l] = a[l] + (b != nullptr ? b[l] : 0.f);
  }
  __syncthreads();
  if (threadIdx.x < world) {
    __threadfence_system();
    red_release_sys_add(t.cnt[threadIdx.x], 1u);
  }
}

// AdamW on the owned slice [first, first + len) with per-layer clipping from
// coef[layer]; the updated parameters go into every rank's staging buffer at
// the same offset (P2P), then each rank's counter grows by the chunk.
__global__ void adamw_slice_bcast_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                         float* __restrict__ v, int64_t first, int64_t len, int64_t seg_len,
                                         const float* __restrict__ coef, float lr, float b1, float b2, float eps,
                                         float wd, float bc1, float bc2, int rank, int world, int64_t chunk,
                                         SliceTable t) {
  const int64_t c0 = (int64_t)blockIdx.x * chunk;
  if (c0 >= len) return;
  const int64_t c1 = min(len, c0 + chunk);
  for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    const int64_t e = first + i;
    const float gi = g[e] * coef[e / seg_len];
    float pi = p[e];
    pi -= lr * wd * pi;
    const float mi = b1 * m[e] + (1.f - b1) * gi;
    const float vi = b2 * v[e] + (1.f - b2) * gi * gi;
    m[e] = mi;
    v[e] = vi;
    pi -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    p[e] = pi;
    for (int d = 0; d < world; ++d) {
      const int dr = (rank + d) % world;
      if (dr != rank) t.recv[dr][e] = pi;
    }
  }
  __syncthreads();
  if (threadIdx.x < world && threadIdx.x != rank) {
    __threadfence_system();
    red_release_sys_add(t.cnt[threadIdx.x], (uint32_t)(c1 - c0));
  }
}

// coef[l] = min(1, max_norm / (sqrt(sum over ranks of rows[r][l]) + 1e-6)).
__global__ void clip_coef_kernel(const float* __restrict__ rows, int world, int n, float max_norm, float* coef,
                                 float* total) {
  for (int l = blockIdx.x * blockDim.x + threadIdx.x; l < n; l += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += rows[(int64_t)r * n + l];
    total[l] = s;
    coef[l] = max_norm > 0.f ? fminf(1.f, max_norm / (sqrtf(s) + 1e-6f)) : 1.f;
  }
}

static SliceTable slice_table(torch::Tensor table, int world) {
  TORCH_CHECK(table.device().is_cpu() && table.scalar_type() == at::kLong && table.size(0) == 2 &&
                  table.size(1) == world, "slice table must be int64 [2, world] on the CPU");
  SliceTable t{};
  auto* p = table.data_ptr<int64_t>();
  for (int r = 0; r < world; ++r) {
    t.recv[r] = reinterpret_cast<float*>(p[r]);
    t.cnt[r] = reinterpret_cast<uint32_t*>(p[world + r]);
  }
  return t;
}

}  // namespace dsv

void dsv_push_slices(torch::Tensor g, int64_t lo, int64_t hi, int64_t slice, int64_t rank, int64_t world,
                     torch::Tensor table) {
  using namespace dsv;
  if (hi <= lo) return;
  TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && hi <= g.numel(), "push_slices: fp32 block");
  c10::cuda::CUDAGuard guard(g.device());
  const int64_t chunk = 8192;
  const int64_t blocks = (hi - lo + chunk - 1) / chunk;
  push_slices_kernel<<<(unsigned)blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      g.data_ptr<float>(), lo, hi, slice, (int)rank, chunk, slice_table(table, (int)world));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_reduce_slice_sumsq(int64_t recv, int64_t world, int64_t slice, int64_t first, int64_t len, int64_t seg_len,
                            torch::Tensor g, torch::Tensor sq) {
  using namespace dsv;
  if (len <= 0) return;
  SlicePieces pc{};
  int n = 0;
  for (int64_t a = first; a < first + len;) {
    const int64_t seg = a / seg_len;
    const int64_t b = std::min(first + len, (seg + 1) * seg_len);
    TORCH_CHECK(n < kMaxPieces, "reduce_slice_sumsq: the slice spans too many layers");
    pc.lo[n] = a;
    pc.hi[n] = b;
    pc.seg[n] = (int)seg;
    ++n;
    a = b;
  }
  int64_t longest = 0;
  for (int q = 0; q < n; ++q) longest = std::max(longest, pc.hi[q] - pc.lo[q]);
  const int64_t chunk = 8192;
  c10::cuda::CUDAGuard guard(g.device());
  reduce_slice_sumsq_kernel<<<dim3((unsigned)((longest + chunk - 1) / chunk), (unsigned)n), 256, 0,
                              at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const float*>(recv), (int)world,
                                                                  slice, first, chunk, pc, g.data_ptr<float>(),
                                                                  sq.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_exchange_rows(torch::Tensor a, c10::optional<torch::Tensor> b, int64_t rank, int64_t world,
                       torch::Tensor table) {
  using namespace dsv;
  c10::cuda::CUDAGuard guard(a.device());
  exchange_rows_kernel<<<1, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a.data_ptr<float>(), b.has_value() ? b->data_ptr<float>() : nullptr, (int)a.numel(), (int)rank, (int)world,
      slice_table(table, (int)world));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_clip_coef(torch::Tensor rows, double max_norm, torch::Tensor coef, torch::Tensor total) {
  using namespace dsv;
  c10::cuda::CUDAGuard guard(rows.device());
  const int world = (int)rows.size(0), n = (int)rows.size(1);
  clip_coef_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      rows.data_ptr<float>(), world, n, (float)max_norm, coef.data_ptr<float>(), total.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dsv_adamw_slice_bcast(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, int64_t first,
                           int64_t len, int64_t seg_len, torch::Tensor coef, double lr, double b1, double b2,
                           double eps, double wd, int64_t step, int64_t rank, int64_t world, torch::Tensor table) {
  using namespace dsv;
  if (len <= 0) return;
  c10::cuda::CUDAGuard guard(p.device());
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2 = 1.f - (float)std::pow(b2, (double)step);
  const int64_t chunk = 8192;
  const int64_t blocks = (len + chunk - 1) / chunk;
  adamw_slice_bcast_kernel<<<(unsigned)blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), first, len, seg_len,
      coef.data_ptr<float>(), (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, bc1, bc2, (int)rank,
      (int)world, chunk, slice_table(table, (int)world));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
