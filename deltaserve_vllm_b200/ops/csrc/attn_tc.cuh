// Helpers shared by the tcgen05 attention kernels (attn_tc.cu, attn_bwd_tc.cu).
//
// Tile layout: a [rows x 128] bf16 operand tile is two 64-column chunks of
// [rows x 128 B] in the 128-byte-swizzle layout a TMA box {64, rows} writes
// (16-byte unit u of row r stored at unit u ^ (r % 8)); a [rows x 64] tile is
// one chunk. Descriptors address k-step kk (16 elements along the MMA's K):
//   K-major (K contiguous): chunk kk / 4, byte offset (kk % 4) * 32 in the row;
//   MN-major (N contiguous, K = rows): 16 rows per k-step; the next 64 N
//   columns are the next chunk (LBO = chunk bytes).
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

#include "common.cuh"

namespace dsv {

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int kk, uint32_t chunk_bytes) {
  return smem_desc(tile + (kk >> 2) * chunk_bytes + (kk & 3) * 32, 16, 1024, kSwizzle128B);
}
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int kk, uint32_t chunk_bytes) {
  return smem_desc(tile + kk * 16 * 128, chunk_bytes, 1024, kSwizzle128B);
}

// Store 32 consecutive bf16 values (packed from fp32) as 4 swizzled 16-byte
// units starting at unit u0 of row r of a 128-byte-row chunk at `chunk`.
__device__ __forceinline__ void store_row_units(uint8_t* chunk, int r, int u0, const float* v) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint4 w;
    w.x = pack2_bf16(v[u * 8 + 0], v[u * 8 + 1]);
    w.y = pack2_bf16(v[u * 8 + 2], v[u * 8 + 3]);
    w.z = pack2_bf16(v[u * 8 + 4], v[u * 8 + 5]);
    w.w = pack2_bf16(v[u * 8 + 6], v[u * 8 + 7]);
    *reinterpret_cast<uint4*>(chunk + r * 128 + ((((u0 + u) & 7) ^ (r & 7)) << 4)) = w;
  }
}

}  // namespace dsv
