// Allocation-free C entry point of the split-KV paged decode attention.
//
// This entry point has no counterpart in the reference project; it is an
// addition of this library for callers that cannot allocate device memory.
//
// Who needs it: C/C++ hosts that own every byte of device memory through their
// own allocator (an inference runtime with a fixed memory plan, a game or
// simulation engine embedding the kernel) and must not call cudaMalloc behind
// that allocator's back, and latency-critical paths where cudaMalloc/cudaFree
// are not acceptable because they can synchronize the whole device. The
// regular entry point (dsv_paged_decode, via PyTorch) takes its split-KV
// partial-result workspace from the caller's allocator; this one instead uses a
// fixed scratch array compiled into the library, so it allocates nothing.
//
// Contract:
// * Scratch: a file-scope __device__ array of DSV_NOALLOC_SCRATCH_FLOATS floats
//   (4 MiB) that every GPU which loads the library holds until process exit.
//   The call needs batch * num_heads * splits * 130 floats of it and fails with
//   DSV_NOALLOC_ETOOBIG beyond that.
// * The first call on a device looks up the array's device address (with that
//   device current) and caches it; make that first call before any stream
//   capture on the device.
// * Every call shares the one array: calls whose kernels overlap on the GPU
//   (different streams, or different host threads) race on it. Serialise them
//   on one stream. Nothing in the array has to start at zero: each call writes
//   every partial result it later reads.
// * keys_per_split: a multiple of 64 keys per split, or 0 to let each sequence
//   split its own context evenly over `splits` (as dsv_paged_decode does).
// * Errors: DSV_NOALLOC_ECUDA is returned without launching when a CUDA error
//   from an earlier call is already pending on the thread (it is left in place
//   for its owner); a failed launch of this call is consumed and reported.
// * Inputs and outputs are caller-owned device pointers with the layouts of
//   dsv_paged_decode: q [batch, q_stride] bf16 (head h at h*128), caches
//   [num_blocks, num_kv_heads, block_size, 128] bf16, block_tables
//   [batch, max_blocks] int32, ctx_lens [batch] int32, out [batch, out_stride]
//   bf16.
#pragma once

#include <cuda_runtime.h>

#define DSV_NOALLOC_SCRATCH_FLOATS (1 << 20)

enum {
  DSV_NOALLOC_OK = 0,
  DSV_NOALLOC_EINVAL = 1,    // bad argument (null pointer, group size, split size < 0 or not a multiple of 64)
  DSV_NOALLOC_ETOOBIG = 2,   // batch * heads * splits exceeds the scratch array
  DSV_NOALLOC_ECUDA = 3,     // a CUDA call failed (device lookup, symbol address, launch)
};

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int dsv_paged_decode_noalloc(
    const void* q, int q_stride, const void* k_cache, const void* v_cache, int num_kv_heads, int block_size,
    const int* block_tables, int max_blocks, const int* ctx_lens, int batch, void* out, int out_stride,
    int num_heads, float scale, int splits, int keys_per_split, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
