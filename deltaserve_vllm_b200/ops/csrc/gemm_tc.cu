// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M, N] = A[M, K] . B^T            (B stored [N, K] row-major: "K-major")
//   C[M, K] = A[M, N] . W              (W stored [N, K] row-major: "MN-major" B)
//   + optional fused multi-LoRA expand:  C += Z[M, S*SEG] . B2[N, S*SEG]^T, where
//     only the LoRA slots present in an M tile are visited (segmented expand).
//
// Design (one CTA per SM, 256 threads):
//   warp 0      TMA producer: A/B tiles (128 x 64 and BN x 64 bf16, 128-byte
//               swizzle) into a STAGES-deep shared-memory ring;
//   warp 1      one elected thread issues tcgen05.mma (M=128, N=BN, K=16) into a
//               TMEM accumulator, and tcgen05.commit releases the smem stage;
//   warp 2      allocates / frees TMEM (two accumulators of BN fp32 columns, so
//               the epilogue of tile i overlaps the main loop of tile i+1);
//   warps 4-7   epilogue: tcgen05.ld the accumulator (each warp owns 32 TMEM
//               lanes = 32 rows), convert, fuse (SwiGLU, FT-row save) and store.
// Tiles are walked M-fastest so CTAs running together share one weight tile
// (read once from HBM, the activation tiles hit L2).
//
// No TMA load here uses cluster multicast, and every wait is bounded
// (common.cuh): a stuck pipeline records an error code and the kernel returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "tmap.h"

namespace dsv {


enum Epilogue : int { kEpiBF16 = 0, kEpiF32 = 1, kEpiSwiGLU = 2, kEpiF32Accum = 3, kEpiPeerAR = 4,
                      kEpiShrink = 5, kEpiBF16T = 6, kEpiSwiGLUBwd = 7, kEpiCEStats = 8, kEpiCEGrad = 9,
                      kEpiPushRows = 10, kEpiF32T = 11, kEpiLoraBt = 12 };

// Weight-gradient GEMMs of the LoRA factors (kEpiF32T, kEpiLoraBt) reduce over
// the token dimension: both operands are token-major ([tokens, M] and
// [tokens, N] row-major), so A is read MN-major like B.
template <int EPI>
constexpr bool a_mn_major() { return EPI == kEpiF32T || EPI == kEpiLoraBt; }

constexpr int kMaxPeers = 8;
constexpr int kAgChunk = 512;      // columns per copy unit of the gathered all-gather GEMM
constexpr int kErrWaitGather = 0x4301;
constexpr int kArSmReserve = 20;  // SMs a fused all-reduce launch leaves free (backward NCCL cap + its waits)

// Fused all-reduce over peer memory (kEpiPeerAR). Every rank holds one
// workspace, mapped into every other rank's address space:
//   recv[world][owned_cap][BM*BN] bf16 — partial tiles pushed by each rank to
//                                        the tile's owner (rank L % world);
//   out[M][ldo] bf16                   — the reduced result;
//   rflag[owned_cap]                   — arrivals per owned tile (reset by owner);
//   fflag[tiles]                       — "final tile written" per output tile;
//   tile_cnt[tiles] (local)            — split-K arrivals (last split reduces).
struct PeerArgs {
  int rank, world, owned_cap, ldo;
  int reducers;           // CTAs [0, reducers) reduce / broadcast; the rest run the GEMM
  uint32_t* tile_cnt;
  __nv_bfloat16* recv[kMaxPeers];
  __nv_bfloat16* out[kMaxPeers];
  uint32_t* rflag[kMaxPeers];
  uint32_t* fflag[kMaxPeers];
};

// Row push to the row owner (kEpiPushRows, the tensor-parallel backward's
// "GEMM -> reduce-scatter"): 128-row block mt belongs to rank mt % world; the
// bf16 partial of a tile goes into the owner's receive rows
//   recv[owner][((rank * blocks_cap) + mt / world) * 128 + r][ld]
// (P2P stores), then one thread adds the tile's column count to the owner's
// arrival counter cnt[owner][mt / world] with release semantics. Nothing
// here waits: the owner's wait kernel counts world * N columns per block.
struct PushArgs {
  int rank, world, blocks_cap, ld;
  const float* add;       // optional fp32 [M, ld] added to the accumulator before the push
  int ld_add;
  __nv_bfloat16* recv[kMaxPeers];
  uint32_t* cnt[kMaxPeers];
};

struct GemmArgs {
  int M, N, K;            // C is M x N; K is the reduction length of the main term
  int lora_seg;           // LoRA: columns of Z / B2 per slot (multiple of 64); 0 = no LoRA term
  int num_slots;          // LoRA slots (<= 32)
  const uint32_t* tile_slots;  // [ceil(M/128)] bitmask of slots present in each M tile
  void* C;
  int ldc;                // elements
  __nv_bfloat16* save;    // optional: raw accumulator rows [save_lo, save_hi) -> save[save_dst + r - save_lo]
  int ld_save, save_lo, save_hi, save_dst;
  int max_ctas;           // host only: grid cap (0 = one CTA per SM, persistent)
  int k_splits;           // > 1: split-K, fp32 partials to `partial`, reduced by a second kernel
  // Launched right after the LoRA shrink that writes Z, allowed to start before it
  // ends: the producer waits for it (griddep_wait) before its first LoRA block, or
  // at the end when none of its tiles has one (the grid never outlives the shrink).
  int wait_prev;
  // All-gather -> GEMM: the 128-row blocks of A come from the rank that owns
  // them (ag_rows rows per rank, a multiple of 128), each through that rank's
  // tensor map (ag_maps: ag_world maps in global memory over the ranks' peer
  // buffers; TMA loads from peer memory, no multicast). Null: A is local.
  const CUtensorMap* ag_maps;
  int ag_rows, ag_world;
  // Copy-once gather: the epilogue warps of the running CTAs first copy the
  // remote row blocks, in units of 128 rows x kAgChunk columns claimed from
  // *ag_ticket, from the owners' shards (ag_src[r], plain P2P loads) into
  // this rank's gathered buffer (ag_gathered [M, K], read by the producer
  // through tmA), adding 1 to ag_cnt[block] per unit; a producer loads a
  // remote block once its count reached ag_expect (own blocks come from
  // ag_maps[ag_rank]). So each remote block crosses NVLink once, whatever the
  // number of N tiles.
  __nv_bfloat16* ag_gathered;
  uint32_t* ag_cnt;
  uint32_t* ag_ticket;
  uint32_t ag_expect;
  int ag_rank;
  const __nv_bfloat16* ag_src[8];
  float* partial;         // [k_splits, M, N]
  PeerArgs peer;          // kEpiPeerAR only
  // kEpiShrink: B is the stacked LoRA A [slots * pr, K]; output column
  // c = slot * pr + j lands in Z[row, slot * seg + j] when the row's slot is
  // `slot`, else 0; the segment's padding columns [pr, seg) are zeroed.
  const int* shrink_slot_ids;
  int shrink_pr, shrink_seg;
  // Swapped operands (kEpiBF16T, decode): the LoRA slots of every tile are
  // the OR of tile_slots[0, slot_or) (the token tiles), not tile_slots[mt].
  int slot_or;
  // kEpiSwiGLUBwd: the accumulator is d(act) [M, N]; aux holds the saved
  // gate/up pre-activations [M, 2N] (64-column interleave), C receives their
  // gradient [M, 2N] (same interleave), aux_out (optional) the activation
  // silu(g) * u [M, N].
  const __nv_bfloat16* aux;
  int ld_aux;
  __nv_bfloat16* aux_out;
  int ld_aux_out;
  // LM head + cross-entropy (B is this rank's slice of the vocabulary, K-major):
  // kEpiCEStats writes, per row and N tile, the tile's max logit and
  // sum(exp(logit - max)) to ce_stats[row * n_tiles + tile], and the logit of
  // the row's label to ce_tgt[row] when the label falls in the tile;
  // kEpiCEGrad writes (softmax - onehot) * ce_scale in bf16 to C (zero on
  // rows without a label), from the row's log-sum-exp ce_lse[row].
  // Labels are global token ids (-1 = none); column n of this GEMM is token
  // ce_v0 + n.
  const int64_t* ce_labels;
  int64_t ce_v0;
  float2* ce_stats;
  int ce_ld;              // row pitch of ce_stats (float2 elements)
  float* ce_tgt;
  const float* ce_lse;
  float ce_scale;
  PushArgs push;          // kEpiPushRows only
  // kEpiF32T: C is [N, M] fp32 (the transposed product; columns >= N skipped).
  // kEpiLoraBt: the product is [M = output features, N = P * R]; row m keeps
  // only the R columns of its own projection p(m) (p = 0 below bt_b1, 1 below
  // bt_b2, else 2; or alternating 64-column blocks when bt_interleave) and
  // stores them scaled by bt_scale into C[j, m] (C is [R, M] fp32).
  int bt_r, bt_b1, bt_b2, bt_interleave;
  float bt_scale;
};

// Work unit = (M tile, N tile, K split); M fastest, then N, then split.
struct Tile {
  int mt, nt, ks, kb_lo, n_main;
  uint32_t slots;
};

__device__ __forceinline__ Tile decode_tile(int t, const GemmArgs& a, int m_tiles, int n_tiles, int kb_main) {
  Tile r;
  const int mn = m_tiles * n_tiles;
  r.ks = t / mn;
  const int rem = t - r.ks * mn;
  r.mt = rem % m_tiles;
  r.nt = rem / m_tiles;
  const int per = (kb_main + a.k_splits - 1) / a.k_splits;
  r.kb_lo = r.ks * per;
  r.n_main = min(kb_main, r.kb_lo + per) - r.kb_lo;
  // LoRA expand blocks ride with the last split only.
  r.slots = 0u;
  if (a.lora_seg > 0 && r.ks == a.k_splits - 1) {
    if (a.slot_or > 0) {
      for (int i = 0; i < a.slot_or; ++i) r.slots |= a.tile_slots[i];
    } else {
      r.slots = a.tile_slots[r.mt];
    }
  }
  return r;
}

constexpr int BM = 128;
constexpr int BK = 64;

template <int BN, bool B_MN>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 256) ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STAGING = 4 * 2048;  // epilogue: 2 KB per epilogue warp (32 rows x 64 B)
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + STAGING;
};

__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const float* v, int n_valid) {
  // 32 values -> bf16; vector path when all 32 columns are in range and 16B aligned.
  if (n_valid >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
    uint32_t packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      packed[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
  } else {
    for (int i = 0; i < 32 && i < n_valid; ++i) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

__device__ __forceinline__ void store_row_f32(float* dst, const float* v, int n_valid, bool accum) {
  if (!accum && n_valid >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    for (int i = 0; i < 32 && i < n_valid; ++i) dst[i] = accum ? dst[i] + v[i] : v[i];
  }
}

// ---------------------------------------------------------------- fused all-reduce
// Epilogue side (warps 4-7, one output row per thread): the tile's bf16
// partial goes straight into the owner's receive slot over NVLink, then one
// thread bumps the owner's arrival counter with release semantics. With
// split-K the splits first meet in the fp32 workspace and the last split to
// arrive (atomic ticket) sums them and pushes.
// Write 32 rows x 32 columns (this warp's rows, columns c..c+31 of the
// tile) to the owner's receive tile: each lane puts its row into the warp's
// 2 KB staging area, then the warp stores row segments so that every store
// instruction writes eight full 64-byte row pieces (whole sectors over
// NVLink instead of 16-byte fragments of 32 different rows).
template <int BN>
__device__ __forceinline__ void push_rows_32x32(uint4* stg, const float* v, __nv_bfloat16* tile_base, int q,
                                                int lane, int c, int rows_valid) {
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    pk[i] = *reinterpret_cast<uint32_t*>(&h);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k)
    stg[lane * 4 + (k ^ (lane & 3))] = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2), ch = lane & 3;
    const uint4 val = stg[r * 4 + (ch ^ (r & 3))];
    if (q * 32 + r < rows_valid)
      *reinterpret_cast<uint4*>(tile_base + (size_t)(q * 32 + r) * BN + c + ch * 8) = val;
  }
  __syncwarp();
}

template <int BN>
__device__ __forceinline__ void peer_push_tile(const GemmArgs& args, const Tile& tl, uint32_t t_row, int row,
                                               bool row_ok, bool acc_ok, int q, int lane, int m_tiles,
                                               uint4* stg) {
  __shared__ int s_last;
  const PeerArgs& P = args.peer;
  const int L = tl.nt * m_tiles + tl.mt;
  const int owner = L % P.world, local = L / P.world;
  const int n0 = tl.nt * BN;
  const int rows_valid = min(BM, args.M - tl.mt * BM);
  __nv_bfloat16* tile_base = P.recv[owner] + ((size_t)P.rank * P.owned_cap + local) * (BM * BN);
  bool push = true;
  if (args.k_splits > 1) {
#pragma unroll 1
    for (int c = 0; c < BN && acc_ok; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      if (row_ok) store_row_f32(args.partial + ((size_t)tl.ks * args.M + row) * args.N + n0 + c, v, 32, false);
    }
    named_bar_sync(1, 128);
    if (q == 0 && lane == 0) {
      __threadfence();
      const unsigned old = atomicAdd(P.tile_cnt + L, 1u);
      s_last = (old == (unsigned)(args.k_splits - 1)) ? 1 : 0;
      if (s_last) P.tile_cnt[L] = 0u;   // ticket reset for the next call
      __threadfence();
    }
    named_bar_sync(1, 128);
    push = s_last != 0;
    if (push) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
        if (row_ok) {
          for (int sp = 0; sp < args.k_splits; ++sp) {
            const float4* src =
                reinterpret_cast<const float4*>(args.partial + ((size_t)sp * args.M + row) * args.N + n0 + c);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 f = __ldcg(src + i);
              v[4 * i] += f.x;
              v[4 * i + 1] += f.y;
              v[4 * i + 2] += f.z;
              v[4 * i + 3] += f.w;
            }
          }
        }
        push_rows_32x32<BN>(stg, v, tile_base, q, lane, c, rows_valid);
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN && acc_ok; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      push_rows_32x32<BN>(stg, v, tile_base, q, lane, c, rows_valid);
    }
  }
  named_bar_sync(1, 128);
  if (push && q == 0 && lane == 0) {
    __threadfence_system();
    red_release_sys_add(P.rflag[owner] + local, 1u);
  }
}

// Reducer CTAs (all 256 threads), running next to the GEMM CTAs of the same
// launch: as each owned tile's partials arrive from every rank, sum them from
// local memory and write the bf16 result into every rank's output (P2P
// stores), flag each rank; then wait until every output tile of this rank has
// been delivered by its owner. Phases never wait on work of the
// same phase, and the grid fits on the GPU next to the other streams' NCCL
// kernels (every CTA can be resident), so the cross-rank waits cannot
// deadlock; each wait is bounded.
// The owned tiles' partials stream into shared memory with 1-D bulk copies
// (this GPU's own receive buffer: plain cp.async.bulk, no multicast), in
// row chunks of world x rc x BN bf16 (<= 64 KB), double-buffered so the copy
// of the next chunk overlaps the sum and P2P broadcast of this one.
template <int BN>
__device__ __forceinline__ void peer_reducer(const GemmArgs& args, int m_tiles, int n_tiles, int rid, int nr,
                                             uint8_t* smem) {
  const PeerArgs& P = args.peer;
  const int T = m_tiles * n_tiles;
  const int n_owned = (T - P.rank + P.world - 1) / P.world;
  constexpr int VPR = BN / 8;  // 16-byte vectors per tile row
  const size_t slot_stride = (size_t)P.owned_cap * BM * BN;
  const int rc = min(BM, (32768 / (BN * 2) * 2) / P.world);   // rows per chunk: world*rc*BN*2 <= 64 KB
  const int chunks = BM / rc;
  const uint32_t slot_bytes = (uint32_t)(rc * BN * 2);
  const int buf_bytes = P.world * (int)slot_bytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * buf_bytes);  // [2]
  fence_proxy_async_smem();
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  const int my_tiles = rid < n_owned ? (n_owned - rid + nr - 1) / nr : 0;
  const int items = my_tiles * chunks;
  // Thread 0 issues item i (this CTA's tile i / chunks, row chunk i % chunks)
  // into buffer i & 1. The first chunk of a tile needs the tile's partials
  // from every rank: without `block` it only issues when they are there.
  auto issue = [&](int i, bool block) -> bool {
    const int j = rid + (i / chunks) * nr, c = i % chunks;
    if (c == 0) {
      if (!block && ld_acquire_sys(P.rflag[P.rank] + j) < (uint32_t)P.world) return false;
      wait_flag_geq(P.rflag[P.rank] + j, (uint32_t)P.world);
      st_relaxed_sys(P.rflag[P.rank] + j, 0u);
    }
    uint8_t* dst = smem + (i & 1) * buf_bytes;
    fence_proxy_async_smem();  // the buffer's last generic reads come before the copy into it
    mbar_arrive_expect_tx(&bar[i & 1], (uint32_t)buf_bytes);
    const __nv_bfloat16* src = P.recv[P.rank] + (size_t)j * BM * BN + (size_t)c * rc * BN;
    for (int sl = 0; sl < P.world; ++sl)
      bulk_load_1d(dst + sl * slot_bytes, src + sl * slot_stride, slot_bytes, &bar[i & 1]);
    return true;
  };
  int issued = 0;  // thread 0's count of issued items
  if (threadIdx.x == 0 && items > 0) issued = issue(0, true) ? 1 : 0;
  bool ok = true;
  int waited = 0;
  for (int i = 0; i < items && ok; ++i) {
    // Prefetch the next chunk while this one is summed, if its data is ready.
    if (threadIdx.x == 0 && issued == i + 1 && i + 1 < items && issue(i + 1, false)) issued = i + 2;
    ok = mbar_wait(&bar[i & 1], (uint32_t)((i >> 1) & 1), kErrWaitPeer);
    if (!ok) break;
    waited = i + 1;
    const int j = rid + (i / chunks) * nr, c = i % chunks;
    const int L = j * P.world + P.rank;
    const int mt = L % m_tiles, nt = L / m_tiles;
    const int m0 = mt * BM + c * rc, n0 = nt * BN;
    const int rows = max(0, min(rc, args.M - m0));
    const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(smem + (i & 1) * buf_bytes);
    for (int e = threadIdx.x; e < rows * VPR; e += blockDim.x) {
      const int r = e / VPR, c8 = (e - r * VPR) * 8;
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
      for (int sl = 0; sl < P.world; ++sl) {
        const uint4 u = *reinterpret_cast<const uint4*>(sb + sl * (slot_bytes / 2) + r * BN + c8);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(h[k]);
          acc[2 * k] += f.x;
          acc[2 * k + 1] += f.y;
        }
      }
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __nv_bfloat162 h2 = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
        ow[k] = *reinterpret_cast<uint32_t*>(&h2);
      }
      const size_t off = (size_t)(m0 + r) * P.ldo + n0 + c8;
      for (int d = 0; d < P.world; ++d) {
        const int dr = (P.rank + d) % P.world;  // stagger the peers
        *reinterpret_cast<uint4*>(P.out[dr] + off) = o;
      }
    }
    __syncthreads();  // buffer i & 1 is free again; every store of this chunk issued
    if (c == chunks - 1 && threadIdx.x < P.world) {
      __threadfence_system();
      st_release_sys(P.fflag[threadIdx.x] + L, 1u);
    }
    // Not prefetched (its partials were still on the way): issue it now.
    if (threadIdx.x == 0 && issued == i + 1 && i + 1 < items) issued = issue(i + 1, true) ? i + 2 : issued;
  }
  // Copies of this GPU's own memory always land: wait for any still in flight
  // (bounded, ignoring other CTAs' errors) before shared memory is released.
  if (threadIdx.x == 0) {
    for (int i = waited; i < issued; ++i) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&bar[i & 1], (uint32_t)((i >> 1) & 1))) {
        if (globaltimer_ns() - t0 > kWaitNs) {
          set_error(kErrWaitPeer);
          break;
        }
      }
    }
  }
  __syncthreads();
  for (int L = rid; L < T; L += nr) {
    if (threadIdx.x == 0) {
      wait_flag_geq(P.fflag[P.rank] + L, 1u);
      st_relaxed_sys(P.fflag[P.rank] + L, 0u);
    }
  }
}

// Row push (kEpiPushRows): the 128 x BN tile's bf16 partial goes to the row
// block's owner rank (P2P stores through the warp's staging area, as in
// push_rows_32x32, with the receive rows `ld` elements apart), then one
// thread publishes the tile's column count on the owner's block counter.
// Every epilogue warp of the CTA calls this for every tile (also after a
// failed accumulator wait, with the TMEM reads skipped), so the four warps
// always meet at the named barrier.
__device__ __forceinline__ void push_rows_pitch(uint4* stg, const float* v, __nv_bfloat16* tile_base, int ld, int q,
                                                int lane, int c, int rows_valid) {
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    pk[i] = *reinterpret_cast<uint32_t*>(&h);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k)
    stg[lane * 4 + (k ^ (lane & 3))] = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2), ch = lane & 3;
    const uint4 val = stg[r * 4 + (ch ^ (r & 3))];
    if (q * 32 + r < rows_valid)
      *reinterpret_cast<uint4*>(tile_base + (size_t)(q * 32 + r) * ld + c + ch * 8) = val;
  }
  __syncwarp();
}

template <int BN>
__device__ __forceinline__ void push_rows_tile(const GemmArgs& args, uint32_t t_row, int mt128, int n0, int q,
                                               int lane, bool acc_ok, uint4* stg) {
  const PushArgs& P = args.push;
  const int owner = mt128 % P.world, local = mt128 / P.world;
  const int rows_valid = min(BM, args.M - mt128 * BM);   // <= 0: a pair CTA past the last row
  const int row = mt128 * BM + q * 32 + lane;
  __nv_bfloat16* base = P.recv[owner] + (size_t)(P.rank * P.blocks_cap + local) * BM * P.ld + n0;
#pragma unroll 1
  for (int c = 0; c < BN && acc_ok && rows_valid > 0; c += 32) {
    if (n0 + c >= args.N) break;
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c, r);
    tmem_ld_wait();
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    if (P.add != nullptr && row < args.M) {
      const float4* a4 = reinterpret_cast<const float4*>(P.add + (size_t)row * P.ld_add + n0 + c);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 f = a4[i];
        v[4 * i] += f.x;
        v[4 * i + 1] += f.y;
        v[4 * i + 2] += f.z;
        v[4 * i + 3] += f.w;
      }
    }
    push_rows_pitch(stg, v, base, P.ld, q, lane, c, rows_valid);
  }
  named_bar_sync(1, 128);
  if (q == 0 && lane == 0 && acc_ok && rows_valid > 0) {
    __threadfence_system();
    red_release_sys_add(P.cnt[owner] + local, (uint32_t)min(BN, args.N - n0));
  }
}

// Epilogue of one tile row for the plain store kinds (bf16 / fp32 /
// fp32-accumulate, or SwiGLU over 64-interleaved gate/up columns), plus the
// optional raw-row capture: this thread's TMEM lane `t_row` holds output row
// `row`, columns n0 .. n0 + BN. Shared by the 1-CTA and 2-CTA kernels.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_rows(const GemmArgs& args, uint32_t t_row, int row, bool row_ok, int n0,
                                              bool do_save) {
  if constexpr (EPI == kEpiSwiGLUBwd) {
    // 32 d(act) columns at a time, all inside one 64-column block of the
    // interleave: their gate columns start at (col / 64) * 128 + col % 64,
    // the up columns 64 further.
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      const int col = n0 + c;
      if (!row_ok || col >= args.N) continue;
      const int gcol = (col >> 6) * 128 + (col & 63);
      const uint4* gp = reinterpret_cast<const uint4*>(args.aux + (size_t)row * args.ld_aux + gcol);
      const uint4* up = reinterpret_cast<const uint4*>(args.aux + (size_t)row * args.ld_aux + gcol + 64);
      float dg[32], du[32], act[32];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint4 gq = gp[v], uq = up[v];
        const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gq);
        const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&uq);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int i = v * 8 + e;
          const float g = bf2f(gb[e]), u = bf2f(ub[e]);
          const float da = __uint_as_float(r[i]);
          const float sg = 1.f / (1.f + __expf(-g));
          const float silu = g * sg;
          dg[i] = da * u * sg * (1.f + g * (1.f - sg));
          du[i] = da * silu;
          act[i] = silu * u;
        }
      }
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc + gcol;
      store_row_bf16(dst, dg, 32);
      store_row_bf16(dst + 64, du, 32);
      if (args.aux_out != nullptr) store_row_bf16(args.aux_out + (size_t)row * args.ld_aux_out + col, act, 32);
    }
  } else if constexpr (EPI == kEpiSwiGLU) {
    // Columns come interleaved in blocks of 64: [gate(64) | up(64)] per 128.
#pragma unroll 1
    for (int c = 0; c < BN; c += 128) {
#pragma unroll 1
      for (int h = 0; h < 64; h += 32) {
        uint32_t g[32], u[32];
        tmem_ld_32x32b_x32(t_row + c + h, g);
        tmem_ld_32x32b_x32(t_row + c + 64 + h, u);
        tmem_ld_wait();
        float o[32], gf[32], uf[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          gf[i] = __uint_as_float(g[i]);
          uf[i] = __uint_as_float(u[i]);
          float sg = gf[i] / (1.0f + __expf(-gf[i]));
          o[i] = sg * uf[i];
        }
        const int gcol = n0 + c;  // first gate column of this 128 block
        if (row_ok && gcol < args.N) {
          const int ocol = gcol / 2 + h;
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc + ocol;
          store_row_bf16(dst, o, min(32, args.N / 2 - ocol));
          if (do_save) {
            __nv_bfloat16* sv = args.save + (size_t)(row - args.save_lo + args.save_dst) * args.ld_save;
            store_row_bf16(sv + gcol + h, gf, min(32, args.N - (gcol + h)));
            store_row_bf16(sv + gcol + 64 + h, uf, min(32, args.N - (gcol + 64 + h)));
          }
        }
      }
    }
  } else if constexpr (EPI == kEpiF32T) {
    float* Cf = reinterpret_cast<float*>(args.C);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      if (!row_ok) continue;
#pragma unroll 8
      for (int i = 0; i < 32; ++i) {
        const int col = n0 + c + i;
        if (col < args.N) Cf[(size_t)col * args.ldc + row] = __uint_as_float(r[i]);
      }
    }
  } else if constexpr (EPI == kEpiLoraBt) {
    float* Cf = reinterpret_cast<float*>(args.C);
    const int R = args.bt_r;
    const int p = args.bt_interleave ? ((row >> 6) & 1) : (row < args.bt_b1 ? 0 : (row < args.bt_b2 ? 1 : 2));
    const int lo = p * R;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      if (!row_ok) continue;
#pragma unroll 8
      for (int i = 0; i < 32; ++i) {
        const int j = n0 + c + i - lo;
        if (j >= 0 && j < R) Cf[(size_t)j * args.ldc + row] = args.bt_scale * __uint_as_float(r[i]);
      }
    }
  } else if constexpr (EPI == kEpiCEStats) {
    // Online max / sum-exp over this tile's columns (32 at a time), and the
    // label's logit when the label falls in the tile.
    int lab = -1;
    if (row_ok) {
      const int64_t g = args.ce_labels[row];
      const int64_t L = g - args.ce_v0;
      if (g >= 0 && L >= n0 && L < n0 + BN && L < args.N) lab = (int)(L - n0);
    }
    float m = -INFINITY, ssum = 0.f, tv = 0.f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      const int nv = min(32, args.N - (n0 + c));   // the same for every lane
      if (nv <= 0) continue;
      float cm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) cm = fmaxf(cm, __uint_as_float(r[i]));
      const float mn = fmaxf(m, cm);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) acc += __expf(__uint_as_float(r[i]) - mn);
      ssum = ssum * __expf(m - mn) + acc;
      m = mn;
      if (lab >= c && lab < c + 32) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i == lab - c) tv = __uint_as_float(r[i]);
      }
    }
    if (row_ok) {
      args.ce_stats[(size_t)row * args.ce_ld + n0 / BN] = make_float2(m, ssum);
      if (lab >= 0) args.ce_tgt[row] = tv;
    }
  } else if constexpr (EPI == kEpiCEGrad) {
    // d(loss)/d(logit) = (softmax - onehot) / n_valid, recomputed from the
    // row's log-sum-exp; rows without a label get zeros.
    int lab = -1;
    float lse = 0.f, sc = 0.f;
    if (row_ok) {
      const int64_t g = args.ce_labels[row];
      if (g >= 0) {
        sc = args.ce_scale;
        lse = args.ce_lse[row];
        const int64_t L = g - args.ce_v0;
        if (L >= 0 && L < args.N) lab = (int)L;
      }
    }
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      const int col = n0 + c;
      if (!row_ok || col >= args.N) continue;
      float v[32];
      if (sc != 0.f) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          v[i] = (__expf(__uint_as_float(r[i]) - lse) - (col + i == lab ? 1.f : 0.f)) * sc;
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      store_row_bf16(reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc + col, v,
                     min(32, args.N - col));
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c, r);
      tmem_ld_wait();
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      const int col = n0 + c;
      if (row_ok && col < args.N) {
        const int nv = min(32, args.N - col);
        if constexpr (EPI == kEpiBF16) {
          store_row_bf16(reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc + col, v, nv);
        } else {
          store_row_f32(reinterpret_cast<float*>(args.C) + (size_t)row * args.ldc + col, v, nv,
                        EPI == kEpiF32Accum);
        }
        if (do_save) {
          store_row_bf16(args.save + (size_t)(row - args.save_lo + args.save_dst) * args.ld_save + col, v, nv);
        }
      }
    }
  }
}

template <int BN, bool B_MN, int EPI>
__global__ void __launch_bounds__(256, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmZ, const __grid_constant__ CUtensorMap tmB2, GemmArgs args) {
  using Cfg = GemmCfg<BN, B_MN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;  // [2]
  uint64_t* acce_bar = accf_bar + 2;        // [2]
  uint64_t* drain_bar = acce_bar + 2;       // [1]
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(drain_bar + 1);
  uint4* staging = reinterpret_cast<uint4*>(smem + STAGES * Cfg::STAGE_BYTES + 256);  // [4 warps][2 KB]

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m_tiles = (args.M + BM - 1) / BM;
  const int num_n_tiles = (args.N + BN - 1) / BN;
  const int num_tiles = num_m_tiles * num_n_tiles * args.k_splits;
  const int kb_main = (args.K + BK - 1) / BK;
  const int kb_per_slot = args.lora_seg / BK;
  // Work split of the persistent grid: with the fused all-reduce the first
  // `reducers` CTAs only reduce / broadcast (no TMEM, no pipeline).
  int cta0 = blockIdx.x, ncta = gridDim.x;
  if constexpr (EPI == kEpiPeerAR) {
    if ((int)blockIdx.x < args.peer.reducers) {
      peer_reducer<BN>(args, num_m_tiles, num_n_tiles, blockIdx.x, args.peer.reducers, smem);
      return;
    }
    cta0 -= args.peer.reducers;
    ncta -= args.peer.reducers;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 4);
    }
    mbar_init(drain_bar, 1);
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(tmem_base_smem, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.ag_maps != nullptr)
      for (int r = 0; r < args.ag_world; ++r) tma_prefetch_desc(&args.ag_maps[r]);
    if (args.lora_seg > 0) {
      tma_prefetch_desc(&tmZ);
      tma_prefetch_desc(&tmB2);
    }
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int fills[STAGES > 0 ? STAGES : 1];
    for (int s = 0; s < STAGES; ++s) fills[s] = 0;
    bool dep_done = args.wait_prev == 0;
    for (int t = cta0; t < num_tiles && ok; t += ncta) {
      const Tile tl = decode_tile(t, args, num_m_tiles, num_n_tiles, kb_main);
      const int m0 = tl.mt * BM, n0 = tl.nt * BN;
      const uint32_t slots = tl.slots;
      const int n_lora = __popc(slots) * kb_per_slot;
      if (args.ag_gathered != nullptr && m0 / args.ag_rows != args.ag_rank) {
        // A remote row block: wait until every unit of it is in the gathered buffer.
        const uint64_t t0 = globaltimer_ns();
        uint32_t n = 0;
        while (ld_acquire_gpu(&args.ag_cnt[tl.mt]) < args.ag_expect) {
          if ((++n & 255u) == 0 && globaltimer_ns() - t0 > kWaitNs) { set_error(kErrWaitGather); ok = false; break; }
        }
        if (!ok) break;
        fence_proxy_async_global();     // the copies (generic stores) before this thread's TMA reads
      }
      for (int j = 0; j < tl.n_main + n_lora; ++j) {
        if (j == tl.n_main && !dep_done) {
          griddep_wait();
          dep_done = true;
        }
        if (!mbar_wait(&empty_bar[stage], phase ^ 1, kErrWaitEmpty)) { ok = false; break; }
        uint8_t* sA = smem + stage * Cfg::STAGE_BYTES;
        uint8_t* sB = sA + Cfg::A_BYTES;
        mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
        if (j < tl.n_main) {
          const int k0 = (tl.kb_lo + j) * BK;
          if constexpr (a_mn_major<EPI>()) {
#pragma unroll
            for (int jj = 0; jj < BM / 64; ++jj) tma_load_2d(sA + jj * (64 * BK * 2), &tmA, &full_bar[stage], m0 + jj * 64, k0);
          } else {
            if (args.ag_maps != nullptr && m0 / args.ag_rows == args.ag_rank)
              tma_load_2d(sA, &args.ag_maps[args.ag_rank], &full_bar[stage], k0, m0 % args.ag_rows);
            else if (args.ag_maps != nullptr && args.ag_gathered == nullptr)   // straight from the owner
              tma_load_2d(sA, &args.ag_maps[m0 / args.ag_rows], &full_bar[stage], k0, m0 % args.ag_rows);
            else
              tma_load_2d(sA, &tmA, &full_bar[stage], k0, m0);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sB + j * (64 * BK * 2), &tmB, &full_bar[stage], n0 + j * 64, k0);
          } else {
            tma_load_2d(sB, &tmB, &full_bar[stage], k0, n0);
          }
        } else {
          // LoRA expand block: the (lb / kb_per_slot)-th present slot.
          int lb = j - tl.n_main;
          int which = lb / kb_per_slot, sub = lb % kb_per_slot;
          uint32_t m = slots;
          for (int i = 0; i < which; ++i) m &= m - 1;
          const int slot = __ffs(m) - 1;
          const int k0 = slot * args.lora_seg + sub * BK;
          tma_load_2d(sA, &tmZ, &full_bar[stage], k0, m0);
          if constexpr (B_MN) {
            // MN-major launch: B2 is [S*SEG, N] like B (the backward's dX += dZ . A).
#pragma unroll
            for (int jj = 0; jj < BN / 64; ++jj)
              tma_load_2d(sB + jj * (64 * BK * 2), &tmB2, &full_bar[stage], n0 + jj * 64, k0);
          } else {
            tma_load_2d(sB, &tmB2, &full_bar[stage], k0, n0);
          }
        }
        fills[stage]++;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    if (!dep_done) griddep_wait();
    // Drain: every copy this thread issued has landed before the CTA can exit.
    for (int s = 0; s < STAGES; ++s) {
      if (fills[s] == 0) continue;
      uint32_t par = (uint32_t)((fills[s] - 1) & 1);
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full_bar[s], par)) {
        if (globaltimer_ns() - t0 > kWaitNs) { set_error(kErrWaitFull); break; }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, a_mn_major<EPI>(), B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int iter = 0;
    bool ok = true;
    for (int t = cta0; t < num_tiles && ok; t += ncta, ++iter) {
      const Tile tl = decode_tile(t, args, num_m_tiles, num_n_tiles, kb_main);
      const int n_kb = tl.n_main + __popc(tl.slots) * kb_per_slot;
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1, kErrWaitAccEmpty)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < n_kb; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, kErrWaitFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + stage * Cfg::STAGE_BYTES);
        const uint32_t b_addr = a_addr + Cfg::A_BYTES;
        const bool lora_blk = kb >= tl.n_main;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t da = a_mn_major<EPI>() ? smem_desc(a_addr + k * 16 * 128, 64 * BK * 2, 1024, kSwizzle128B)
                                                : smem_desc(a_addr + k * 32, 16, 1024, kSwizzle128B);
          uint64_t db;
          (void)lora_blk;
          if (B_MN) {
            db = smem_desc(b_addr + k * 16 * 128, 64 * BK * 2, 1024, kSwizzle128B);
          } else {
            db = smem_desc(b_addr + k * 32, 16, 1024, kSwizzle128B);
          }
          tc_mma_f16(d_tmem, da, db, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
        }
        tc_commit(&empty_bar[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      tc_commit(&accf_bar[acc]);
    }
    // Every MMA issued by this thread has finished before TMEM is freed.
    tc_commit(drain_bar);
    uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(drain_bar, 0)) {
      if (globaltimer_ns() - t0 > kWaitNs) { set_error(kErrWaitAccFull); break; }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int q = warp - 4;  // TMEM lane quarter
    if (args.ag_gathered != nullptr) {
      // Copy-once gather (see GemmArgs::ag_gathered). Units (row block,
      // kAgChunk columns) are claimed from a ticket counter, so only CTAs that
      // are running copy and a producer never waits on a CTA that has not
      // started; a later launch over the same rows (ticket past the end)
      // copies nothing. Within a unit, 32 lanes cover 512 contiguous bytes of
      // a row, eight 16-byte loads in flight per thread.
      const int e = threadIdx.x - 128;
      const int chunks = (args.K + kAgChunk - 1) / kAgChunk;
      const int units = num_m_tiles * chunks;
      __shared__ int ag_unit;
      for (;;) {
        if (e == 0) ag_unit = (int)atomicAdd(args.ag_ticket, 1u);
        named_bar_sync(1, 128);
        const int u = ag_unit;
        named_bar_sync(1, 128);
        if (u >= units || u < 0) break;
        const int blk = u / chunks, ch = u - blk * chunks;
        const int owner = blk * BM / args.ag_rows;
        if (owner == args.ag_rank) continue;                         // own rows are read in place
        const int c0 = ch * kAgChunk;
        const int n16 = (min(args.K, c0 + kAgChunk) - c0) / 8;      // 16-byte vectors per row
        const int total = min(BM, args.M - blk * BM) * n16;
        const __nv_bfloat16* sbase = args.ag_src[owner] + (size_t)(blk * BM % args.ag_rows) * args.K + c0;
        __nv_bfloat16* dbase = args.ag_gathered + (size_t)blk * BM * args.K + c0;
        for (int i0 = e; i0 < total; i0 += 128 * 8) {
          uint4 v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int i = i0 + k * 128;
            if (i < total) {
              const int r = i / n16, c = i - r * n16;
              v[k] = *reinterpret_cast<const uint4*>(sbase + (size_t)r * args.K + c * 8);
            }
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int i = i0 + k * 128;
            if (i < total) {
              const int r = i / n16, c = i - r * n16;
              *reinterpret_cast<uint4*>(dbase + (size_t)r * args.K + c * 8) = v[k];
            }
          }
        }
        fence_proxy_async_global();        // this thread's stores before the consumers' TMA reads
        named_bar_sync(1, 128);            // the four epilogue warps' copies of the unit
        if (e == 0) {
          __threadfence();
          red_release_gpu_add(&args.ag_cnt[blk], 1u);
        }
      }
    }
    int iter = 0;
    for (int t = cta0; t < num_tiles; t += ncta, ++iter) {
      const Tile tl = decode_tile(t, args, num_m_tiles, num_n_tiles, kb_main);
      const int m0 = tl.mt * BM, n0 = tl.nt * BN;
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      bool acc_ok = __all_sync(0xffffffffu, mbar_wait(&accf_bar[acc], acc_phase, kErrWaitAccFull));
      // The fused all-reduce's epilogue warps meet at named barriers: they keep
      // iterating after a failed wait (TMEM reads skipped) so they always meet.
      if (EPI != kEpiPeerAR && EPI != kEpiPushRows && !acc_ok) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < args.M;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      const bool do_save = args.save != nullptr && row_ok && row >= args.save_lo && row < args.save_hi;
      if constexpr (EPI == kEpiPeerAR) {
        // Keeps iterating after a failed wait (with the TMEM reads skipped) so
        // the four epilogue warps always meet at their named barriers.
        peer_push_tile<BN>(args, tl, t_row, row, row_ok && acc_ok, acc_ok, q, lane, num_m_tiles,
                           staging + q * 128);
      } else if constexpr (EPI == kEpiPushRows) {
        push_rows_tile<BN>(args, t_row, tl.mt, n0, q, lane, acc_ok, staging + q * 128);
      } else if (args.k_splits > 1) {
        // Split-K: raw fp32 partial sums; the reduce kernel applies the epilogue.
#pragma unroll 1
        for (int c = 0; c < BN && acc_ok; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c, r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          const int col = n0 + c;
          if (row_ok && col < args.N)
            store_row_f32(args.partial + ((size_t)tl.ks * args.M + row) * args.N + col, v,
                          min(32, args.N - col), false);
        }
      } else if constexpr (EPI == kEpiBF16T) {
        // Swapped operands: accumulator rows are output features (this
        // thread's TMEM lane), columns are tokens; C is [tokens, features].
        // A warp writes 32 consecutive features of one token per store.
        __nv_bfloat16* cb = reinterpret_cast<__nv_bfloat16*>(args.C);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c, r);
          tmem_ld_wait();
          if (!row_ok) continue;
#pragma unroll 8
          for (int i = 0; i < 32; ++i) {
            const int tok = n0 + c + i;
            if (tok < args.N) cb[(size_t)tok * args.ldc + row] = f2bf(__uint_as_float(r[i]));
          }
        }
      } else if constexpr (EPI == kEpiShrink) {
        const int srow = row_ok ? args.shrink_slot_ids[row] : -1;
        const int PR = args.shrink_pr, SEG = args.shrink_seg;
        __nv_bfloat16* zr = reinterpret_cast<__nv_bfloat16*>(args.C) + (size_t)row * args.ldc;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c, r);
          tmem_ld_wait();
          if (!row_ok) continue;
#pragma unroll 4
          for (int i = 0; i < 32; ++i) {
            const int cc = n0 + c + i;
            if (cc >= args.N) break;
            const int sl = cc / PR, j = cc - sl * PR;
            zr[sl * SEG + j] = f2bf(sl == srow ? __uint_as_float(r[i]) : 0.f);
            for (int zc = PR + j; zc < SEG; zc += PR) zr[sl * SEG + zc] = f2bf(0.f);
          }
        }
      } else {
        epilogue_rows<BN, EPI>(args, t_row, row, row_ok, n0, do_save);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  if constexpr (EPI == kEpiPeerAR) {
    // No dedicated reducers (one wave of GEMM work): the GEMM CTAs reduce and
    // broadcast the owned tiles themselves once their own tiles are pushed.
    if (args.peer.reducers == 0) peer_reducer<BN>(args, num_m_tiles, num_n_tiles, cta0, ncta, smem);
  }
}

// ---------------------------------------------------------------- CTA-pair GEMM
// Same pipeline as gemm_tc_kernel, on a cluster of two CTAs sharing one
// 256 x BN tile through the pair MMA (tcgen05 cta_group::2): CTA r stages
// rows [r*128, r*128+128) of the A tile and columns [r*BN/2, (r+1)*BN/2) of
// the B tile; the even CTA's MMA thread issues the M=256 MMAs, each CTA's
// TMEM receives its own 128 accumulator rows and its epilogue stores them.
// Per SM, shared-memory traffic per MMA drops from A+B to A+B/2, which is
// what limits the single-CTA 128 x 256 tile.
//
// Barriers: the even CTA's full[s] counts the bytes of both CTAs' TMA loads
// (each load signals it through its shared::cluster address); the MMA
// commit releases empty[s] in both CTAs and signals both CTAs' accf[a];
// both CTAs' epilogue warps arrive on the even CTA's acce[a] (count 8).
// Every wait is bounded; every thread reaches the final cluster barrier.
template <int BN, bool B_MN>
struct GemmCfgPair {
  static constexpr int A_BYTES = BM * BK * 2;          // this CTA's 128 rows
  static constexpr int B_BYTES = (BN / 2) * BK * 2;    // this CTA's BN/2 columns
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 256) ? 6 : 8;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STAGING = 4 * 2048;  // push epilogue: 2 KB per epilogue warp
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + STAGING;
};

template <int BN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmZ, const __grid_constant__ CUtensorMap tmB2,
                        GemmArgs args) {
  static_assert(EPI == kEpiBF16 || EPI == kEpiF32 || EPI == kEpiF32Accum || EPI == kEpiSwiGLU ||
                    EPI == kEpiCEStats || EPI == kEpiCEGrad || EPI == kEpiPushRows || EPI == kEpiSwiGLUBwd,
                "pair GEMM: row-wise epilogues only");
  using Cfg = GemmCfgPair<BN, B_MN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;  // [2]
  uint64_t* acce_bar = accf_bar + 2;        // [2] (used in the even CTA)
  uint64_t* drain_bar = acce_bar + 2;       // [1]
  uint64_t* exit_bar = drain_bar + 1;       // [1] the peer CTA is done with the pair
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(exit_bar + 1);
  uint4* staging = reinterpret_cast<uint4*>(smem + STAGES * Cfg::STAGE_BYTES + 256);  // [4 warps][2 KB]

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();  // 0 = MMA-issuing CTA
  const int num_m128 = (args.M + BM - 1) / BM;
  const int num_m_tiles = (args.M + 2 * BM - 1) / (2 * BM);
  const int num_n_tiles = (args.N + BN - 1) / BN;
  const int num_tiles = num_m_tiles * num_n_tiles;
  const int kb_main = (args.K + BK - 1) / BK;
  const int kb_per_slot = args.lora_seg / BK;
  const int pair0 = blockIdx.x / 2, npairs = gridDim.x / 2;
  // LoRA slots of a 256-row tile: both of its 128-row halves.
  auto tile_slots_of = [&](int mt) -> uint32_t {
    if (args.lora_seg <= 0) return 0u;
    uint32_t m = args.tile_slots[2 * mt];
    if (2 * mt + 1 < num_m128) m |= args.tile_slots[2 * mt + 1];
    return m;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 8);
    }
    mbar_init(drain_bar, 1);
    mbar_init(exit_bar, 1);
    fence_mbarrier_init_cluster();
  }
  // Both CTAs' barriers are initialised before any remote arrive; nothing
  // that can block precedes this barrier.
  cluster_sync_all();
  if (warp == 2) tmem_alloc_pair(tmem_base_smem, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.lora_seg > 0) {
      tma_prefetch_desc(&tmZ);
      tma_prefetch_desc(&tmB2);
    }
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int fills[STAGES];
    for (int s = 0; s < STAGES; ++s) fills[s] = 0;
    bool dep_done = args.wait_prev == 0;
    for (int t = pair0; t < num_tiles && ok; t += npairs) {
      const int mt = t % num_m_tiles, nt = t / num_m_tiles;
      const int m0 = mt * 2 * BM + (int)rank * BM;
      const int nb0 = nt * BN + (int)rank * (BN / 2);
      const uint32_t slots = tile_slots_of(mt);
      const int n_lora = __popc(slots) * kb_per_slot;
      for (int j = 0; j < kb_main + n_lora; ++j) {
        if (j == kb_main && !dep_done) {
          griddep_wait();
          dep_done = true;
        }
        if (!mbar_wait(&empty_bar[stage], phase ^ 1, kErrWaitEmpty)) { ok = false; break; }
        uint8_t* sA = smem + stage * Cfg::STAGE_BYTES;
        uint8_t* sB = sA + Cfg::A_BYTES;
        if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
        const uint32_t bar = mapa_shared(smem_u32(&full_bar[stage]), 0);
        if (j < kb_main) {
          const int k0 = j * BK;
          tma_load_2d_pair(sA, &tmA, bar, k0, m0);
          if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 128; ++c) tma_load_2d_pair(sB + c * (64 * BK * 2), &tmB, bar, nb0 + c * 64, k0);
          } else {
            tma_load_2d_pair(sB, &tmB, bar, k0, nb0);
          }
        } else {
          int lb = j - kb_main;
          int which = lb / kb_per_slot, sub = lb % kb_per_slot;
          uint32_t m = slots;
          for (int i = 0; i < which; ++i) m &= m - 1;
          const int slot = __ffs(m) - 1;
          const int k0 = slot * args.lora_seg + sub * BK;
          tma_load_2d_pair(sA, &tmZ, bar, k0, m0);
          if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 128; ++c) tma_load_2d_pair(sB + c * (64 * BK * 2), &tmB2, bar, nb0 + c * 64, k0);
          } else {
            tma_load_2d_pair(sB, &tmB2, bar, k0, nb0);
          }
        }
        fills[stage]++;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    if (!dep_done) griddep_wait();
    // Drain (even CTA): its full barriers count both CTAs' copies, so once
    // they completed no copy of either CTA is in flight.
    if (rank == 0) {
      for (int s = 0; s < STAGES; ++s) {
        if (fills[s] == 0) continue;
        uint32_t par = (uint32_t)((fills[s] - 1) & 1);
        uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full_bar[s], par)) {
          if (globaltimer_ns() - t0 > kWaitNs) { set_error(kErrWaitFull); break; }
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    constexpr uint32_t IDESC = idesc_bf16_f32(2 * BM, BN, false, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int iter = 0;
    bool ok = true;
    bool issued = false;
    for (int t = pair0; t < num_tiles && ok; t += npairs, ++iter) {
      const int mt = t % num_m_tiles;
      const int n_kb = kb_main + __popc(tile_slots_of(mt)) * kb_per_slot;
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1, kErrWaitAccEmpty)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < n_kb; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, kErrWaitFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + stage * Cfg::STAGE_BYTES);
        const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t da = smem_desc(a_addr + k * 32, 16, 1024, kSwizzle128B);
          const uint64_t db = B_MN ? smem_desc(b_addr + k * 16 * 128, 64 * BK * 2, 1024, kSwizzle128B)
                                   : smem_desc(b_addr + k * 32, 16, 1024, kSwizzle128B);
          tc_mma_f16_pair(d_tmem, da, db, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
        }
        issued = true;
        tc_commit_pair_mc(&empty_bar[stage], (uint16_t)0x3);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      tc_commit_pair_mc(&accf_bar[acc], (uint16_t)0x3);
    }
    // Every pair MMA issued here has finished before either CTA frees TMEM.
    if (issued) {
      tc_commit_pair_mc(drain_bar, (uint16_t)0x1);
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain_bar, 0)) {
        if (globaltimer_ns() - t0 > kWaitNs) { set_error(kErrWaitAccFull); break; }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp - 4;
    const uint32_t acce_leader0 = mapa_shared(smem_u32(&acce_bar[0]), 0);
    int iter = 0;
    for (int t = pair0; t < num_tiles; t += npairs, ++iter) {
      const int mt = t % num_m_tiles, nt = t / num_m_tiles;
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      const bool acc_ok = __all_sync(0xffffffffu, mbar_wait(&accf_bar[acc], acc_phase, kErrWaitAccFull));
      if (EPI != kEpiPushRows && !acc_ok) break;
      tc_fence_after();
      const int row = mt * 2 * BM + (int)rank * BM + q * 32 + lane;
      const bool row_ok = row < args.M;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      const bool do_save = args.save != nullptr && row_ok && row >= args.save_lo && row < args.save_hi;
      if constexpr (EPI == kEpiPushRows) {
        // This CTA's 128 rows are one row block of the push.
        push_rows_tile<BN>(args, t_row, mt * 2 + (int)rank, nt * BN, q, lane, acc_ok, staging + q * 128);
      } else {
        epilogue_rows<BN, EPI>(args, t_row, row, row_ok, nt * BN, do_save);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_leader0 + (uint32_t)(acc * sizeof(uint64_t)));
    }
  }
  // Exit handshake (bounded): each CTA tells its peer it is done with the
  // pair (its MMAs drained / its TMEM reads and copies finished) and waits
  // for the peer's word before freeing TMEM and leaving.
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_cluster(mapa_shared(smem_u32(exit_bar), rank ^ 1u));
    uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(exit_bar, 0)) {
      if (globaltimer_ns() - t0 > kWaitNs) { set_error(kErrWaitPeer); break; }
    }
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
}

// Split-K epilogue: sum the fp32 partials of every split and apply the
// epilogue (bf16 / fp32 / fp32-accumulate store, or SwiGLU over interleaved
// gate/up pairs), plus the optional raw-accumulator row capture.
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N, int epi, void* C,
                                     int ldc, __nv_bfloat16* save, int ld_save, int save_lo, int save_hi,
                                     int save_dst) {
  const size_t plane = (size_t)M * N;
  if (epi == kEpiSwiGLU) {
    const int half = N / 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)M * half;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int row = (int)(i / half), j = (int)(i % half);
      const int cg = (j / 64) * 128 + (j % 64);
      float g = 0.f, u = 0.f;
      for (int s = 0; s < splits; ++s) {
        g += partial[s * plane + (size_t)row * N + cg];
        u += partial[s * plane + (size_t)row * N + cg + 64];
      }
      reinterpret_cast<__nv_bfloat16*>(C)[(size_t)row * ldc + j] = f2bf(g / (1.f + __expf(-g)) * u);
      if (save != nullptr && row >= save_lo && row < save_hi) {
        __nv_bfloat16* sv = save + (size_t)(row - save_lo + save_dst) * ld_save;
        sv[cg] = f2bf(g);
        sv[cg + 64] = f2bf(u);
      }
    }
    return;
  }
  if (epi == kEpiBF16T) {
    // Partials are [features M, tokens N]; C is [tokens, features]: walk it
    // feature-fastest so consecutive threads store consecutive features.
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)plane;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int feat = (int)(i % M), tok = (int)(i / M);
      float v = 0.f;
      for (int s = 0; s < splits; ++s) v += partial[s * plane + (size_t)feat * N + tok];
      reinterpret_cast<__nv_bfloat16*>(C)[(size_t)tok * ldc + feat] = f2bf(v);
    }
    return;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)plane;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / N), col = (int)(i % N);
    float v = 0.f;
    for (int s = 0; s < splits; ++s) v += partial[s * plane + i];
    if (epi == kEpiBF16) reinterpret_cast<__nv_bfloat16*>(C)[(size_t)row * ldc + col] = f2bf(v);
    else if (epi == kEpiF32) reinterpret_cast<float*>(C)[(size_t)row * ldc + col] = v;
    else reinterpret_cast<float*>(C)[(size_t)row * ldc + col] += v;
    if (save != nullptr && row >= save_lo && row < save_hi)
      save[(size_t)(row - save_lo + save_dst) * ld_save + col] = f2bf(v);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "dsv: cannot resolve cuTensorMapEncodeTiled from the CUDA driver");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct TmKey {
  uint64_t ptr, rows, cols, ld;
  uint32_t box_rows;
  bool operator==(const TmKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows;
  }
};
struct TmKeyHash {
  size_t operator()(const TmKey& k) const {
    return std::hash<uint64_t>()(k.ptr) ^ (std::hash<uint64_t>()(k.rows) * 31) ^ (std::hash<uint64_t>()(k.cols) * 131) ^
           (std::hash<uint64_t>()(k.ld) * 1031) ^ (std::hash<uint32_t>()(k.box_rows) * 7);
  }
};

// Tensor map of a row-major bf16 matrix [rows, cols] with leading dimension
// `ld` elements; box = 64 columns (128 bytes, 128-byte swizzle) x box_rows.
// Maps are cached by (pointer, shape, box): weights and the engine's
// persistent activation buffers are encoded once.
CUtensorMap make_tmap_bf16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  static std::unordered_map<TmKey, CUtensorMap, TmKeyHash> cache;
  static std::mutex mu;
  TmKey key{reinterpret_cast<uint64_t>(ptr), rows, cols, ld, box_rows};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "dsv gemm: operand base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "dsv gemm: row pitch must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), gdim, gstride, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "dsv gemm: cuTensorMapEncodeTiled failed (", (int)r, ")");
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, m);
  return m;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Launch with programmatic stream serialization (the kernel may start while
// the previous grid in the stream still runs; it calls griddep_wait first
// where it reads that grid's output).
template <typename Kern>
static void launch_overlapping(Kern kern, dim3 grid, int smem, cudaStream_t stream, const CUtensorMap& a,
                               const CUtensorMap& b, const CUtensorMap& z, const CUtensorMap& b2,
                               const GemmArgs& args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TORCH_CHECK(cudaLaunchKernelEx(&cfg, kern, a, b, z, b2, args) == cudaSuccess, "dsv gemm: overlapping launch failed");
}

template <int BN, bool B_MN, int EPI>
static void launch(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& z, const CUtensorMap& b2,
                   const GemmArgs& args, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, B_MN>;
  auto kern = gemm_tc_kernel<BN, B_MN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    attr_set = true;
  }
  // Work units include the K splits: each split of a tile is its own CTA's work.
  const int tiles = ((args.M + BM - 1) / BM) * ((args.N + BN - 1) / BN) * std::max(1, args.k_splits);
  // Persistent (one CTA per SM) by default; a larger cap makes CTAs retire
  // after one tile so a higher-priority stream can interleave at tile
  // granularity (used for the low-priority backward).
  const int grid = std::min(tiles, args.max_ctas > 0 ? args.max_ctas : num_sms());
  if (args.wait_prev) {
    launch_overlapping(kern, dim3(grid), Cfg::SMEM, stream, a, b, z, b2, args);
  } else {
    kern<<<grid, 256, Cfg::SMEM, stream>>>(a, b, z, b2, args);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// CTA-pair launch (BN = 256): clusters of two CTAs, one 256 x 256 tile per
// pair at a time; persistent unless the grid cap asks for one tile per pair.
template <bool B_MN, int EPI>
static void launch_pair(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& z, const CUtensorMap& b2,
                        const GemmArgs& args, cudaStream_t stream) {
  using Cfg = GemmCfgPair<256, B_MN>;
  auto kern = gemm_tc_pair_kernel<256, B_MN, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    attr_set = true;
  }
  const int tiles = ((args.M + 2 * BM - 1) / (2 * BM)) * ((args.N + 255) / 256);
  const int pairs = std::min(tiles, args.max_ctas > 0 ? std::max(1, args.max_ctas / 2) : num_sms() / 2);
  if (args.wait_prev) {
    launch_overlapping(kern, dim3(2 * pairs), Cfg::SMEM, stream, a, b, z, b2, args);
  } else {
    kern<<<2 * pairs, 256, Cfg::SMEM, stream>>>(a, b, z, b2, args);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Pair tiles pay off once there are enough of them to occupy the GPU.
// Split-K factor for a GEMM of `tiles` output tiles and `kbs` K-blocks on
// `sms` persistent CTAs. The (tile, split) units are dealt round-robin, so
// the kernel lasts about ceil(units / sms) units of (kbs / splits) K-blocks;
// each split beyond the first adds a little fp32 partial traffic (weighted
// 4 % per split here). Every split keeps at least 4 K-blocks and none is empty.
static int balanced_splits(int tiles, int kbs, int sms, int max_splits) {
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= max_splits; ++s) {
    if (s > 1 && kbs / s < 4) break;
    const int per = (kbs + s - 1) / s;
    const int sp = (kbs + per - 1) / per;
    const int64_t units = (int64_t)tiles * sp;
    const int64_t rounds = (units + sms - 1) / sms;
    const double cost = (double)rounds * per * (1.0 + 0.04 * (sp - 1));
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

static bool use_pair(int M, int N, int epi, bool b_mn, int bn, int splits, int64_t force_bn, int64_t max_ctas) {
  static int mode = -1;  // DSV_GEMM_PAIR=0 disables the pair kernel (1-CTA tiles everywhere)
  if (mode < 0) {
    const char* e = std::getenv("DSV_GEMM_PAIR");
    mode = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  if (mode == 0 || splits != 1 || bn != 256 || force_bn != 0) return false;
  if (!(epi == kEpiBF16 || epi == kEpiF32 || epi == kEpiF32Accum || (epi == kEpiSwiGLU && !b_mn) ||
        ((epi == kEpiCEStats || epi == kEpiCEGrad) && !b_mn) || ((epi == kEpiPushRows || epi == kEpiSwiGLUBwd) && b_mn)))
    return false;
  if (max_ctas > 0 && max_ctas < num_sms()) return false;
  const int tiles = ((M + 255) / 256) * ((N + 255) / 256);
  return M >= 256 && tiles >= num_sms() / 2;
}

template <bool B_MN, int EPI>
static void dispatch_bn(int bn, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& z,
                        const CUtensorMap& b2, const GemmArgs& args, cudaStream_t s) {
  if (bn == 256) launch<256, B_MN, EPI>(a, b, z, b2, args, s);
  else if (bn == 128) launch<128, B_MN, EPI>(a, b, z, b2, args, s);
  else launch<64, B_MN, EPI>(a, b, z, b2, args, s);
}

// Pick the N tile: the widest tile that still gives every SM work.
static int pick_bn(int M, int N, int epi, bool b_mn) {
  if (epi == kEpiSwiGLU) return (N % 256 == 0 && ((M + 127) / 128) * (N / 256) >= num_sms()) ? 256 : 128;
  const int mt = (M + 127) / 128;
  if (mt * ((N + 255) / 256) >= num_sms()) return 256;
  if (mt * ((N + 127) / 128) >= num_sms() / 2 || b_mn) return 128;
  return 64;
}

}  // namespace dsv

// `extra` (the CE and row-push entry points) carries the fields of those
// epilogues; the plain entry point passes nullptr.
static int dsv_gemm_impl(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool b_mn, int64_t epi,
                          c10::optional<torch::Tensor> z, c10::optional<torch::Tensor> b2,
                          c10::optional<torch::Tensor> tile_slots, int64_t lora_seg, c10::optional<torch::Tensor> save,
                          int64_t save_lo, int64_t save_hi, int64_t save_dst, int64_t force_bn, int64_t max_ctas,
                          c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> aux_out,
                          const dsv::GemmArgs* extra, bool overlap_prev = false) {
  using namespace dsv;
  const bool special = epi == kEpiCEStats || epi == kEpiCEGrad || epi == kEpiPushRows;
  TORCH_CHECK(special == (extra != nullptr), "dsv_gemm: epilogue needs its own entry point");
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "dsv_gemm: CUDA tensors expected");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "dsv_gemm: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "dsv_gemm: row-major 2-D operands");
  const int M = (int)a.size(0);
  const int K = (int)a.size(1);
  const int N = b_mn ? (int)b.size(1) : (int)b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "dsv_gemm: reduction length mismatch");
  TORCH_CHECK(out.stride(-1) == 1, "dsv_gemm: output rows must be contiguous");
  if (M == 0 || N == 0) return 64;
  if (epi == kEpiSwiGLU) TORCH_CHECK(N % 128 == 0 && out.size(1) * 2 == N, "dsv_gemm: SwiGLU needs N % 128 == 0");
  if (epi == kEpiSwiGLUBwd) {
    TORCH_CHECK(b_mn && N % 64 == 0 && out.size(1) == 2 * N && aux.has_value(),
                "dsv_gemm: SwiGLU backward needs MN-major B, N % 64 == 0, out [M, 2N] and aux");
    TORCH_CHECK(aux->scalar_type() == at::kBFloat16 && aux->size(0) >= M && aux->size(1) == 2 * N &&
                    aux->stride(1) == 1 && aux->stride(0) % 8 == 0 &&
                    reinterpret_cast<uintptr_t>(aux->data_ptr()) % 16 == 0,
                "dsv_gemm: aux must be bf16 [M, 2N] with 16-byte aligned rows");
    TORCH_CHECK(out.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
                "dsv_gemm: SwiGLU backward output rows must be 16-byte aligned");
    if (aux_out.has_value())
      TORCH_CHECK(aux_out->scalar_type() == at::kBFloat16 && aux_out->size(0) >= M && aux_out->size(1) == N &&
                      aux_out->stride(1) == 1, "dsv_gemm: aux_out must be bf16 [M, N]");
  }
  const bool f32_out = (epi == kEpiF32 || epi == kEpiF32Accum || epi == kEpiCEStats);
  if (epi != kEpiPushRows)  // the push writes peer buffers, not `out`
    TORCH_CHECK(out.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "dsv_gemm: output dtype");
  TORCH_CHECK(K > 0, "dsv_gemm: empty reduction");
  c10::cuda::CUDAGuard guard(a.device());
  // Decode-sized batches (one M tile, plain bf16 store, no row capture): swap
  // the operands so the weights fill the 128-row side of the MMA and stream
  // at full tile width; the tokens become a 64/128-wide N tile and the
  // epilogue stores the transposed accumulator.
  if (!b_mn && M <= 128 && epi == kEpiBF16 && !save.has_value() && force_bn == 0 &&
      (max_ctas == 0 || max_ctas < num_sms()) && N >= 256 && (N % 8) == 0) {
    const int bnt = M <= 64 ? 64 : 128;
    const int tiles = (N + BM - 1) / BM;
    const int kbs = (K + BK - 1) / BK;
    // A grid cap (a share of the SMs) is honoured: the units are balanced over the capped grid.
    const int ctas = max_ctas > 0 ? (int)max_ctas : num_sms();
    const int splits = kbs >= 8 ? balanced_splits(tiles, kbs, ctas, 16) : 1;
    GemmArgs args{};
    args.M = N;
    args.N = M;
    args.K = K;
    args.k_splits = splits;
    args.max_ctas = (int)max_ctas;
    args.wait_prev = (overlap_prev && lora_seg > 0) ? 1 : 0;
    args.C = out.data_ptr();
    args.ldc = (int)out.stride(0);
    at::Tensor partial;
    if (splits > 1) {
      partial = at::empty({splits, N, M}, a.options().dtype(at::kFloat));
      args.partial = partial.data_ptr<float>();
    }
    CUtensorMap ta = make_tmap_bf16(b.data_ptr(), N, K, b.stride(0), BM);
    CUtensorMap tb = make_tmap_bf16(a.data_ptr(), M, K, a.stride(0), bnt);
    CUtensorMap tz = ta, tb2 = tb;
    if (lora_seg > 0) {
      TORCH_CHECK(z.has_value() && b2.has_value() && tile_slots.has_value(), "dsv_gemm: LoRA operands missing");
      TORCH_CHECK(lora_seg % 64 == 0, "dsv_gemm: lora_seg must be a multiple of 64");
      auto& zt = *z;
      auto& bt = *b2;
      TORCH_CHECK(zt.size(0) >= M && bt.size(0) == N && zt.size(1) == bt.size(1), "dsv_gemm: LoRA shapes");
      TORCH_CHECK(tile_slots->scalar_type() == at::kInt && tile_slots->numel() >= 1, "dsv_gemm: tile_slots");
      tz = make_tmap_bf16(bt.data_ptr(), N, bt.size(1), bt.stride(0), BM);     // expand factor: A side
      tb2 = make_tmap_bf16(zt.data_ptr(), M, zt.size(1), zt.stride(0), bnt);   // shrunk tokens: B side
      args.lora_seg = (int)lora_seg;
      args.num_slots = (int)(zt.size(1) / lora_seg);
      args.tile_slots = reinterpret_cast<const uint32_t*>(tile_slots->data_ptr<int>());
      args.slot_or = 1;
    }
    cudaStream_t st = at::cuda::getCurrentCUDAStream();
    if (bnt == 64) launch<64, false, kEpiBF16T>(ta, tb, tz, tb2, args, st);
    else launch<128, false, kEpiBF16T>(ta, tb, tz, tb2, args, st);
    if (splits > 1) {
      // A separate, fully parallel reduction measured faster than letting the
      // last split of each tile reduce it (a serial tail of 128 threads).
      const int64_t work = (int64_t)M * N;
      const int blocks = (int)std::min<int64_t>(4096, (work + 255) / 256);
      splitk_reduce_kernel<<<blocks, 256, 0, st>>>(args.partial, splits, N, M, (int)kEpiBF16T, out.data_ptr(),
                                                   args.ldc, nullptr, 0, 0, 0, 0);
      C10_CUDA_KERNEL_LAUNCH_CHECK();
    }
    return bnt;
  }
  int bn = force_bn > 0 ? (int)force_bn : pick_bn(M, N, (int)epi, b_mn);
  if (b_mn && bn < 64) bn = 64;
  if (epi == kEpiSwiGLU && bn < 128) bn = 128;
  // Split-K for problems with too few output tiles to fill the GPU (decode:
  // one M tile; the trainer's rank-sized LoRA products: one skinny side):
  // each split streams a slice of K, fp32 partials are reduced after in a
  // fixed order (deterministic). Not with a real grid cap or the SwiGLU
  // backward epilogue (its product is never materialised).
  int splits = 1;
  {
    const int kbs = (K + BK - 1) / BK;
    const int m_t = (M + BM - 1) / BM;
    const bool uncapped = max_ctas == 0 || max_ctas >= num_sms();
    if (!b_mn && m_t == 1 && max_ctas == 0 && force_bn == 0 && bn == 64 && epi != kEpiSwiGLU) bn = 128;
    if (uncapped && epi != kEpiSwiGLUBwd && !special) {
      const int tiles = m_t * ((N + bn - 1) / bn);
      if (tiles < num_sms() / 2 && kbs >= 8) {
        splits = std::max(1, std::min({num_sms() / tiles, kbs / 4, 16}));
        const int per = (kbs + splits - 1) / splits;
        splits = (kbs + per - 1) / per;  // no empty split
      }
    }
  }
  GemmArgs args{};
  args.k_splits = splits;
  args.wait_prev = (overlap_prev && lora_seg > 0) ? 1 : 0;
  at::Tensor partial;
  if (splits > 1) {
    partial = at::empty({splits, M, N}, a.options().dtype(at::kFloat));
    args.partial = partial.data_ptr<float>();
  }
  args.M = M;
  args.N = N;
  args.K = K;
  args.C = out.data_ptr();
  args.ldc = (int)out.stride(0);
  args.max_ctas = (int)max_ctas;
  if (extra != nullptr) {
    args.ce_labels = extra->ce_labels;
    args.ce_v0 = extra->ce_v0;
    args.ce_stats = extra->ce_stats;
    args.ce_ld = extra->ce_ld;
    args.ce_tgt = extra->ce_tgt;
    args.ce_lse = extra->ce_lse;
    args.ce_scale = extra->ce_scale;
    args.push = extra->push;
  }
  const bool pair = use_pair(M, N, (int)epi, b_mn, bn, splits, force_bn, max_ctas);
  const int b_box = pair ? bn / 2 : bn;  // a pair CTA stages half of the B tile
  CUtensorMap ta = make_tmap_bf16(a.data_ptr(), M, K, a.stride(0), BM);
  CUtensorMap tb = b_mn ? make_tmap_bf16(b.data_ptr(), K, N, b.stride(0), BK)
                        : make_tmap_bf16(b.data_ptr(), N, K, b.stride(0), b_box);
  CUtensorMap tz = ta, tb2 = tb;
  if (lora_seg > 0) {
    TORCH_CHECK(z.has_value() && b2.has_value() && tile_slots.has_value(), "dsv_gemm: LoRA operands missing");
    TORCH_CHECK(lora_seg % 64 == 0, "dsv_gemm: lora_seg must be a multiple of 64");
    auto& zt = *z;
    auto& bt = *b2;
    if (b_mn) {  // B2 is [S*SEG, N] (same orientation as B); rows past its end read as zero
      TORCH_CHECK(zt.size(0) >= M && bt.size(1) == N && zt.size(1) >= bt.size(0), "dsv_gemm: LoRA shapes");
    } else {     // B2 is [N, S*SEG]
      TORCH_CHECK(zt.size(0) >= M && bt.size(0) == N && zt.size(1) == bt.size(1), "dsv_gemm: LoRA shapes");
    }
    TORCH_CHECK(tile_slots->scalar_type() == at::kInt && tile_slots->numel() >= (M + BM - 1) / BM, "dsv_gemm: tile_slots");
    tz = make_tmap_bf16(zt.data_ptr(), M, zt.size(1), zt.stride(0), BM);
    tb2 = b_mn ? make_tmap_bf16(bt.data_ptr(), bt.size(0), N, bt.stride(0), BK)
               : make_tmap_bf16(bt.data_ptr(), N, bt.size(1), bt.stride(0), b_box);
    args.lora_seg = (int)lora_seg;
    args.num_slots = (int)(zt.size(1) / lora_seg);
    args.tile_slots = reinterpret_cast<const uint32_t*>(tile_slots->data_ptr<int>());
  }
  if (epi == kEpiSwiGLUBwd) {
    args.aux = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr());
    args.ld_aux = (int)aux->stride(0);
    if (aux_out.has_value()) {
      args.aux_out = reinterpret_cast<__nv_bfloat16*>(aux_out->data_ptr());
      args.ld_aux_out = (int)aux_out->stride(0);
    }
  }
  if (save.has_value()) {
    TORCH_CHECK(save->scalar_type() == at::kBFloat16 && save->stride(1) == 1, "dsv_gemm: save buffer");
    args.save = reinterpret_cast<__nv_bfloat16*>(save->data_ptr());
    args.ld_save = (int)save->stride(0);
    args.save_lo = (int)save_lo;
    args.save_hi = (int)save_hi;
    args.save_dst = (int)save_dst;
  }
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  if (pair) {
    if (b_mn) {
      if (epi == kEpiBF16) launch_pair<true, kEpiBF16>(ta, tb, tz, tb2, args, s);
      else if (epi == kEpiF32) launch_pair<true, kEpiF32>(ta, tb, tz, tb2, args, s);
      else if (epi == kEpiPushRows) launch_pair<true, kEpiPushRows>(ta, tb, tz, tb2, args, s);
      else if (epi == kEpiSwiGLUBwd) launch_pair<true, kEpiSwiGLUBwd>(ta, tb, tz, tb2, args, s);
      else launch_pair<true, kEpiF32Accum>(ta, tb, tz, tb2, args, s);
    } else {
      if (epi == kEpiBF16) launch_pair<false, kEpiBF16>(ta, tb, tz, tb2, args, s);
      else if (epi == kEpiF32) launch_pair<false, kEpiF32>(ta, tb, tz, tb2, args, s);
      else if (epi == kEpiF32Accum) launch_pair<false, kEpiF32Accum>(ta, tb, tz, tb2, args, s);
      else if (epi == kEpiCEStats) launch_pair<false, kEpiCEStats>(ta, tb, tz, tb2, args, s);
      else if (epi == kEpiCEGrad) launch_pair<false, kEpiCEGrad>(ta, tb, tz, tb2, args, s);
      else launch_pair<false, kEpiSwiGLU>(ta, tb, tz, tb2, args, s);
    }
    return 256;
  }
  if (b_mn) {
    if (epi == kEpiBF16) dispatch_bn<true, kEpiBF16>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiF32) dispatch_bn<true, kEpiF32>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiF32Accum) dispatch_bn<true, kEpiF32Accum>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiSwiGLUBwd) dispatch_bn<true, kEpiSwiGLUBwd>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiPushRows) dispatch_bn<true, kEpiPushRows>(bn, ta, tb, tz, tb2, args, s);
    else TORCH_CHECK(false, "dsv_gemm: unsupported epilogue for MN-major B");
  } else {
    if (epi == kEpiBF16) dispatch_bn<false, kEpiBF16>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiF32) dispatch_bn<false, kEpiF32>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiF32Accum) dispatch_bn<false, kEpiF32Accum>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiSwiGLU) dispatch_bn<false, kEpiSwiGLU>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiCEStats) dispatch_bn<false, kEpiCEStats>(bn, ta, tb, tz, tb2, args, s);
    else if (epi == kEpiCEGrad) dispatch_bn<false, kEpiCEGrad>(bn, ta, tb, tz, tb2, args, s);
    else TORCH_CHECK(false, "dsv_gemm: unsupported epilogue for K-major B");
  }
  if (splits > 1) {
    const int64_t work = (epi == kEpiSwiGLU) ? (int64_t)M * (N / 2) : (int64_t)M * N;
    const int blocks = (int)std::min<int64_t>(4096, (work + 255) / 256);
    splitk_reduce_kernel<<<blocks, 256, 0, s>>>(args.partial, splits, M, N, (int)epi, out.data_ptr(), args.ldc,
                                                args.save, args.ld_save, args.save_lo, args.save_hi,
                                                args.save_dst);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return bn;
}

// out = a @ b^T (b_mn=false, b is [N, K]) or a @ b (b_mn=true, b is [K_red, N]);
// optional LoRA expand z @ b2^T over the slots listed per M tile.
void dsv_gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool b_mn, int64_t epi,
              c10::optional<torch::Tensor> z, c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> tile_slots,
              int64_t lora_seg, c10::optional<torch::Tensor> save, int64_t save_lo, int64_t save_hi,
              int64_t save_dst, int64_t force_bn, int64_t max_ctas, c10::optional<torch::Tensor> aux,
              c10::optional<torch::Tensor> aux_out, bool overlap_prev) {
  dsv_gemm_impl(a, b, out, b_mn, epi, z, b2, tile_slots, lora_seg, save, save_lo, save_hi, save_dst, force_bn,
                max_ctas, aux, aux_out, nullptr, overlap_prev);
}

// LM-head statistics for cross-entropy without storing logits: for
// logits = h @ w^T (w = rows [v0, v0 + N) of the vocabulary, [N, K]), writes
// per row and N tile the tile's (max, sum exp(logit - max)) into `stats`
// (fp32 [M, >= 2 * ceil(N / 64)], read as float2 pairs) and the label's logit
// into tgt[row] when the label lies in this slice (other rows untouched).
// Returns the number of N tiles written per row.
int64_t dsv_gemm_ce_stats(torch::Tensor h, torch::Tensor w, torch::Tensor labels, int64_t v0, torch::Tensor stats,
                          torch::Tensor tgt, int64_t max_ctas) {
  using namespace dsv;
  const int M = (int)h.size(0), N = (int)w.size(0);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() >= M,
              "ce_stats: labels must be int64 [>= M]");
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.dim() == 2 && stats.size(0) >= M && stats.stride(1) == 1 &&
                  stats.size(1) >= 2 * ((N + 63) / 64) && stats.stride(0) % 2 == 0,
              "ce_stats: stats must be fp32 [M, >= 2 * ceil(N / 64)]");
  TORCH_CHECK(tgt.scalar_type() == at::kFloat && tgt.is_contiguous() && tgt.numel() >= M, "ce_stats: tgt fp32 [M]");
  GemmArgs ex{};
  ex.ce_labels = labels.data_ptr<int64_t>();
  ex.ce_v0 = v0;
  ex.ce_stats = reinterpret_cast<float2*>(stats.data_ptr<float>());
  ex.ce_ld = (int)(stats.stride(0) / 2);
  ex.ce_tgt = tgt.data_ptr<float>();
  const int bn = dsv_gemm_impl(h, w, stats, false, kEpiCEStats, c10::nullopt, c10::nullopt, c10::nullopt, 0,
                               c10::nullopt, 0, 0, 0, 0, max_ctas, c10::nullopt, c10::nullopt, &ex);
  return (N + bn - 1) / bn;
}

// Cross-entropy gradient rows from recomputed logits: dlog = (softmax - onehot)
// * scale in bf16 for logits = h @ w^T, w = rows [v0, v0 + N) of the
// vocabulary; lse [M] is each row's log-sum-exp over the whole vocabulary;
// rows whose label is -1 get zeros.
void dsv_gemm_ce_grad(torch::Tensor h, torch::Tensor w, torch::Tensor labels, int64_t v0, torch::Tensor lse,
                      double scale, torch::Tensor dlog, int64_t max_ctas) {
  using namespace dsv;
  const int M = (int)h.size(0);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() >= M,
              "ce_grad: labels must be int64 [>= M]");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() >= M, "ce_grad: lse fp32 [M]");
  TORCH_CHECK(dlog.scalar_type() == at::kBFloat16 && dlog.size(0) >= M && dlog.size(1) == w.size(0),
              "ce_grad: dlog must be bf16 [M, N]");
  GemmArgs ex{};
  ex.ce_labels = labels.data_ptr<int64_t>();
  ex.ce_v0 = v0;
  ex.ce_lse = lse.data_ptr<float>();
  ex.ce_scale = (float)scale;
  dsv_gemm_impl(h, w, dlog, false, kEpiCEGrad, c10::nullopt, c10::nullopt, c10::nullopt, 0, c10::nullopt, 0, 0, 0,
                0, max_ctas, c10::nullopt, c10::nullopt, &ex);
}

// a @ b (MN-major b, [K, N]) (+ the LoRA term z @ b2) pushed to the row
// owners as bf16 partials (see PushArgs): `table` is an int64 CPU tensor
// [2, world] of device addresses (receive rows and block counters of every
// rank); `add` (optional fp32 [M, >= N]) is added before the push.
void dsv_gemm_push(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> z, c10::optional<torch::Tensor> b2,
                   c10::optional<torch::Tensor> tile_slots, int64_t lora_seg, torch::Tensor table, int64_t rank,
                   int64_t world, int64_t blocks_cap, int64_t ld, c10::optional<torch::Tensor> add,
                   int64_t max_ctas) {
  using namespace dsv;
  const int M = (int)a.size(0), N = (int)b.size(1);
  TORCH_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "gemm_push: rank/world");
  TORCH_CHECK(table.device().is_cpu() && table.scalar_type() == at::kLong && table.size(0) == 2 &&
                  table.size(1) == world, "gemm_push: table must be int64 [2, world] on the CPU");
  TORCH_CHECK(N % 32 == 0 && ld >= N && ld % 8 == 0, "gemm_push: N % 32 == 0 and a 16-byte row pitch >= N");
  TORCH_CHECK(((M + BM - 1) / BM + world - 1) / world <= blocks_cap, "gemm_push: too many rows for the workspace");
  GemmArgs ex{};
  PushArgs& P = ex.push;
  P.rank = (int)rank;
  P.world = (int)world;
  P.blocks_cap = (int)blocks_cap;
  P.ld = (int)ld;
  if (add.has_value()) {
    TORCH_CHECK(add->scalar_type() == at::kFloat && add->size(0) >= M && add->size(1) >= N && add->stride(1) == 1 &&
                    add->stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(add->data_ptr()) % 16 == 0,
                "gemm_push: add must be fp32 [M, >= N] with 16-byte aligned rows");
    P.add = add->data_ptr<float>();
    P.ld_add = (int)add->stride(0);
  }
  auto* tab = table.data_ptr<int64_t>();
  for (int r = 0; r < world; ++r) {
    P.recv[r] = reinterpret_cast<__nv_bfloat16*>(tab[r]);
    P.cnt[r] = reinterpret_cast<uint32_t*>(tab[world + r]);
  }
  dsv_gemm_impl(a, b, a, true, kEpiPushRows, z, b2, tile_slots, lora_seg, c10::nullopt, 0, 0, 0, 0, max_ctas,
                c10::nullopt, c10::nullopt, &ex);
}

// LoRA factor gradients, reducing over the token dimension (both operands
// token-major, read MN-major): a [T, M], b [T, N] bf16.
//   kind 0 (kEpiF32T):   out [N, M] fp32 = (a^T b)^T = b^T a   (dA = dZ^T X from a = X, b = dZ);
//   kind 1 (kEpiLoraBt): out [R, M] fp32, out[j, m] = scale * (a^T b)[m, p(m) * R + j]
//                        (dB of every projection of a group from a = dY, b = Z).
// n_valid bounds the columns of b that are used (the rest may be padding).
void dsv_gemm_wgrad(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t kind, int64_t n_valid, int64_t R,
                    int64_t b1, int64_t b2, bool interleave, double scale, int64_t max_ctas) {
  using namespace dsv;
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm_wgrad: CUDA tensors expected");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kFloat,
              "gemm_wgrad: bf16 operands, fp32 output");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1,
              "gemm_wgrad: row-major 2-D tensors");
  const int T = (int)a.size(0), M = (int)a.size(1), N = (int)n_valid;
  TORCH_CHECK(b.size(0) == T && N >= 1 && N <= b.size(1) && N <= 256, "gemm_wgrad: b must be [T, >= n_valid <= 256]");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "gemm_wgrad: 16-byte row pitch");
  if (kind == 0) {
    TORCH_CHECK(out.size(0) >= N && out.size(1) >= M, "gemm_wgrad: out must be [N, M]");
  } else {
    TORCH_CHECK(out.size(0) >= R && out.size(1) >= M && R >= 1, "gemm_wgrad: out must be [R, M]");
  }
  if (T == 0 || M == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args{};
  args.M = M;
  args.N = N;
  args.K = T;
  args.k_splits = 1;
  args.C = out.data_ptr();
  args.ldc = (int)out.stride(0);
  args.bt_r = (int)R;
  args.bt_b1 = (int)b1;
  args.bt_b2 = (int)b2;
  args.bt_interleave = interleave ? 1 : 0;
  args.bt_scale = (float)scale;
  args.max_ctas = (int)max_ctas;
  const int bn = N <= 64 ? 64 : (N <= 128 ? 128 : 256);
  CUtensorMap ta = make_tmap_bf16(a.data_ptr(), T, M, a.stride(0), BK);
  CUtensorMap tb = make_tmap_bf16(b.data_ptr(), T, b.size(1), b.stride(0), BK);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (kind == 0) {
    if (bn == 64) launch<64, true, kEpiF32T>(ta, tb, ta, tb, args, st);
    else if (bn == 128) launch<128, true, kEpiF32T>(ta, tb, ta, tb, args, st);
    else launch<256, true, kEpiF32T>(ta, tb, ta, tb, args, st);
  } else {
    if (bn == 64) launch<64, true, kEpiLoraBt>(ta, tb, ta, tb, args, st);
    else if (bn == 128) launch<128, true, kEpiLoraBt>(ta, tb, ta, tb, args, st);
    else launch<256, true, kEpiLoraBt>(ta, tb, ta, tb, args, st);
  }
}

// Multi-LoRA shrink on the tensor cores: Z[T, slots*seg] from x[T, K] and the
// stacked A factors [slots*pr, K], each row keeping only its own slot's
// segment (rows with slot -1 get zeros). For large T; small T uses the GEMV
// kernel in lora_misc.cu.
void dsv_lora_shrink_tc(torch::Tensor x, torch::Tensor A, torch::Tensor slot_ids, torch::Tensor Z, int64_t pr,
                        int64_t seg) {
  using namespace dsv;
  constexpr int BN = 64;
  const int T = (int)x.size(0), K = (int)x.size(1), N = (int)A.size(0);
  TORCH_CHECK(A.size(1) == K && x.stride(1) == 1 && A.stride(1) == 1 && A.is_contiguous(), "lora_shrink_tc: shapes");
  TORCH_CHECK(N % pr == 0 && Z.size(1) == (N / pr) * seg && Z.size(0) >= T && Z.stride(1) == 1, "lora_shrink_tc: Z");
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  GemmArgs args{};
  args.M = T;
  args.N = N;
  args.K = K;
  args.k_splits = 1;
  args.C = Z.data_ptr();
  args.ldc = (int)Z.stride(0);
  args.shrink_slot_ids = slot_ids.data_ptr<int>();
  args.shrink_pr = (int)pr;
  args.shrink_seg = (int)seg;
  CUtensorMap ta = make_tmap_bf16(x.data_ptr(), T, K, x.stride(0), BM);
  CUtensorMap tb = make_tmap_bf16(A.data_ptr(), N, K, A.stride(0), BN);
  launch<BN, false, kEpiShrink>(ta, tb, ta, tb, args, at::cuda::getCurrentCUDAStream());
}

// Tensor maps ({64 columns, 128 rows} boxes, 128-byte swizzle) of `rows` x
// `cols` bf16 matrices with leading dimension `ld` at each address of `ptrs`
// (int64 CPU tensor, one per rank): the A operand of the all-gather GEMMs.
// Returns their bytes (uint8 CPU [n, 128]) for the caller to place on the device.
torch::Tensor dsv_peer_tmaps(torch::Tensor ptrs, int64_t rows, int64_t cols, int64_t ld) {
  using namespace dsv;
  TORCH_CHECK(ptrs.device().is_cpu() && ptrs.scalar_type() == at::kLong && ptrs.dim() == 1 && ptrs.numel() <= kMaxPeers,
              "peer_tmaps: ptrs must be an int64 CPU tensor of <= 8 addresses");
  static_assert(sizeof(CUtensorMap) == 128, "CUtensorMap is 128 bytes");
  auto out = torch::empty({ptrs.numel(), 128}, torch::dtype(torch::kUInt8));
  for (int64_t r = 0; r < ptrs.numel(); ++r) {
    const CUtensorMap m = make_tmap_bf16(reinterpret_cast<const void*>(ptrs[r].item<int64_t>()), rows, cols, ld, BM);
    std::memcpy(out.data_ptr<uint8_t>() + r * 128, &m, 128);
  }
  return out;
}

namespace {
// Copy-once gather arguments (see GemmArgs::ag_gathered): the gathered buffer
// [>= M, K] of this rank, the per-block unit counters (zeroed by the caller
// when the shards hold new rows) and the ranks' shard addresses.
void set_gather(dsv::GemmArgs& args, const torch::Tensor& gathered, const torch::Tensor& cnt, const torch::Tensor& src,
                int64_t rank, int M, int K) {
  using namespace dsv;
  TORCH_CHECK(gathered.is_cuda() && gathered.scalar_type() == at::kBFloat16 && gathered.is_contiguous() &&
                  gathered.size(0) >= M && gathered.size(1) == K, "gemm_ag: gathered must be bf16 [>= M, K]");
  TORCH_CHECK(cnt.is_cuda() && cnt.scalar_type() == at::kInt && cnt.numel() >= (M + BM - 1) / BM + 1,
              "gemm_ag: cnt must be int32 [>= M / 128 + 1] on the device (block counters, then the ticket)");
  TORCH_CHECK(src.device().is_cpu() && src.scalar_type() == at::kLong && src.numel() == args.ag_world,
              "gemm_ag: src must hold the ranks' shard addresses (int64 CPU)");
  TORCH_CHECK(K % 8 == 0, "gemm_ag: K must be a multiple of 8");
  args.ag_gathered = reinterpret_cast<__nv_bfloat16*>(gathered.data_ptr());
  args.ag_cnt = reinterpret_cast<uint32_t*>(cnt.data_ptr<int>());
  args.ag_ticket = args.ag_cnt + (cnt.numel() - 1);
  args.ag_expect = (uint32_t)((K + kAgChunk - 1) / kAgChunk);
  args.ag_rank = (int)rank;
  for (int r = 0; r < args.ag_world; ++r)
    args.ag_src[r] = reinterpret_cast<const __nv_bfloat16*>(src[r].item<int64_t>());
}

void check_ag(const torch::Tensor& maps, int64_t ag_rows, int64_t world, const torch::Tensor& a_local) {
  TORCH_CHECK(maps.is_cuda() && maps.scalar_type() == at::kByte && maps.is_contiguous() && maps.numel() == world * 128 &&
                  reinterpret_cast<uintptr_t>(maps.data_ptr()) % 64 == 0,
              "gemm_ag: maps must be a 64-byte aligned uint8 CUDA tensor [world, 128]");
  TORCH_CHECK(world >= 1 && world <= dsv::kMaxPeers && ag_rows > 0 && ag_rows % dsv::BM == 0,
              "gemm_ag: rows per rank must be a positive multiple of 128, world <= 8");
  TORCH_CHECK(a_local.is_cuda() && a_local.scalar_type() == at::kBFloat16 && a_local.dim() == 2 &&
                  a_local.stride(1) == 1 && a_local.size(0) >= ag_rows,
              "gemm_ag: a_local must be this rank's bf16 shard [>= ag_rows, K]");
}
}  // namespace

// out[M, N] = A_all @ b^T (+ LoRA expand) with M = ag_rows * world, where
// A_all's rows [r * ag_rows, (r + 1) * ag_rows) are rank r's shard, read by
// TMA straight from that rank's memory (the all-gather fused into the GEMM's
// loads). epi: bf16 store or SwiGLU.
void dsv_gemm_ag(torch::Tensor maps, int64_t ag_rows, int64_t world, torch::Tensor a_local, torch::Tensor b,
                 torch::Tensor out, int64_t epi, c10::optional<torch::Tensor> z, c10::optional<torch::Tensor> b2,
                 c10::optional<torch::Tensor> tile_slots, int64_t lora_seg, c10::optional<torch::Tensor> gathered,
                 c10::optional<torch::Tensor> cnt, c10::optional<torch::Tensor> src, int64_t rank) {
  using namespace dsv;
  check_ag(maps, ag_rows, world, a_local);
  TORCH_CHECK(epi == kEpiBF16 || epi == kEpiSwiGLU, "gemm_ag: bf16 or SwiGLU epilogue");
  TORCH_CHECK(b.is_cuda() && b.scalar_type() == at::kBFloat16 && b.dim() == 2 && b.stride(1) == 1 &&
                  b.size(1) == a_local.size(1), "gemm_ag: b must be bf16 [N, K]");
  const int M = (int)(ag_rows * world), K = (int)a_local.size(1), N = (int)b.size(0);
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.size(0) >= M &&
                  out.size(1) == (epi == kEpiSwiGLU ? N / 2 : N), "gemm_ag: out must be bf16 [M, N (or N/2)]");
  if (epi == kEpiSwiGLU) TORCH_CHECK(N % 128 == 0, "gemm_ag: SwiGLU needs N % 128 == 0");
  c10::cuda::CUDAGuard guard(b.device());
  GemmArgs args{};
  args.M = M;
  args.N = N;
  args.K = K;
  args.k_splits = 1;
  args.C = out.data_ptr();
  args.ldc = (int)out.stride(0);
  args.ag_maps = reinterpret_cast<const CUtensorMap*>(maps.data_ptr());
  args.ag_rows = (int)ag_rows;
  args.ag_world = (int)world;
  args.ag_rank = (int)rank;
  const int bn = (epi == kEpiSwiGLU) ? std::max(128, pick_bn(M, N, (int)epi, false)) : pick_bn(M, N, (int)epi, false);
  CUtensorMap ta;
  if (gathered.has_value()) {
    TORCH_CHECK(cnt.has_value() && src.has_value(), "gemm_ag: the copy-once gather needs cnt and src");
    set_gather(args, *gathered, *cnt, *src, rank, M, K);
    ta = make_tmap_bf16(gathered->data_ptr(), gathered->size(0), K, K, BM);
  } else {
    ta = make_tmap_bf16(a_local.data_ptr(), a_local.size(0), K, a_local.stride(0), BM);
  }
  CUtensorMap tb = make_tmap_bf16(b.data_ptr(), N, K, b.stride(0), bn);
  CUtensorMap tz = ta, tb2 = tb;
  if (lora_seg > 0) {
    TORCH_CHECK(z.has_value() && b2.has_value() && tile_slots.has_value(), "gemm_ag: LoRA operands missing");
    TORCH_CHECK(lora_seg % 64 == 0 && z->size(0) >= M && b2->size(0) == N && z->size(1) == b2->size(1) &&
                    tile_slots->numel() >= (M + BM - 1) / BM, "gemm_ag: LoRA shapes");
    tz = make_tmap_bf16(z->data_ptr(), M, z->size(1), z->stride(0), BM);
    tb2 = make_tmap_bf16(b2->data_ptr(), N, b2->size(1), b2->stride(0), bn);
    args.lora_seg = (int)lora_seg;
    args.num_slots = (int)(z->size(1) / lora_seg);
    args.tile_slots = reinterpret_cast<const uint32_t*>(tile_slots->data_ptr<int>());
  }
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  if (epi == kEpiSwiGLU) dispatch_bn<false, kEpiSwiGLU>(bn, ta, tb, tz, tb2, args, s);
  else dispatch_bn<false, kEpiBF16>(bn, ta, tb, tz, tb2, args, s);
}

// The LoRA shrink of an all-gathered input: Z[M, slots * seg] for the
// M = ag_rows * world rows of every rank's shard (A rows read from their
// owners as in dsv_gemm_ag), each row keeping its own slot's segment.
void dsv_lora_shrink_ag(torch::Tensor maps, int64_t ag_rows, int64_t world, torch::Tensor x_local, torch::Tensor A,
                        torch::Tensor slot_ids, torch::Tensor Z, int64_t pr, int64_t seg,
                        c10::optional<torch::Tensor> gathered, c10::optional<torch::Tensor> cnt,
                        c10::optional<torch::Tensor> src, int64_t rank) {
  using namespace dsv;
  check_ag(maps, ag_rows, world, x_local);
  constexpr int BN = 64;
  const int M = (int)(ag_rows * world), K = (int)x_local.size(1), N = (int)A.size(0);
  TORCH_CHECK(A.size(1) == K && A.is_contiguous() && N % pr == 0 && Z.size(1) == (N / pr) * seg && Z.size(0) >= M &&
                  slot_ids.numel() >= M, "lora_shrink_ag: shapes");
  c10::cuda::CUDAGuard guard(A.device());
  GemmArgs args{};
  args.M = M;
  args.N = N;
  args.K = K;
  args.k_splits = 1;
  args.C = Z.data_ptr();
  args.ldc = (int)Z.stride(0);
  args.shrink_slot_ids = slot_ids.data_ptr<int>();
  args.shrink_pr = (int)pr;
  args.shrink_seg = (int)seg;
  args.ag_maps = reinterpret_cast<const CUtensorMap*>(maps.data_ptr());
  args.ag_rows = (int)ag_rows;
  args.ag_world = (int)world;
  args.ag_rank = (int)rank;
  CUtensorMap ta;
  if (gathered.has_value()) {
    TORCH_CHECK(cnt.has_value() && src.has_value(), "lora_shrink_ag: the copy-once gather needs cnt and src");
    set_gather(args, *gathered, *cnt, *src, rank, M, K);
    ta = make_tmap_bf16(gathered->data_ptr(), gathered->size(0), K, K, BM);
  } else {
    ta = make_tmap_bf16(x_local.data_ptr(), x_local.size(0), K, x_local.stride(0), BM);
  }
  CUtensorMap tb = make_tmap_bf16(A.data_ptr(), N, K, A.stride(0), BN);
  launch<BN, false, kEpiShrink>(ta, tb, ta, tb, args, at::cuda::getCurrentCUDAStream());
}

// out = all_reduce_over_ranks(a @ b^T (+ LoRA expand)), fused: the GEMM's
// epilogue pushes bf16 partial tiles to their owner rank over peer memory and
// the same launch reduces the owned tiles and broadcasts them.
// `peer` is an int64 CPU tensor [4, world] of device addresses
// (recv, out, rflag, fflag per rank); `tile_cnt` this rank's split-K tickets.
// Returns the [M, N] result: a view of this rank's output buffer, valid until
// the next call on the same workspace.
torch::Tensor dsv_gemm_ar(torch::Tensor a, torch::Tensor b, c10::optional<torch::Tensor> z,
                          c10::optional<torch::Tensor> b2, c10::optional<torch::Tensor> tile_slots, int64_t lora_seg,
                          torch::Tensor peer, int64_t tile_cnt, int64_t rank, int64_t world, int64_t owned_cap,
                          int64_t out_rows, int64_t force_splits, int64_t force_reducers) {
  using namespace dsv;
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "dsv_gemm_ar: CUDA tensors expected");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "dsv_gemm_ar: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "dsv_gemm_ar: row-major 2-D");
  TORCH_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "dsv_gemm_ar: rank/world");
  TORCH_CHECK(peer.device().is_cpu() && peer.scalar_type() == at::kLong && peer.size(0) == 4 && peer.size(1) == world,
              "dsv_gemm_ar: peer table must be int64 [4, world] on the CPU");
  constexpr int BN = 128;
  const int M = (int)a.size(0), K = (int)a.size(1), N = (int)b.size(0);
  TORCH_CHECK(b.size(1) == K, "dsv_gemm_ar: reduction length mismatch");
  TORCH_CHECK(N % BN == 0, "dsv_gemm_ar: N must be a multiple of 128");
  TORCH_CHECK(M <= out_rows, "dsv_gemm_ar: M exceeds the workspace rows");
  const int m_tiles = (M + BM - 1) / BM, n_tiles = N / BN, tiles = m_tiles * n_tiles;
  TORCH_CHECK((tiles + world - 1) / world <= owned_cap, "dsv_gemm_ar: workspace too small for this shape");
  auto opts = a.options();
  auto* tab = peer.data_ptr<int64_t>();
  torch::Tensor out = torch::from_blob(reinterpret_cast<void*>(tab[1 * world + rank]), {M, N}, opts);
  if (M == 0) return out;
  c10::cuda::CUDAGuard guard(a.device());
  int splits = 1;
  const int kbs = (K + BK - 1) / BK;
  if (force_splits > 0) {
    splits = (int)force_splits;
  } else if (m_tiles == 1 && tiles < num_sms() / 2 && kbs >= 8) {
    splits = std::max(1, std::min({(num_sms() - kArSmReserve - 8) / tiles, kbs / 4, 16}));
  }
  if (splits > 1) {
    const int per = (kbs + splits - 1) / splits;
    splits = (kbs + per - 1) / per;
  }
  GemmArgs args{};
  args.M = M;
  args.N = N;
  args.K = K;
  args.k_splits = splits;
  at::Tensor partial;
  if (splits > 1) {
    partial = at::empty({splits, M, N}, opts.dtype(at::kFloat));
    args.partial = partial.data_ptr<float>();
  }
  PeerArgs& P = args.peer;
  P.rank = (int)rank;
  P.world = (int)world;
  P.owned_cap = (int)owned_cap;
  P.ldo = N;
  P.tile_cnt = reinterpret_cast<uint32_t*>(tile_cnt);
  for (int r = 0; r < world; ++r) {
    P.recv[r] = reinterpret_cast<__nv_bfloat16*>(tab[0 * world + r]);
    P.out[r] = reinterpret_cast<__nv_bfloat16*>(tab[1 * world + r]);
    P.rflag[r] = reinterpret_cast<uint32_t*>(tab[2 * world + r]);
    P.fflag[r] = reinterpret_cast<uint32_t*>(tab[3 * world + r]);
  }
  CUtensorMap ta = make_tmap_bf16(a.data_ptr(), M, K, a.stride(0), BM);
  CUtensorMap tb = make_tmap_bf16(b.data_ptr(), N, K, b.stride(0), BN);
  CUtensorMap tz = ta, tb2 = tb;
  if (lora_seg > 0) {
    TORCH_CHECK(z.has_value() && b2.has_value() && tile_slots.has_value(), "dsv_gemm_ar: LoRA operands missing");
    TORCH_CHECK(lora_seg % 64 == 0, "dsv_gemm_ar: lora_seg must be a multiple of 64");
    auto& zt = *z;
    auto& bt = *b2;
    TORCH_CHECK(zt.size(0) >= M && bt.size(0) == N && zt.size(1) == bt.size(1), "dsv_gemm_ar: LoRA shapes");
    TORCH_CHECK(tile_slots->scalar_type() == at::kInt && tile_slots->numel() >= m_tiles, "dsv_gemm_ar: tile_slots");
    tz = make_tmap_bf16(zt.data_ptr(), M, zt.size(1), zt.stride(0), BM);
    tb2 = make_tmap_bf16(bt.data_ptr(), N, bt.size(1), bt.stride(0), BN);
    args.lora_seg = (int)lora_seg;
    args.num_slots = (int)(zt.size(1) / lora_seg);
    args.tile_slots = reinterpret_cast<const uint32_t*>(tile_slots->data_ptr<int>());
  }
  using Cfg = GemmCfg<BN, false>;
  auto kern = gemm_tc_kernel<BN, false, kEpiPeerAR>;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    attr_set = true;
  }
  // One CTA per SM at most, and kArSmReserve SMs left to other streams: every
  // CTA of this grid can be resident at once even while the backward stream
  // runs an NCCL kernel (capped at the same number of CTAs by init_tp), so a
  // CTA waiting on a peer never keeps the peer's partner CTA (or the peer's
  // NCCL kernel) from being scheduled. A cooperative launch would give the
  // same guarantee but waits for the whole GPU to drain first.
  const int n_owned = (tiles - (int)rank + (int)world - 1) / (int)world;
  const int budget = std::max(2, num_sms() - kArSmReserve);
  // One wave of GEMM work: the GEMM CTAs reduce afterwards (reducers = 0).
  // Several waves: dedicated reducer CTAs overlap the exchange with the GEMM.
  // Measured at TP=2 (M = 64..4096): reducing in the GEMM CTAs after their
  // tiles beats dedicated reducer CTAs at every size, so that is the default.
  (void)n_owned;
  P.reducers = 0;
  if (force_reducers >= 0) P.reducers = (int)std::min<int64_t>(force_reducers, budget / 2);
  const int gemm_ctas = std::max(1, std::min(tiles * splits, budget - P.reducers));
  const int grid = P.reducers + gemm_ctas;
  gemm_tc_kernel<BN, false, kEpiPeerAR><<<grid, 256, Cfg::SMEM, at::cuda::getCurrentCUDAStream()>>>(
      ta, tb, tz, tb2, args);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

DSV_ERROR_ACCESSOR(dsv_read_error_gemm)
