// Layer-boundary fusion of tensor-parallel decode: the row-parallel GEMM, the all-reduce + residual
// add + RMSNorm, and the next column-parallel GEMM, in two kernels that exchange data through the
// one-shot Lamport landing buffers of the symmetric heap (fused_ar.h):
//
//   gemm_push   : Y_r = X_r W_r^T on the tensor cores; the epilogue pushes Y_r (bf16, Lamport-encoded)
//                 straight into land1[slot][r] of every rank - no local Y, no separate collective.
//   ar_norm_gemm: waits for the W pushed partials, h = residual + sum_r Y_r (written back to the
//                 residual), RMSNorm folded into the next GEMM: Z = (h * gamma) W2^T scaled per row by
//                 rsqrt(mean(h^2) + eps). Its weight stream starts before the partials arrive.
//
// Both are cluster split-K GEMMs (grid = output tiles x splits, the splits of a tile form a cluster
// and sum their partial tiles through distributed shared memory). Decode shapes: M <= 256 rows.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fused_ar.h"

namespace cob {

constexpr int kMaxPieces = 512;  // ar_norm_gemm: CTAs per call (tiles x splits)

struct FusedGemmParams {
  char* base[kMaxWorld];  // heaps as seen from this GPU (emulate: every rank's heap region)
  Layout L;
  int rank, world, emulate;  // emulate: rank = blockIdx.z, all ranks in one launch on one GPU
  int M, N, K;               // this rank's GEMM: [M, K] x [N, K]^T, weights stacked by rank when emulating
  int kps;                   // 64-wide k-steps per split (splits = gridDim.y)
  unsigned long long timeout_ns;
  int l2_prefetch;           // weight tiles beyond the ring prefetched into L2 before the activations are awaited
  // packed weights (nullptr: the row-major weight through its tensor map): per rank, ceil(N / 128)
  // x (K / 64) blocks of 128 x 64 elements in the swizzled shared-memory image (see gemm.h), ranks
  // stacked when emulating; w_tiles = ceil(N / 128)
  const uint8_t* wp;
  int w_tiles;
  int* err;                  // device word: nonzero after a timed-out wait in this kernel
  // ar_norm_gemm only
  void* residual;            // [M, K] in / out (each element read and written by one thread)
  const void* gamma;         // [K]
  float eps;
  void* act;                 // [ranks * M_max, K] staging of h * gamma (TMA source of the B operand)
  int act_rows;              // M_max: rows per rank in `act`
  uint32_t* flags;           // [ranks][kMaxPieces] epoch of the last piece written by CTA p
  float* pss;                // [ranks][kMaxPieces][M_max] per-piece partial sums of squares
  void* Y;                   // [M, N] output (ldy = N); emulate: rank r at Y + r * M * N
  long long x_rs, res_rs;    // emulate element strides between ranks' X / residual
  // ar_norm_gemm epilogue applied to each 128-row output tile as two halves (rows f and 64 + f):
  //   kEpiPlain  : Y[M, N]
  //   kEpiSwiglu : Y[M, N / 2] = silu(gate) * up, weights tile-interleaved (tile t = 64 gate rows
  //                t*64.. then the 64 matching up rows)
  //   kEpiRopeKv : tile t = head t of [q heads | k heads | v heads] (head_dim 128): q heads rotated
  //                (RoPE at positions[b]) into Y = q_out [M, nq, 128]; k heads rotated and v heads copied
  //                into the paged caches [blocks, nkv, bs, 128] at slot positions[b]
  int epi;
  const int* positions;      // [M]
  const float* cos_t;        // [max_pos, 64]
  const float* sin_t;
  const int* block_tables;   // [M, max_blocks]
  int max_blocks, nq, nkv, bs;
  void* k_cache;
  void* v_cache;
  long long cache_rs;        // emulate element stride between ranks' caches
};

enum FusedEpi : int { kEpiPlain = 0, kEpiSwiglu = 1, kEpiRopeKv = 2 };

struct FusedGemmPlan {
  int bn, tiles, splits, kps, smem, ctas;
  int xctas;  // CTAs along the output dimension (== tiles, or fewer looping over tiles when splits == 1)
};

// Geometry for M rows, N outputs, K inner: BN (MMA N) and the split count (0 = choose). `consumer`:
// plan for ar_norm_gemm (whole grid resident, at most kMaxBlocks CTAs). The paired epilogues
// (swiglu, rope) need 2..8 splits per tile (each CTA of a cluster finishes whole row pairs); a plan
// that cannot meet that returns splits == 0.
FusedGemmPlan plan_fused_gemm(int M, int N, int K, int splits, int num_sms, bool consumer, int epi = kEpiPlain);
// Clusters of `splits` consumer CTAs (batch tile width bn) that the occupancy calculator says can be
// resident on this device at once (-1 on error). launch_ar_norm_gemm rejects grids with more.
int ar_norm_gemm_resident_clusters(int bn, int splits);

// tmW: [ranks * N, K] weights, box 64 x 128; tmX: [rows, K] activations, box 64 x BN.
cudaError_t launch_gemm_push(const FusedGemmParams& p, const CUtensorMap& tmW, const CUtensorMap& tmX,
                             const FusedGemmPlan& plan, int ranks, bool pdl, cudaStream_t stream);
// tmW as above; tmA: the `act` staging buffer [ranks * M_max, K], box 64 x BN.
cudaError_t launch_ar_norm_gemm(const FusedGemmParams& p, const CUtensorMap& tmW, const CUtensorMap& tmA,
                                const FusedGemmPlan& plan, int ranks, bool pdl, cudaStream_t stream);

}  // namespace cob
