// Host entry of the sm_100a decode GEMM (plain CUDA, no torch types).
#pragma once

#include <cuda_runtime.h>

#include "types.h"

namespace cob {

struct GemmPlan {
  int bn;     // padded batch width (tcgen05 N): 16, 32, 64, 128 or 256
  int tiles;  // 128-row output tiles
  int ctas;   // persistent CTAs (stream-K partition of tiles x k-steps)
};

GemmPlan plan_gemm(int M, int N, int K, int num_sms, int ctas_override);

// Profiling: when non-null, every decode GEMM launch writes kStampSlots %globaltimer stamps per CTA
// (entry, set-up, weights issued, dependency wait, last load, first stage landed, last MMA, last
// accumulator ready, last tile stored, end) at stamps[cta * kStampSlots + phase].
constexpr int kStampSlots = 16;
long long*& gemm_stamps();
// With a stride > 0, launch n (counted from the last reset of gemm_stamp_launches) writes at
// gemm_stamps() + n * stride, so every GEMM of a captured decode step keeps its own stamps.
long long& gemm_stamp_stride();
long long& gemm_stamp_launches();
long long* next_gemm_stamps();
// fp32 workspace needed for the partial tiles of a launch with `num_ctas` CTAs
size_t gemm_workspace_bytes(int num_ctas, int bn);

// Y[M, N] (row stride ldy) = X[M, K] * W[N, K]^T; bf16 or fp16 in and out, fp32 accumulation.
// M <= 256. `ws` is the fp32 partial-tile workspace, `tile_ctr` max_tiles int32 that must be zero
// before the first call (the kernel restores them). `err` (device int) is set if a bounded wait
// timed out.
cudaError_t gemm_decode(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, float* ws,
                        size_t ws_bytes, int* tile_ctr, int max_tiles, int* err, int num_sms, int ctas_override,
                        bool pdl, bool small_smem, int cluster_splits, unsigned long long timeout_ns,
                        cudaStream_t stream, GemmPlan* used, bool packed = false, bool swiglu = false);
// cluster_splits > 0 selects the cluster split-K schedule (grid tiles x splits, DSMEM reduction,
// M <= 64, splits <= 16; above 8 a non-portable cluster size) instead of stream-K.
// packed: W is the packed weight layout (see pack_weight in the Python package): for output tile
// t = n / 128 and k-step k = K-column / 64, block t * (K / 64) + k of 128 x 64 elements (16 KB) holds
// rows t*128.. and columns k*64.. exactly as the 128-byte-swizzled shared-memory image (16-byte chunk c
// of row r stored at chunk c ^ (r % 8)), rows past N zero. K must be a multiple of 64.
// swiglu: W's rows are gate and up features interleaved by 64 (rows 128t..128t+63 gate features
// 64t.., rows 128t+64..128t+127 the matching up features), Y is [M, N / 2] (row stride ldy) holding
// silu(gate) * up of the bf16/fp16-rounded projections. Needs N a multiple of 128 and either the cluster
// schedule with a split count (after rounding K into equal k-step shares) of 2, 4, 8 or 16, or stream-K
// with M <= 16 (the workspace then also holds a [64][16] float exchange area per CTA).

}  // namespace cob
