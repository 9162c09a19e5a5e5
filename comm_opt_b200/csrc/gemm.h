// Host entry of the sm_100a decode GEMM (plain CUDA, no torch types).
#pragma once

#include <cuda_runtime.h>

#include "types.h"

namespace cob {

struct GemmPlan {
  int bn;      // padded batch width (tcgen05 N): 16, 32, 64, 128 or 256
  int tiles;   // 128-row output tiles
  int splits;  // K split over a thread-block cluster (1..8)
  int kps;     // 64-wide K steps per split
};

GemmPlan plan_gemm(int M, int N, int K, int num_sms, int splits_override);

// Y[M, N] (row stride ldy) = X[M, K] * W[N, K]^T; bf16 or fp16 in and out, fp32 accumulation.
// M <= 256. `err` (device int) receives 1 if a bounded wait timed out.
cudaError_t gemm_decode(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int* err,
                        int num_sms, int splits_override, bool pdl, unsigned long long timeout_ns,
                        cudaStream_t stream, GemmPlan* used);

}  // namespace cob
