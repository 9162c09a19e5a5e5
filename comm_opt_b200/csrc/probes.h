// Primitive probes (see probes.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cob {

struct RsProbeParams {
  char* base[8];          // per-rank probe heap (accumulator at acc_off, arrival counter at ctr_off)
  long long acc_off, ctr_off;
  const void* x;          // this rank's input: world slices of n elements (f32 or bf16)
  long long x_rank_bytes; // emulate mode: bytes between ranks' inputs
  int rank, world, n, variant, emulate;  // variant 0 red.f32, 1 red.v4.f32, 2 red.bf16x2, 3 red.v4.bf16x2
  unsigned long long timeout_ns;
  int* err;
};

cudaError_t rs_atomic_probe(const RsProbeParams& p, int blocks, cudaStream_t s);
// out[0] = SM cycles, out[1] = %globaltimer nanoseconds over a spin of `ns` nanoseconds
cudaError_t clock_calibration(unsigned long long ns, long long* out, cudaStream_t s);

}  // namespace cob
