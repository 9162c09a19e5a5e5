// Primitive probes used to choose algorithms on NVLink 5 (the reference's M8/M11 probes,
// exp/M11_before_prototype/rs_probe.cu and exp/M8_ll128_atomic_a100/*, re-designed for sm_100a):
//   * reduce-scatter by remote atomics: every rank adds its slice for owner d straight into d's
//     accumulator with `red.global.add` - scalar f32, 16-byte vector f32 (red.v4.f32), scalar bf16x2
//     and 16-byte vector bf16x2 (red.v4.bf16x2; native on sm_90+, CAS-emulated on the reference's A100);
//     completion through a per-owner arrival counter, bounded wait, error word on timeout;
//   * clock calibration: SM cycles per %globaltimer nanosecond.
#include "common.cuh"
#include "probes.h"

namespace cob {
namespace {

__device__ __forceinline__ void red_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
__device__ __forceinline__ void red_v4_f32(float* p, const float4& v) {
  asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void red_bf16x2(void* p, uint32_t v) {
  asm volatile("red.global.add.noftz.bf16x2 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_v4_bf16x2(void* p, const uint4& v) {
  asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__global__ void __launch_bounds__(256) k_rs_atomic(const RsProbeParams p) {
  const int rank = p.emulate ? (int)blockIdx.y : p.rank;
  const int W = p.world;
  const char* xb = reinterpret_cast<const char*>(p.x) + (size_t)rank * p.x_rank_bytes;
  const int es = p.variant <= 1 ? 4 : 2;
  const size_t slice_bytes = (size_t)p.n * es;
  pdl_wait();
  // push: this rank's slice for every owner, added into the owner's accumulator
  for (int d0 = 0; d0 < W; ++d0) {
    const int d = (rank + d0) % W;
    char* acc = p.base[d] + p.acc_off;
    const char* src = xb + (size_t)d * slice_bytes;
    if (p.variant == 0) {
      for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n; i += gridDim.x * blockDim.x)
        red_f32(reinterpret_cast<float*>(acc) + i, reinterpret_cast<const float*>(src)[i]);
    } else if (p.variant == 1) {
      for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n / 4; i += gridDim.x * blockDim.x)
        red_v4_f32(reinterpret_cast<float*>(acc) + 4 * i, reinterpret_cast<const float4*>(src)[i]);
    } else if (p.variant == 2) {
      for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n / 2; i += gridDim.x * blockDim.x)
        red_bf16x2(reinterpret_cast<uint32_t*>(acc) + i, reinterpret_cast<const uint32_t*>(src)[i]);
    } else {
      for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n / 8; i += gridDim.x * blockDim.x)
        red_v4_bf16x2(reinterpret_cast<uint4*>(acc) + i, reinterpret_cast<const uint4*>(src)[i]);
    }
  }
  // arrival: make this block's additions visible system-wide, then count it at every owner
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < (unsigned)W) {
    unsigned int* ctr = reinterpret_cast<unsigned int*>(p.base[threadIdx.x] + p.ctr_off);
    atomicAdd_system(ctr, 1u);
  }
  // owner: wait until every block of every rank has arrived (bounded)
  if (threadIdx.x == 0) {
    const unsigned int* mine = reinterpret_cast<const unsigned int*>(p.base[rank] + p.ctr_off);
    const unsigned int target = (unsigned)W * gridDim.x;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_u32(mine) < target) {
      if (globaltimer() - t0 > p.timeout_ns) {
        atomicOr(p.err, 1);
        break;
      }
    }
  }
}

__global__ void k_clock_calib(unsigned long long ns, long long* out) {
  const uint64_t t0 = globaltimer();
  const long long c0 = clock64();
  uint64_t t = t0;
  while (t - t0 < ns) t = globaltimer();
  out[0] = clock64() - c0;
  out[1] = (long long)(t - t0);
}

}  // namespace

cudaError_t rs_atomic_probe(const RsProbeParams& p, int blocks, cudaStream_t s) {
  if (p.world < 1 || p.world > 8 || p.variant < 0 || p.variant > 3 || p.n <= 0 || p.n % 8) return cudaErrorInvalidValue;
  return launch_k(k_rs_atomic, dim3(blocks, p.emulate ? p.world : 1), dim3(256), 0, s, p);
}

cudaError_t clock_calibration(unsigned long long ns, long long* out, cudaStream_t s) {
  k_clock_calib<<<1, 1, 0, s>>>(ns, out);
  return cudaGetLastError();
}

}  // namespace cob
