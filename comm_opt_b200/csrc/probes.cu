// Primitive probes used to choose algorithms on NVLink 5 (the reference's M8/M11 probes,
// exp/M11_before_prototype/rs_probe.cu and exp/M8_ll128_atomic_a100/*, re-designed for sm_100a):
//   * reduce-scatter by remote atomics: every rank adds its slice for owner d straight into d's
//     accumulator with `red.global.add` - scalar f32, 16-byte vector f32 (red.v4.f32), scalar bf16x2
//     and 16-byte vector bf16x2 (red.v4.bf16x2; native on sm_90+, CAS-emulated on the reference's A100);
//     completion through a per-owner arrival counter, bounded wait, error word on timeout;
//   * clock calibration: SM cycles per %globaltimer nanosecond;
//   * push vs pull primitives (the reference's LL128 probes, exp/M12_push_vs_pull/ll128_probe.cu:101-183,
//     and steady-state probe, exp/M13_push_retest/m13_probe.cu:120-215): all-gather and reduce-scatter
//     of 32-bit words in pull form (stage locally, flag barrier, load from peers) and push form (store
//     into the peers' landing words, poll own landing). Arrival is per 32-bit word (Lamport sentinel),
//     not per 128-byte line; launches reuse the buffers without clearing (epoch-parity slots, cleared
//     on consumption) and the payload is a hash of (rank, index, epoch), so any stale or torn word is
//     counted.
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


// ----------------------------------------------------------------------------- push / pull primitives
__host__ __device__ __forceinline__ uint32_t prim_word(int rank, int i, uint64_t e) {
  // splitmix-style mix of (rank, index, epoch); never the sentinel 0x80000000
  uint64_t z = ((uint64_t)rank << 40) ^ ((uint64_t)(uint32_t)i << 8) ^ (e * 0xD1B54A32D192ED03ull);
  z ^= z >> 31;
  z *= 0x94D049BB133111EBull;
  z ^= z >> 29;
  const uint32_t w = (uint32_t)z;
  return w == 0x80000000u ? 0x80000001u : w;
}

__device__ __forceinline__ uint32_t ld_vol_u32p(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_vol_u32p(uint32_t* p, uint32_t v) {
  asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(1024) k_prim(const PrimParams p) {
  const int rank = p.emulate ? (int)blockIdx.y : p.rank;
  const int W = p.world, S = p.n / W;  // slice of every rank
  char* mine = p.base[rank];
  unsigned long long* ep = reinterpret_cast<unsigned long long*>(mine);
  pdl_wait();
  const uint64_t e = ld_vol_u64(&ep[blockIdx.x]) + 1;
  const int slot = (int)(e & 1);
  auto stage = [&](int r) { return reinterpret_cast<uint32_t*>(p.base[r] + p.stage_off) + (size_t)slot * p.n; };
  auto land = [&](int owner, int src) {
    return reinterpret_cast<uint32_t*>(p.base[owner] + p.land_off) + ((size_t)slot * 8 + src) * S;
  };
  const int tid = blockIdx.x * blockDim.x + threadIdx.x, nthreads = gridDim.x * blockDim.x;
  unsigned int bad = 0;
  bool ok = true;
  uint64_t t0 = 0;
  auto expired = [&](uint32_t& spins) {
    if ((++spins & 255u) != 0u) return false;
    const uint64_t t = globaltimer();
    if (t0 == 0) t0 = t;
    return t - t0 > p.timeout_ns;
  };
  if (p.mode == kAgPull || p.mode == kRsPull) {
    // stage: AG contributes this rank's slice, RS the whole vector, slice by slice, so that thread
    // `tid` of every rank handles the same in-slice indices (the flag barrier is per block)
    for (int d = (p.mode == kAgPull ? rank : 0); d < (p.mode == kAgPull ? rank + 1 : W); ++d)
      for (int i = tid; i < S; i += nthreads) stage(rank)[d * S + i] = prim_word(rank, d * S + i, e);
    __threadfence_system();
    __syncthreads();
    // flag barrier among block b of every rank (the index sets below are the same per block)
    if (threadIdx.x < (unsigned)W) {
      unsigned long long* dst =
          reinterpret_cast<unsigned long long*>(p.base[threadIdx.x] + p.flags_off) + (size_t)blockIdx.x * 8 + rank;
      st_release_u64(dst, e);
      const unsigned long long* f =
          reinterpret_cast<unsigned long long*>(mine + p.flags_off) + (size_t)blockIdx.x * 8 + threadIdx.x;
      uint32_t spins = 0;
      while ((long long)(ld_acquire_u64(f) - e) < 0) {
        if (expired(spins)) {
          atomicOr(p.err, 1);
          break;
        }
      }
    }
    __syncthreads();
    if (p.mode == kAgPull) {
      // same thread -> index mapping as the staging loop: every word read was staged by block b
      for (int s0 = 0; s0 < W; ++s0) {
        const int src = (rank + s0) % W;
        for (int i = tid; i < S; i += nthreads) bad += ld_vol_u32p(stage(src) + src * S + i) != prim_word(src, src * S + i, e);
      }
    } else {
      for (int i = tid; i < S; i += nthreads) {
        uint32_t acc = 0, want = 0;
        for (int s0 = 0; s0 < W; ++s0) {
          const int src = (rank + s0) % W;
          acc += ld_vol_u32p(stage(src) + rank * S + i);
          want += prim_word(src, rank * S + i, e);
        }
        bad += acc != want;
      }
    }
  } else {
    // push: AG stores this rank's slice into every rank's land[.][rank]; RS stores slice d into d
    if (p.mode == kAgPush) {
      for (int i = tid; i < S; i += nthreads) {
        const uint32_t w = prim_word(rank, rank * S + i, e);
        for (int d0 = 0; d0 < W; ++d0) st_vol_u32p(land((rank + d0) % W, rank) + i, w);
      }
    } else {
      for (int d0 = 0; d0 < W; ++d0) {
        const int d = (rank + d0) % W;
        for (int i = tid; i < S; i += nthreads) st_vol_u32p(land(d, rank) + i, prim_word(rank, d * S + i, e));
      }
    }
    // receive: poll own landing words (sentinel = not yet arrived), check, restore the sentinel
    for (int i = tid; i < S; i += nthreads) {
      uint32_t acc = 0, want = 0;
      for (int s0 = 0; s0 < W && ok; ++s0) {
        const int src = (rank + s0) % W;
        uint32_t* a = land(rank, src) + i;
        uint32_t v = ld_vol_u32p(a), spins = 0;
        while (v == 0x80000000u) {
          if (expired(spins)) {
            atomicOr(p.err, 1);
            ok = false;
            break;
          }
          v = ld_vol_u32p(a);
        }
        st_vol_u32p(a, 0x80000000u);
        if (p.mode == kAgPush) {
          bad += v != prim_word(src, src * S + i, e);
        } else {
          acc += v;
          want += prim_word(src, rank * S + i, e);
        }
      }
      if (p.mode == kRsPush) bad += acc != want;
    }
  }
  if (bad) atomicAdd(p.bad + (p.emulate ? rank : 0), bad);
  // next call's epoch (read only after this grid completed)
  for (int j = blockIdx.x + (int)threadIdx.x * (int)gridDim.x; j < kPrimMaxBlocks; j += (int)(blockDim.x * gridDim.x))
    ep[j] = e;
}

}  // namespace

size_t prim_heap_bytes(int world, int n, long long* flags_off, long long* stage_off, long long* land_off) {
  auto up = [](long long v) { return (v + 4095) / 4096 * 4096; };
  *flags_off = up(8LL * kPrimMaxBlocks);
  *stage_off = *flags_off + up(8LL * kPrimMaxBlocks * 8);
  *land_off = *stage_off + up(2LL * n * 4);
  return (size_t)(*land_off + up(2LL * 8 * (n / world) * 4));
}

cudaError_t prim_probe(const PrimParams& p, int blocks, int threads, cudaStream_t s) {
  if (p.world < 1 || p.world > 8 || p.n <= 0 || p.n % p.world || p.mode < 0 || p.mode > 3) return cudaErrorInvalidValue;
  if (blocks < 1 || blocks > kPrimMaxBlocks || threads < 32 || threads > 1024 || threads % 32) return cudaErrorInvalidValue;
  // blocks wait for blocks of other ranks (and, emulated, of the same launch): all must be resident
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_prim, threads, 0);
  if (e != cudaSuccess) return e;
  if ((long long)blocks * (p.emulate ? p.world : 1) > (long long)sms * per_sm) return cudaErrorInvalidValue;
  return launch_k(k_prim, dim3(blocks, p.emulate ? p.world : 1), dim3(threads), 0, s, p);
}

cudaError_t rs_atomic_probe(const RsProbeParams& p, int blocks, cudaStream_t s) {
  if (p.world < 1 || p.world > 8 || p.variant < 0 || p.variant > 3 || p.n <= 0 || p.n % 8) return cudaErrorInvalidValue;
  return launch_k(k_rs_atomic, dim3(blocks, p.emulate ? p.world : 1), dim3(256), 0, s, p);
}

cudaError_t clock_calibration(unsigned long long ns, long long* out, cudaStream_t s) {
  k_clock_calib<<<1, 1, 0, s>>>(ns, out);
  return cudaGetLastError();
}

}  // namespace cob
