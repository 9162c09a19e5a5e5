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
//     counted;
//   * line atomicity (the reference's M8 premise test, exp/M8_ll128_atomic_a100/test_ll128_atomic.cu:24-50,
//     extended to the store forms that LL128-style protocols rely on), bounded by one deadline.
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
  // emulated ranks read their own input at rank * x_rank_bytes; a real rank's x is its own input
  const char* xb = reinterpret_cast<const char*>(p.x) + (p.emulate ? (size_t)rank * p.x_rank_bytes : 0);
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
__device__ __forceinline__ uint32_t mm_ld_reduce_add_u32(const void* mc) {
  uint32_t v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.u32 %0, [%1];" : "=r"(v) : "l"(mc) : "memory");
  return v;
}
__device__ __forceinline__ void mm_st_u32(void* mc, uint32_t v) {
  asm volatile("multimem.st.relaxed.sys.global.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
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
  if (p.mode == kRsNvls || p.mode == kAgNvls) {
    // same thread -> in-slice index mapping on every rank, so block b's barrier covers every word
    // that block b then reads
    if (p.mode == kRsNvls) {
      for (int d = 0; d < W; ++d)
        for (int i = tid; i < S; i += nthreads) stage(rank)[d * S + i] = prim_word(rank, d * S + i, e);
    } else {
      for (int i = tid; i < S; i += nthreads)
        mm_st_u32(p.mc + p.stage_off + ((size_t)slot * p.n + (size_t)rank * S + i) * 4, prim_word(rank, rank * S + i, e));
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {  // multicast barrier of block b: one add per rank and call
      // counters [0, K) gather every rank's adds; [K, 2K) count this rank's multicast calls of each
      // block locally, so that calls of the other modes (and grids) in between need no matching adds
      const size_t off = (size_t)p.nvls_off + (size_t)blockIdx.x * 4;
      uint32_t* calls = reinterpret_cast<uint32_t*>(mine + p.nvls_off) + kPrimMaxBlocks + blockIdx.x;
      const uint32_t nc = *calls + 1u;
      mm_red_add_u32(p.mc + off, 1u);
      const uint32_t target = nc * (uint32_t)W;
      uint32_t spins = 0;
      while ((int)(ld_acquire_u32(p.base[rank] + off) - target) < 0) {
        if (expired(spins)) {
          atomicOr(p.err, 1);
          break;
        }
      }
      *calls = nc;
    }
    __syncthreads();
    if (p.mode == kRsNvls) {
      for (int i = tid; i < S; i += nthreads) {
        const uint32_t acc = mm_ld_reduce_add_u32(p.mc + p.stage_off + ((size_t)slot * p.n + (size_t)rank * S + i) * 4);
        uint32_t want = 0;
        for (int src = 0; src < W; ++src) want += prim_word(src, rank * S + i, e);
        bad += acc != want;
      }
    } else {
      for (int src = 0; src < W; ++src)
        for (int i = tid; i < S; i += nthreads) bad += ld_vol_u32p(stage(rank) + src * S + i) != prim_word(src, src * S + i, e);
    }
  } else if (p.mode == kAgPull || p.mode == kRsPull) {
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

// ----------------------------------------------------------------------------- line atomicity
constexpr int kLineThreads = 256;

__device__ __forceinline__ void red_sys_add_u32(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_sys_v4(uint32_t* p, const uint4& v) {
  asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t ld_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_sys_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}

// expected final word w of line l (store modes: epoch e; atomic mode: W - 1 writers other than target)
__device__ __forceinline__ uint32_t line_expect(const LineProbeParams& p, long long l, int w) {
  if (p.mode == kLineAtomic)
    return w == 31 ? (uint32_t)(p.world - 1) : (uint32_t)(p.world * (p.world + 1) / 2 - (p.target + 1));
  return w == 31 ? p.epoch : prim_word(w, (int)l, p.epoch);
}

// writer `widx` (0 .. W-2, the ranks other than the target in order) with `nwb` blocks, this block `wb`
template <int MODE>
__device__ void line_write(const LineProbeParams& p, int widx, int wb, int nwb) {
  uint32_t* lines = reinterpret_cast<uint32_t*>(p.base[p.target] + p.lines_off);
  const int lane = threadIdx.x & 31;
  const long long warp = (long long)wb * (kLineThreads / 32) + (threadIdx.x >> 5);
  const long long nwarps = (long long)nwb * (kLineThreads / 32);
  const int wrank = widx < p.target ? widx : widx + 1;
  const int nw = p.world - 1;
  if (MODE == kLineAtomic) {
    const uint32_t add = lane == 31 ? 1u : (uint32_t)(wrank + 1);
    for (long long l = warp; l < p.n_lines; l += nwarps) red_sys_add_u32(lines + l * 32 + lane, add);
  } else if (MODE == kLineStore4) {
    // this writer's lines: widx, widx + nw, widx + 2 nw, ...
    for (long long j = warp;; j += nwarps) {
      const long long l = widx + j * nw;
      if (l >= p.n_lines) break;
      st_sys_u32(lines + l * 32 + lane, line_expect(p, l, lane));
    }
  } else {
    // 8 lanes per line, 4 lines per warp instruction
    const int sub = lane >> 3, q = lane & 7;
    for (long long j0 = warp * 4;; j0 += nwarps * 4) {
      if (widx + j0 * nw >= p.n_lines) break;  // uniform across the warp
      const long long l = widx + (j0 + sub) * nw;
      if (l < p.n_lines)
        st_sys_v4(lines + l * 32 + 4 * q, make_uint4(line_expect(p, l, 4 * q), line_expect(p, l, 4 * q + 1),
                                                      line_expect(p, l, 4 * q + 2), line_expect(p, l, 4 * q + 3)));
    }
  }
}

template <int MODE>
__device__ void line_observe(const LineProbeParams& p, int ob, int nob) {
  const uint32_t* lines = reinterpret_cast<const uint32_t*>(p.base[p.target] + p.lines_off);
  const int lane = threadIdx.x & 31;
  const long long warp = (long long)ob * (kLineThreads / 32) + (threadIdx.x >> 5);
  const long long nwarps = (long long)nob * (kLineThreads / 32);
  const uint32_t want_flag = line_expect(p, 0, 31);
  unsigned long long viol = 0, raced = 0, tmo = 0, seen = 0;
  const uint64_t t0 = globaltimer();
  bool expired = false;
  for (long long l = warp; l < p.n_lines; l += nwarps) {
    if (expired) {
      ++tmo;  // not read: the deadline passed
      continue;
    }
    for (uint32_t spin = 0;; ++spin) {
      bool bad = false;
      uint32_t flag;
      if (MODE == kLineStore16) {
        // one 16-byte load per lane covers the line with lanes 0..7 (lanes 8..31 re-read it)
        const uint4 v = ld_sys_v4(lines + l * 32 + 4 * (lane & 7));
        flag = __shfl_sync(0xffffffffu, v.w, 7);
        const int w = 4 * (lane & 7);
        bad = v.x != line_expect(p, l, w) || v.y != line_expect(p, l, w + 1) || v.z != line_expect(p, l, w + 2) ||
              (w + 3 != 31 && v.w != line_expect(p, l, w + 3));
      } else {
        const uint32_t v = ld_sys_u32(lines + l * 32 + lane);
        flag = __shfl_sync(0xffffffffu, v, 31);
        bad = lane != 31 && v != line_expect(p, l, lane);
      }
      if (flag == want_flag) {  // flag comes from one lane: the branch is uniform
        if (__any_sync(0xffffffffu, bad)) ++viol;
        if (spin) ++raced;
        ++seen;
        break;
      }
      if ((spin & 63u) == 63u) {
        const int late = (lane == 0) && (globaltimer() - t0 > p.timeout_ns);
        if (__shfl_sync(0xffffffffu, late, 0)) {
          expired = true;
          ++tmo;
          break;
        }
      }
    }
  }
  if (lane == 0) {
    if (viol) atomicAdd(p.counters + 0, viol);
    if (raced) atomicAdd(p.counters + 1, raced);
    if (tmo) atomicAdd(p.counters + 2, tmo);
    if (seen) atomicAdd(p.counters + 3, seen);
  }
}

template <int MODE>
__global__ void __launch_bounds__(kLineThreads) k_line(const LineProbeParams p) {
  int b = blockIdx.x;
  if (p.emulate) {
    if (b < p.observer_blocks) {
      line_observe<MODE>(p, b, p.observer_blocks);
    } else {
      b -= p.observer_blocks;
      line_write<MODE>(p, b / p.writer_blocks, b % p.writer_blocks, p.writer_blocks);
    }
  } else if (p.rank == p.target) {
    line_observe<MODE>(p, b, p.observer_blocks);
  } else {
    line_write<MODE>(p, p.rank < p.target ? p.rank : p.rank - 1, b, p.writer_blocks);
  }
}

__global__ void __launch_bounds__(kLineThreads) k_line_check(const LineProbeParams p) {
  const uint32_t* lines = reinterpret_cast<const uint32_t*>(p.base[p.target] + p.lines_off);
  const int lane = threadIdx.x & 31;
  const long long warp = (long long)blockIdx.x * (kLineThreads / 32) + (threadIdx.x >> 5);
  const long long nwarps = (long long)gridDim.x * (kLineThreads / 32);
  unsigned long long bad = 0;
  for (long long l = warp; l < p.n_lines; l += nwarps)
    bad += __any_sync(0xffffffffu, ld_sys_u32(lines + l * 32 + lane) != line_expect(p, l, lane)) ? 1 : 0;
  if (lane == 0 && bad) atomicAdd(p.counters + 4, bad);
}

}  // namespace

cudaError_t line_probe(const LineProbeParams& p, cudaStream_t s) {
  if (p.world < 2 || p.world > 8 || p.target < 0 || p.target >= p.world || p.mode < 0 || p.mode > 2)
    return cudaErrorInvalidValue;
  if (p.n_lines < 1 || p.n_lines > (1LL << 24) || p.lines_off < 0 || p.lines_off % 128) return cudaErrorInvalidValue;
  if (p.observer_blocks < 1 || p.observer_blocks > 1024 || p.writer_blocks < 1 || p.writer_blocks > 4096)
    return cudaErrorInvalidValue;
  if (p.mode != kLineAtomic && p.epoch == 0) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(p.base[p.target]) % 16 || !p.counters) return cudaErrorInvalidValue;
  if (!p.emulate && (p.rank < 0 || p.rank >= p.world)) return cudaErrorInvalidValue;
  void (*k)(const LineProbeParams) = p.mode == kLineAtomic ? k_line<kLineAtomic>
                                     : p.mode == kLineStore4 ? k_line<kLineStore4> : k_line<kLineStore16>;
  int blocks = 0;
  if (p.emulate) {
    blocks = p.observer_blocks + (p.world - 1) * p.writer_blocks;
    // the observer spins on lines written by other blocks of this launch: all must be resident
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kLineThreads, 0);
    if (e != cudaSuccess) return e;
    if ((long long)blocks > (long long)sms * per_sm) return cudaErrorInvalidValue;
  } else {
    blocks = p.rank == p.target ? p.observer_blocks : p.writer_blocks;
  }
  k<<<blocks, kLineThreads, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t line_check(const LineProbeParams& p, cudaStream_t s) {
  if (p.world < 2 || p.world > 8 || p.target < 0 || p.target >= p.world || p.n_lines < 1 || p.n_lines > (1LL << 24) ||
      p.lines_off % 128 || !p.counters || (p.mode != kLineAtomic && p.epoch == 0))
    return cudaErrorInvalidValue;
  const long long want = (p.n_lines + kLineThreads / 32 - 1) / (kLineThreads / 32);
  k_line_check<<<(int)(want < 1184 ? want : 1184), kLineThreads, 0, s>>>(p);
  return cudaGetLastError();
}

size_t prim_heap_bytes(int world, int n, long long* flags_off, long long* stage_off, long long* land_off,
                       long long* nvls_off) {
  auto up = [](long long v) { return (v + 4095) / 4096 * 4096; };
  *flags_off = up(8LL * kPrimMaxBlocks);
  *nvls_off = *flags_off + up(8LL * kPrimMaxBlocks * 8);
  *stage_off = *nvls_off + up(8LL * kPrimMaxBlocks);  // barrier counters, then local call counts
  *land_off = *stage_off + up(2LL * n * 4);
  return (size_t)(*land_off + up(2LL * 8 * (n / world) * 4));
}

cudaError_t prim_probe(const PrimParams& p, int blocks, int threads, cudaStream_t s) {
  if (p.world < 1 || p.world > 8 || p.n <= 0 || p.n % p.world || p.mode < 0 || p.mode > 5) return cudaErrorInvalidValue;
  if ((p.mode == kRsNvls || p.mode == kAgNvls) && (p.mc == nullptr || p.emulate)) return cudaErrorNotSupported;
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
