// Shared device helpers for the sm_100a kernels of comm_opt_b200.
//
// Everything here is written for Blackwell (sm_100a): 16-byte vector moves over NVLink 5 peer
// mappings, system-scope relaxed/acquire/release accesses for cross-GPU flags, NVSwitch multicast
// (`multimem.*`) for in-switch reductions, `%globaltimer`-bounded waits that report an error word
// instead of hanging, and programmatic-dependent-launch (PDL) hooks.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "types.h"

namespace cob {

// ---------------------------------------------------------------------------------------------
// dtypes
// ---------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// 16-byte vector <-> fp32 conversion for each element type. N = elements per 16-byte vector.
template <typename T>
struct Vec;

template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void to_float(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};

template <>
struct Vec<__half> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void to_float(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void to_float(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // bf16 -> fp32 is a 16-bit left shift of the bit pattern
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  __device__ __forceinline__ static uint4 from_float(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

// ---------------------------------------------------------------------------------------------
// Lamport-style "value carries its own arrival" encoding.
//
// A landing buffer is pre-filled with negative zero (a bit pattern a sender never writes: senders
// turn -0 into +0, which changes no sum). A receiver polls a 16-byte vector until none of its
// elements is -0. Only per-element single-copy atomicity is assumed (every scalar element of a
// vector store is written atomically), not 16- or 128-byte atomicity. After use the receiver
// writes -0 back so the slot is ready for the call two epochs later.
// ---------------------------------------------------------------------------------------------
template <int EBITS>
struct Lamport;

template <>
struct Lamport<16> {
  static constexpr uint32_t kFill = 0x80008000u;
  __device__ __forceinline__ static bool ready_word(uint32_t w) {
    return ((w & 0xFFFFu) != 0x8000u) && ((w >> 16) != 0x8000u);
  }
  __device__ __forceinline__ static uint32_t clean_word(uint32_t w) {
    if ((w & 0xFFFFu) == 0x8000u) w &= 0xFFFF0000u;
    if ((w >> 16) == 0x8000u) w &= 0x0000FFFFu;
    return w;
  }
};

template <>
struct Lamport<32> {
  static constexpr uint32_t kFill = 0x80000000u;
  __device__ __forceinline__ static bool ready_word(uint32_t w) { return w != 0x80000000u; }
  __device__ __forceinline__ static uint32_t clean_word(uint32_t w) { return w == 0x80000000u ? 0u : w; }
};

template <typename T>
struct LamportOf : Lamport<sizeof(T) * 8> {
  __device__ __forceinline__ static bool ready(const uint4& v) {
    return LamportOf::ready_word(v.x) && LamportOf::ready_word(v.y) && LamportOf::ready_word(v.z) &&
           LamportOf::ready_word(v.w);
  }
  __device__ __forceinline__ static uint4 clean(const uint4& v) {
    return make_uint4(LamportOf::clean_word(v.x), LamportOf::clean_word(v.y), LamportOf::clean_word(v.z),
                      LamportOf::clean_word(v.w));
  }
  __device__ __forceinline__ static uint4 fill() {
    return make_uint4(LamportOf::kFill, LamportOf::kFill, LamportOf::kFill, LamportOf::kFill);
  }
};

// ---------------------------------------------------------------------------------------------
// memory operations
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// The same clock for phase stamps: the memory clobber keeps the read in program order with the
// surrounding barriers and memory operations (a plain read may be scheduled ahead of a barrier).
__device__ __forceinline__ uint64_t globaltimer_ordered() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)::"memory");
  return t;
}

__device__ __forceinline__ uint4 ld_vol_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_vol_v4(void* p, const uint4& v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
// read-only path for inputs that no other agent writes during the kernel
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint64_t ld_vol_u64(const void* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_vol_u64(void* p, uint64_t v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_vol_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_acquire_u64(const void* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(void* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// NVSwitch multicast (NVLS). `mc` addresses are inside a multicast object bound to every rank's heap.
template <typename T>
__device__ __forceinline__ uint4 mm_ld_reduce(const void* mc);
template <>
__device__ __forceinline__ uint4 mm_ld_reduce<__nv_bfloat16>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
template <>
__device__ __forceinline__ uint4 mm_ld_reduce<__half>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
template <>
__device__ __forceinline__ uint4 mm_ld_reduce<float>(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void mm_st_v4(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_st_u64(void* mc, uint64_t v) {
  asm volatile("multimem.st.relaxed.sys.global.u64 [%0], %1;" ::"l"(mc), "l"(v) : "memory");
}
__device__ __forceinline__ void mm_red_add_u32(void* mc, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

// Programmatic dependent launch. Both are no-ops when the kernel was not launched with PDL.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Wait for the predecessor, then let the successor launch at once. The successor's CTAs become
// resident beside this kernel's (where resources allow) and run their prologue - barrier set-up,
// tensor-map prefetch, the first weight tiles of a GEMM - while this kernel works; they touch
// nothing this kernel reads or writes before their own pdl_wait(), which returns only after this
// grid has completed. Triggering after (never before) the wait keeps at most two kernels of a
// stream in flight: when a kernel starts, every kernel before its predecessor has completed.
__device__ __forceinline__ void pdl_wait_then_trigger() {
  pdl_wait();
  pdl_trigger();
}

// Process-wide switch: launch every kernel with programmatic stream serialization, so consecutive
// kernels in a stream or CUDA graph overlap launch latency and prologue. Every kernel of this
// library calls pdl_wait() before it reads data produced by (or writes data read by) its
// predecessor. Defined in decode_ops.cu.
bool& pdl_flag();
// Process-wide: weight tiles beyond its shared-memory ring that a GEMM prefetches into L2 before it waits
// for its activations (the previous kernel, or the all-reduce pieces); 0 = none. Defined in decode_ops.cu.
int& l2_prefetch_tiles();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl_flag()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------------------------
// thread-block cluster primitives (distributed shared memory)
// ---------------------------------------------------------------------------------------------
// Cluster barrier split into arrive and wait. The release form orders every earlier memory access of
// the thread, remote NVLink stores included, so it waits until they are acknowledged; the relaxed
// form orders nothing and costs only the barrier itself.
__device__ __forceinline__ void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
// Shared-memory address of `p` (this CTA) as seen in CTA `cta` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(const void* p, int cta) {
  uint32_t out;
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(a), "r"(cta));
  return out;
}
// 64-bit words of this CTA's shared memory that other CTAs of the cluster poll: relaxed at cluster
// scope, so a word is seen whole (single-copy atomic) and eventually, without ordering anything else.
__device__ __forceinline__ void st_cluster_word(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.cluster.shared::cta.u64 [%0], %1;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))),
               "l"(v)
               : "memory");
}
__device__ __forceinline__ unsigned long long ld_cluster_word(uint32_t cluster_addr) {
  unsigned long long v;
  asm volatile("ld.relaxed.cluster.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// Block-wide sum with a fixed reduction tree (identical result in every block and on every rank for
// identical inputs). `scratch` needs blockDim.x/32 floats. Ends with the result broadcast.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < nw ? scratch[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// ---------------------------------------------------------------------------------------------
// bounded waits
// ---------------------------------------------------------------------------------------------
// Error bits in RankState::error. A kernel that gives up on a wait sets a bit, records where in
// err_detail, and returns; the host reads the word and raises.
// Checked build (COB_CHECKED=1 at build time): every heap address the collective kernels form is
// range-checked; an out-of-range index sets kErrBounds in the rank's error word and the access goes to
// a private scratch line instead of faulting the GPU. Off by default (no code in the hot path).
#ifdef COB_CHECKED
static __device__ __align__(16) unsigned char g_cob_oob_scratch[256];  // one per translation unit
static __device__ unsigned int g_cob_oob_count;
#define COB_IN_RANGE(ptr_expr, ok_expr, err_word)                                        \
  ((ok_expr) ? (ptr_expr)                                                                \
             : (atomicOr((err_word), (unsigned int)cob::kErrBounds), atomicAdd(&g_cob_oob_count, 1u), \
                reinterpret_cast<decltype(ptr_expr)>(g_cob_oob_scratch)))
#else
#define COB_IN_RANGE(ptr_expr, ok_expr, err_word) (ptr_expr)
#endif

enum ErrBits : uint32_t {
  kErrTimeoutLanding = 1u << 0,
  kErrTimeoutFlag = 1u << 1,
  kErrTimeoutNvls = 1u << 2,
  kErrTimeoutPartial = 1u << 3,
  kErrBadArgs = 1u << 4,
  kErrTimeoutGather = 1u << 5,
  kErrTimeoutGrid = 1u << 6,
  kErrBounds = 1u << 7,  // checked build only: an index was out of range (the access was skipped)
};

// Per-thread wait budget: cheap spin count, then a %globaltimer deadline. Also gives up early when
// another thread of this rank has already recorded an error (so one stuck peer costs one timeout).
struct Waiter {
  uint64_t deadline;
  uint32_t spins;
  uint64_t timeout_ns;
  const volatile uint32_t* err;
  __device__ __forceinline__ Waiter(uint64_t timeout, const uint32_t* err_word)
      : deadline(0), spins(0), timeout_ns(timeout), err(err_word) {}
  // true -> give up
  __device__ __forceinline__ bool expired() {
    if ((++spins & 255u) != 0u) return false;
    if (*err != 0u) return true;
    const uint64_t t = globaltimer();
    if (deadline == 0) {
      deadline = t + timeout_ns;
      return false;
    }
    return t > deadline;
  }
};

}  // namespace cob
