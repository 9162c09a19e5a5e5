// Single-GPU decode kernels: RMSNorm, add+RMSNorm, embedding, RoPE + paged-KV append, SiLU*mul,
// greedy argmax. Memory-bound elementwise work: 16-byte vector loads, one pass over the data,
// programmatic-dependent-launch wait at the top so a graph of decode kernels overlaps prologues.
#include <float.h>

#include <algorithm>

#include "common.cuh"
#include "ops.h"

namespace cob {

bool& pdl_flag() {
  static bool on = false;
  return on;
}

int& l2_prefetch_tiles() {
  static int tiles = 0;
  return tiles;
}

namespace {

constexpr int kVPT = 4;

template <typename T, bool ADD, int VPT>
__global__ void __launch_bounds__(512) k_rmsnorm(const T* __restrict__ x, T* __restrict__ residual,
                                                 const T* __restrict__ gamma, T* __restrict__ out, int hidden,
                                                 float eps) {
  using V = Vec<T>;
  __shared__ float scr[32];
  pdl_wait();
  const int row = blockIdx.x, hv = hidden / V::N;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * hidden);
  uint4* rr = ADD ? reinterpret_cast<uint4*>(residual + (size_t)row * hidden) : nullptr;
  float h[VPT][V::N];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * blockDim.x;
    if (v < hv) {
      float a[V::N];
      V::to_float(xr[v], a);
      if (ADD) {
        float r[V::N];
        V::to_float(rr[v], r);
#pragma unroll
        for (int i = 0; i < V::N; ++i) a[i] += r[i];
        const uint4 hb = V::from_float(a);
        rr[v] = hb;
        V::to_float(hb, a);
      }
#pragma unroll
      for (int i = 0; i < V::N; ++i) {
        h[k][i] = a[i];
        ss += a[i] * a[i];
      }
    }
  }
  pdl_trigger();
  const float rstd = rsqrtf(block_sum(ss, scr) / (float)hidden + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * hidden);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * blockDim.x;
    if (v < hv) {
      float g[V::N], o[V::N];
      V::to_float(reinterpret_cast<const uint4*>(gamma)[v], g);
#pragma unroll
      for (int i = 0; i < V::N; ++i) o[i] = h[k][i] * rstd * g[i];
      orow[v] = V::from_float(o);
    }
  }
}

template <typename T>
__global__ void k_embedding(const int32_t* __restrict__ ids, const T* __restrict__ table, T* __restrict__ out,
                            int hidden) {
  pdl_wait_then_trigger();
  const int row = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)ids[row] * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)row * hidden);
  const int hv = hidden * (int)sizeof(T) / 16;
  for (int v = threadIdx.x; v < hv; v += blockDim.x) dst[v] = ld_nc_v4(src + v);
}

// One block per (sequence, head): q and k heads are rotated (rotate-half RoPE), q goes to q_out,
// k and v heads go to their slot of the paged cache. `bias` ([(nq + 2 nkv) * D], or nullptr) is the
// QKV projection's bias (Qwen2-style attention), added before the rotation.
template <typename T>
__global__ void __launch_bounds__(64) k_rope_append(const T* __restrict__ qkv, const T* __restrict__ bias,
                                                    const int32_t* __restrict__ positions,
                                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                                    const int32_t* __restrict__ block_tables, int max_blocks,
                                                    T* __restrict__ q_out, T* __restrict__ k_cache,
                                                    T* __restrict__ v_cache, int nq, int nkv, int D, int bs) {
  pdl_wait_then_trigger();
  const int b = blockIdx.x, head = blockIdx.y;
  const int pos = positions[b];
  const int half = D / 2;
  const T* src = qkv + ((size_t)b * (nq + 2 * nkv) + head) * D;
  const T* bh = bias ? bias + (size_t)head * D : nullptr;
  T* dst;
  if (head < nq) {
    dst = q_out + ((size_t)b * nq + head) * D;
  } else {
    const int blk = block_tables[(size_t)b * max_blocks + pos / bs], off = pos % bs;
    const int kv = head < nq + nkv ? head - nq : head - nq - nkv;
    T* cache = head < nq + nkv ? k_cache : v_cache;
    dst = cache + (((size_t)blk * nkv + kv) * bs + off) * D;
  }
  if (head < nq + nkv) {
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float c = cos_t[(size_t)pos * half + i], sn = sin_t[(size_t)pos * half + i];
      float x1 = to_f(src[i]), x2 = to_f(src[i + half]);
      if (bh) {
        x1 += to_f(bh[i]);
        x2 += to_f(bh[i + half]);
      }
      dst[i] = from_f<T>(x1 * c - x2 * sn);
      dst[i + half] = from_f<T>(x2 * c + x1 * sn);
    }
  } else {
    for (int i = threadIdx.x; i < D; i += blockDim.x) dst[i] = bh ? from_f<T>(to_f(src[i]) + to_f(bh[i])) : src[i];
  }
}

// il == 0: row = [gate (inter) | up (inter)]; il > 0: blocks of il gate then il up features
// (the decode GEMMs' gate/up interleave), il a multiple of the vector width.
template <typename T>
__global__ void k_silu_mul(const T* __restrict__ gu, T* __restrict__ out, int inter, int il) {
  using V = Vec<T>;
  pdl_wait_then_trigger();
  const int b = blockIdx.y;
  const int iv = inter / V::N, ilv = il / V::N;
  const uint4* row = reinterpret_cast<const uint4*>(gu + (size_t)b * 2 * inter);
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)b * inter);
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < iv; v += gridDim.x * blockDim.x) {
    const int gv = ilv ? (v / ilv) * 2 * ilv + v % ilv : v;
    const int uvec = ilv ? gv + ilv : v + iv;
    float a[V::N], c[V::N], r[V::N];
    V::to_float(row[gv], a);
    V::to_float(row[uvec], c);
#pragma unroll
    for (int i = 0; i < V::N; ++i) r[i] = a[i] / (1.f + __expf(-a[i])) * c[i];
    o[v] = V::from_float(r);
  }
}

// Greedy argmax key: order-preserving 32-bit image of the value in the high word, inverted index in
// the low word, so the maximum key is the largest value and, among equal values, the lowest index.
__device__ __forceinline__ unsigned long long amax_key(float v, uint32_t idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (0xFFFFFFFFu - idx);
}
__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) { return a > b ? a : b; }

constexpr int kArgmaxChunk = 2048;

// grid (rows, chunks of the local vocabulary): each CTA folds its chunk into keys[row] (atomicMax);
// keys must be zero before (argmax_combine clears them)
template <typename T>
__global__ void __launch_bounds__(256) k_argmax_local(const T* __restrict__ logits, unsigned long long* keys,
                                                      int vocab, int vocab_offset) {
  pdl_wait_then_trigger();
  const int row = blockIdx.x;
  const int i0 = blockIdx.y * kArgmaxChunk, i1 = min(vocab, i0 + kArgmaxChunk);
  const T* lr = logits + (size_t)row * vocab;
  unsigned long long best = 0ull;
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) best = umax64(best, amax_key(to_f(lr[i]), i + vocab_offset));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
  __shared__ unsigned long long sk[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sk[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = umax64(best, sk[w]);
    atomicMax(keys + row, best);
  }
}

// keys gathered from every rank [world][rows] -> global greedy id per row; optionally advance the
// decode positions / lengths and clear this rank's local keys for the next step
__global__ void k_argmax_combine(const unsigned long long* __restrict__ gathered, int32_t* __restrict__ ids, int rows,
                                 int world, int32_t* __restrict__ positions, int32_t* __restrict__ seq_lens,
                                 unsigned long long* __restrict__ local_keys) {
  pdl_wait_then_trigger();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  unsigned long long best = 0ull;
  for (int r = 0; r < world; ++r) best = umax64(best, gathered[(size_t)r * rows + row]);
  ids[row] = (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  if (positions) positions[row] += 1;
  if (seq_lens) seq_lens[row] += 1;
  if (local_keys) local_keys[row] = 0ull;
}

template <typename F>
cudaError_t by_dtype(int dtype, F&& f) {
  switch (dtype) {
    case kF32: return f(float{});
    case kF16: return f(__half{});
    case kBF16: return f(__nv_bfloat16{});
    default: return cudaErrorInvalidValue;
  }
}

int threads_for(int hv) {
  int t = 32;
  while (t < 512 && t * kVPT < hv) t *= 2;
  while (t < 512 && t < hv) t *= 2;
  return t;
}

}  // namespace

cudaError_t rmsnorm(const void* x, const void* gamma, void* out, int rows, int hidden, float eps, int dtype,
                    cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    const int hv = hidden / Vec<T>::N;
    if (hidden % Vec<T>::N || hv > 512 * 2 * kVPT || rows <= 0) return cudaErrorInvalidValue;
    auto k = hv > 512 * kVPT ? k_rmsnorm<T, false, 2 * kVPT> : k_rmsnorm<T, false, kVPT>;
    return launch_k(k, dim3(rows), dim3(threads_for(hv)), 0, s, reinterpret_cast<const T*>(x), (T*)nullptr,
                    reinterpret_cast<const T*>(gamma), reinterpret_cast<T*>(out), hidden, eps);
  });
}

cudaError_t add_rmsnorm(const void* x, void* residual, const void* gamma, void* out, int rows, int hidden,
                        float eps, int dtype, cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    const int hv = hidden / Vec<T>::N;
    if (hidden % Vec<T>::N || hv > 512 * 2 * kVPT || rows <= 0) return cudaErrorInvalidValue;
    auto k = hv > 512 * kVPT ? k_rmsnorm<T, true, 2 * kVPT> : k_rmsnorm<T, true, kVPT>;
    return launch_k(k, dim3(rows), dim3(threads_for(hv)), 0, s, reinterpret_cast<const T*>(x),
                    reinterpret_cast<T*>(residual), reinterpret_cast<const T*>(gamma), reinterpret_cast<T*>(out),
                    hidden, eps);
  });
}

cudaError_t embedding(const int32_t* ids, const void* table, void* out, int rows, int hidden, int dtype,
                      cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if ((hidden * (int)sizeof(T)) % 16 || rows <= 0) return cudaErrorInvalidValue;
    return launch_k(k_embedding<T>, dim3(rows), dim3(256), 0, s, ids, reinterpret_cast<const T*>(table),
                    reinterpret_cast<T*>(out), hidden);
  });
}

cudaError_t rope_append_kv(const void* qkv, const void* bias, const int32_t* positions, const float* cos_t,
                           const float* sin_t, const int32_t* block_tables, int max_blocks_per_seq, void* q_out,
                           void* k_cache, void* v_cache, int batch, int nq, int nkv, int head_dim, int block_size,
                           int dtype, cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (batch <= 0 || head_dim % 2) return cudaErrorInvalidValue;
    return launch_k(k_rope_append<T>, dim3(batch, nq + 2 * nkv), dim3(64), 0, s, reinterpret_cast<const T*>(qkv),
                    reinterpret_cast<const T*>(bias), positions, cos_t, sin_t, block_tables, max_blocks_per_seq, reinterpret_cast<T*>(q_out),
                    reinterpret_cast<T*>(k_cache), reinterpret_cast<T*>(v_cache), nq, nkv, head_dim, block_size);
  });
}

cudaError_t silu_mul(const void* gu, void* out, int rows, int inter, int dtype, cudaStream_t s, int interleave) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (inter % Vec<T>::N || rows <= 0 || interleave < 0 || interleave % Vec<T>::N ||
        (interleave > 0 && inter % interleave))
      return cudaErrorInvalidValue;
    const int iv = inter / Vec<T>::N;
    const int bx = std::min(64, (iv + 255) / 256);
    return launch_k(k_silu_mul<T>, dim3(bx, rows), dim3(256), 0, s, reinterpret_cast<const T*>(gu),
                    reinterpret_cast<T*>(out), inter, interleave);
  });
}

cudaError_t argmax_local(const void* logits, unsigned long long* keys, int rows, int vocab, int vocab_offset,
                         int dtype, cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (rows <= 0 || vocab <= 0) return cudaErrorInvalidValue;
    return launch_k(k_argmax_local<T>, dim3(rows, (vocab + kArgmaxChunk - 1) / kArgmaxChunk), dim3(256), 0, s,
                    reinterpret_cast<const T*>(logits), keys, vocab, vocab_offset);
  });
}

cudaError_t argmax_combine(const unsigned long long* gathered, int32_t* ids, int rows, int world, int32_t* positions,
                           int32_t* seq_lens, unsigned long long* local_keys, cudaStream_t s) {
  if (rows <= 0 || world <= 0) return cudaErrorInvalidValue;
  return launch_k(k_argmax_combine, dim3((rows + 127) / 128), dim3(128), 0, s, gathered, ids, rows, world, positions,
                  seq_lens, local_keys);
}

}  // namespace cob
