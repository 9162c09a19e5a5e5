// Single-GPU decode kernels: RMSNorm, add+RMSNorm, embedding, RoPE + paged-KV append, SiLU*mul,
// greedy argmax. Memory-bound elementwise work: 16-byte vector loads, one pass over the data,
// programmatic-dependent-launch wait at the top so a graph of decode kernels overlaps prologues.
#include <float.h>

#include <algorithm>

#include "common.cuh"
#include "ops.h"

namespace cob {
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
  pdl_wait();
  const int row = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)ids[row] * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)row * hidden);
  const int hv = hidden * (int)sizeof(T) / 16;
  for (int v = threadIdx.x; v < hv; v += blockDim.x) dst[v] = ld_nc_v4(src + v);
}

template <typename T>
__global__ void k_rope_append(const T* __restrict__ qkv, const int32_t* __restrict__ positions,
                              const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                              const int32_t* __restrict__ block_tables, int max_blocks, T* __restrict__ q_out,
                              T* __restrict__ k_cache, T* __restrict__ v_cache, int nq, int nkv, int D, int bs) {
  pdl_wait();
  const int b = blockIdx.x;
  const int pos = positions[b];
  const int half = D / 2;
  const T* row = qkv + (size_t)b * (nq + 2 * nkv) * D;
  const float* c = cos_t + (size_t)pos * half;
  const float* s = sin_t + (size_t)pos * half;
  const int blk = block_tables[(size_t)b * max_blocks + pos / bs], off = pos % bs;
  // rotated pairs of q heads then k heads
  for (int t = threadIdx.x; t < (nq + nkv) * half; t += blockDim.x) {
    const int head = t / half, i = t - head * half;
    const T* src = row + (size_t)head * D;
    const float x1 = to_f(src[i]), x2 = to_f(src[i + half]);
    const float o1 = x1 * c[i] - x2 * s[i], o2 = x2 * c[i] + x1 * s[i];
    T* dst;
    if (head < nq) {
      dst = q_out + ((size_t)b * nq + head) * D;
    } else {
      dst = k_cache + (((size_t)blk * nkv + (head - nq)) * bs + off) * D;
    }
    dst[i] = from_f<T>(o1);
    dst[i + half] = from_f<T>(o2);
  }
  // v heads copied as is
  for (int t = threadIdx.x; t < nkv * D; t += blockDim.x) {
    const int h = t / D, d = t - h * D;
    v_cache[(((size_t)blk * nkv + h) * bs + off) * D + d] = row[(size_t)(nq + nkv + h) * D + d];
  }
}

template <typename T>
__global__ void k_silu_mul(const T* __restrict__ gu, T* __restrict__ out, int inter) {
  using V = Vec<T>;
  pdl_wait();
  const int b = blockIdx.y;
  const int iv = inter / V::N;
  const uint4* g = reinterpret_cast<const uint4*>(gu + (size_t)b * 2 * inter);
  const uint4* u = g + iv;
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)b * inter);
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < iv; v += gridDim.x * blockDim.x) {
    float a[V::N], c[V::N], r[V::N];
    V::to_float(g[v], a);
    V::to_float(u[v], c);
#pragma unroll
    for (int i = 0; i < V::N; ++i) r[i] = a[i] / (1.f + __expf(-a[i])) * c[i];
    o[v] = V::from_float(r);
  }
}

// (value, index) pair reduction: larger value wins, ties -> smaller index
__device__ __forceinline__ void amax_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

template <typename T>
__global__ void __launch_bounds__(1024) k_argmax_local(const T* __restrict__ logits, uint32_t* __restrict__ words,
                                                       int vocab, int vocab_offset) {
  pdl_wait();
  const int row = blockIdx.x;
  const T* lr = logits + (size_t)row * vocab;
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) amax_merge(best, bi, to_f(lr[i]), i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    amax_merge(best, bi, v2, i2);
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -FLT_MAX;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      amax_merge(best, bi, v2, i2);
    }
    if (lane == 0) {
      words[row * 2] = __float_as_uint(best);
      words[row * 2 + 1] = (uint32_t)(bi + vocab_offset);
    }
  }
}

__global__ void k_argmax_combine(const uint32_t* __restrict__ words, int32_t* __restrict__ ids, int rows,
                                 int world, int32_t* __restrict__ positions, int32_t* __restrict__ seq_lens) {
  pdl_wait();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  // decode feedback: the token just produced sits at the next position
  if (positions) positions[row] += 1;
  if (seq_lens) seq_lens[row] += 1;
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int r = 0; r < world; ++r) {
    const uint32_t* w = words + ((size_t)r * rows + row) * 2;
    amax_merge(best, bi, __uint_as_float(w[0]), (int)w[1]);
  }
  ids[row] = bi;
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
    k<<<rows, threads_for(hv), 0, s>>>(reinterpret_cast<const T*>(x), nullptr, reinterpret_cast<const T*>(gamma),
                                       reinterpret_cast<T*>(out), hidden, eps);
    return cudaGetLastError();
  });
}

cudaError_t add_rmsnorm(const void* x, void* residual, const void* gamma, void* out, int rows, int hidden,
                        float eps, int dtype, cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    const int hv = hidden / Vec<T>::N;
    if (hidden % Vec<T>::N || hv > 512 * 2 * kVPT || rows <= 0) return cudaErrorInvalidValue;
    auto k = hv > 512 * kVPT ? k_rmsnorm<T, true, 2 * kVPT> : k_rmsnorm<T, true, kVPT>;
    k<<<rows, threads_for(hv), 0, s>>>(
        reinterpret_cast<const T*>(x), reinterpret_cast<T*>(residual), reinterpret_cast<const T*>(gamma),
        reinterpret_cast<T*>(out), hidden, eps);
    return cudaGetLastError();
  });
}

cudaError_t embedding(const int32_t* ids, const void* table, void* out, int rows, int hidden, int dtype,
                      cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if ((hidden * (int)sizeof(T)) % 16 || rows <= 0) return cudaErrorInvalidValue;
    k_embedding<T><<<rows, 256, 0, s>>>(ids, reinterpret_cast<const T*>(table), reinterpret_cast<T*>(out), hidden);
    return cudaGetLastError();
  });
}

cudaError_t rope_append_kv(const void* qkv, const int32_t* positions, const float* cos_t, const float* sin_t,
                           const int32_t* block_tables, int max_blocks_per_seq, void* q_out, void* k_cache,
                           void* v_cache, int batch, int nq, int nkv, int head_dim, int block_size, int dtype,
                           cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (batch <= 0 || head_dim % 2) return cudaErrorInvalidValue;
    k_rope_append<T><<<batch, 256, 0, s>>>(reinterpret_cast<const T*>(qkv), positions, cos_t, sin_t, block_tables,
                                           max_blocks_per_seq, reinterpret_cast<T*>(q_out),
                                           reinterpret_cast<T*>(k_cache), reinterpret_cast<T*>(v_cache), nq, nkv,
                                           head_dim, block_size);
    return cudaGetLastError();
  });
}

cudaError_t silu_mul(const void* gu, void* out, int rows, int inter, int dtype, cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (inter % Vec<T>::N || rows <= 0) return cudaErrorInvalidValue;
    const int iv = inter / Vec<T>::N;
    const int bx = std::min(64, (iv + 255) / 256);
    k_silu_mul<T><<<dim3(bx, rows), 256, 0, s>>>(reinterpret_cast<const T*>(gu), reinterpret_cast<T*>(out), inter);
    return cudaGetLastError();
  });
}

cudaError_t argmax_local(const void* logits, uint32_t* words, int rows, int vocab, int vocab_offset, int dtype,
                         cudaStream_t s) {
  return by_dtype(dtype, [&](auto t) {
    using T = decltype(t);
    if (rows <= 0 || vocab <= 0) return cudaErrorInvalidValue;
    k_argmax_local<T><<<rows, 1024, 0, s>>>(reinterpret_cast<const T*>(logits), words, vocab, vocab_offset);
    return cudaGetLastError();
  });
}

cudaError_t argmax_combine(const uint32_t* words, int32_t* ids, int rows, int world, int32_t* positions,
                           int32_t* seq_lens, cudaStream_t s) {
  if (rows <= 0 || world <= 0) return cudaErrorInvalidValue;
  k_argmax_combine<<<(rows + 127) / 128, 128, 0, s>>>(words, ids, rows, world, positions, seq_lens);
  return cudaGetLastError();
}

}  // namespace cob
