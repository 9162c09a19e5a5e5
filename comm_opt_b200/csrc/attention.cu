// Paged-KV grouped-query decode attention (one new token per sequence).
//
// Grid (splits, kv_heads, batch); a CTA of 4 warps owns one (sequence, kv head) pair and a range of
// 16-token KV pages. All G = nq / nkv query heads of the group are processed together as the
// 16-row A operand of m16n8k16 tensor-core MMAs (rows >= G are zero padding), so each KV byte is
// read once per group: S = Q K^T and O += P V per page, online softmax in the log2 domain.
// Each warp streams its own pages (double-buffered, XOR-swizzled shared memory so ldmatrix is
// conflict-free); warps are merged in shared memory and splits are merged by the last CTA of the
// (sequence, head) pair, found with an atomic counter that the merging CTA resets to zero.
//
// KV layout: [num_blocks, nkv, 16, D] (one 4 KB contiguous page per head at D = 128, bf16).
#include <float.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "ops.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace cob {
namespace {

namespace cg = cooperative_groups;

constexpr int kBS = 16, kWarps = 4, kRows = 16;  // head dims: 64 and 128 (template parameter D)
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(p)));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// element offset of 16-byte chunk `ch` of row `r` in the Q tile ([16][D], chunk ^= row % 8)
template <int D>
__device__ __forceinline__ int swz(int r, int ch) { return r * D + ((ch ^ (r & 7)) << 3); }
// element offset of chunk `ch` (0..D/8-1) of row `r` in a KV page loaded by D/64 TMA boxes of 64 columns
// with the 128-byte swizzle: [D/64 halves][16 rows][64 cols], chunk-within-half ^= row % 8
__device__ __forceinline__ int swzp(int r, int ch) { return ((ch >> 3) << 10) + r * 64 + (((ch & 7) ^ (r & 7)) << 3); }

__device__ __forceinline__ float safe_exp2_diff(float a, float b) { return a == -INFINITY ? 0.f : exp2f(a - b); }

// 16-byte chunk `ch` (8 elements) of head `head` of one token's projection row `src` (+ bias), rotated by
// RoPE with the position's table row `cs` (cos at [0, D/2), sin at [D/2, D), staged in shared memory):
// element i of the first half pairs with i + D / 2. Rounded to T once, as the separate append kernel
// stores it.
template <typename T, int D>
__device__ __forceinline__ uint4 rope_chunk(const AttnParams& p, const T* src, int head, int ch, const float* cs) {
  using V = Vec<T>;
  constexpr int H = D / 2, HC = H / 8;  // half width, chunks per half
  const bool lo = ch < HC;
  const int pc = lo ? ch + HC : ch - HC;  // partner chunk
  const uint4* row = reinterpret_cast<const uint4*>(src + (size_t)head * D);
  float x[8], y[8];
  V::to_float(row[ch], x);
  V::to_float(row[pc], y);
  if (p.qkv_bias != nullptr) {
    const uint4* bias = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.qkv_bias) + (size_t)head * D);
    float bx[8], by[8];
    V::to_float(bias[ch], bx);
    V::to_float(bias[pc], by);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[j] += bx[j];
      y[j] += by[j];
    }
  }
  const int i0 = (lo ? ch : pc) * 8;  // index into the cos / sin row of this position
  float o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float c = cs[i0 + j], sn = cs[H + i0 + j];
    o[j] = lo ? x[j] * c - y[j] * sn : x[j] * c + y[j] * sn;
  }
  return V::from_float(o);
}

// chunk `ch` of head `head` of a projection row (+ bias): the new token's v
template <typename T>
__device__ __forceinline__ uint4 plain_chunk(const AttnParams& p, const T* src, int head, int ch, int D) {
  using V = Vec<T>;
  const uint4 raw = reinterpret_cast<const uint4*>(src + (size_t)head * D)[ch];
  if (p.qkv_bias == nullptr) return raw;
  float x[8], bx[8];
  V::to_float(raw, x);
  V::to_float(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.qkv_bias) + (size_t)head * D)[ch], bx);
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] += bx[j];
  return V::from_float(x);
}

constexpr int kStages = 3;                    // KV pages in flight per warp (two CTAs per SM)
constexpr int kStagesDeep = 6;                // the deep ring: one CTA per SM
template <int D>
constexpr int kPageElems = kBS * D;           // one K (or V) page: 16 x D
constexpr int kMaxPagesPerSplit = 512;
constexpr int kMaxClusterSplits = 16;         // splits merged inside one (non-portable) cluster

struct alignas(64) AttnArgs {
  CUtensorMap tk, tv;  // K / V caches as 2-D [num_blocks * nkv * 16, 128], box 64 x 16, 128-byte swizzle
  AttnParams p;
  int push;  // cluster merge by pushes into the owners' shared memory (2..8 splits)
};

// Shared memory of the push merge: [splits][per] partial outputs, then [splits][G][2] (max, sum), where
// per = ceil(G * D / splits) output elements belong to each CTA of the cluster.
__host__ __device__ constexpr size_t attn_push_bytes(int splits, int G, int D) {
  return ((size_t)splits * ((G * D + splits - 1) / splits) + (size_t)splits * G * 2) * sizeof(float);
}

template <int D, int S>
__host__ __device__ constexpr size_t attn_smem_bytes() {
  return 1024 /*align*/ + (size_t)kWarps * S * 2 * kPageElems<D> * 2 + (size_t)kRows * D * 2 +
         (size_t)kWarps * S * 8 + kMaxPagesPerSplit * 4 + (size_t)D * 4 /*cos / sin row*/ + 64;
}

// CLUSTER: the splits of one (sequence, kv head) pair form a thread-block cluster (splits <= 16) and
// are merged through distributed shared memory; otherwise they are merged through the global
// scratch by the last split to finish.
// S: KV pages in flight per warp (kStages, or kStagesDeep when the grid fits one CTA per SM).
template <typename T, bool CLUSTER, int D, int S>
__global__ void __launch_bounds__(kWarps * 32) k_decode_attn(const __grid_constant__ AttnArgs args) {
  constexpr int kD = D, PE = kPageElems<D>, kStages = S;
  using namespace sm100;
  const AttnParams& p = args.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  T* sKV = reinterpret_cast<T*>(base);  // [kWarps][kStages][K,V][2 halves][16][64]
  T* sQ = sKV + (size_t)kWarps * kStages * 2 * PE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sQ + kRows * kD);  // [kWarps][kStages]
  int* s_pages = reinterpret_cast<int*>(bars + kWarps * kStages);
  float* s_cs = reinterpret_cast<float*>(s_pages + kMaxPagesPerSplit);  // [D]: cos, sin of the new position
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.nq / p.nkv;
  float* s_red = s_cs + kD;  // push merge: what the cluster's CTAs push to this one (attn_push_bytes)
  // push merge: first half of a cluster barrier that every CTA passes before its first remote store,
  // so each CTA of the cluster has started before its shared memory is written
  if (CLUSTER && args.push) asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
  constexpr int CH = kD / 8;  // 16-byte chunks per row

  if (threadIdx.x == 0) {
    prefetch_tmap(&args.tk);
    prefetch_tmap(&args.tv);
    for (int i = 0; i < kWarps * kStages; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  // The block table and the sequence lengths were written before the previous kernel of the stream
  // started (the step's last kernel, or the host), and every KV page except the one holding the new
  // token is unchanged by the previous kernel (RoPE + KV append, or the QKV GEMM with that epilogue):
  // they are read, and those pages requested, before the dependency wait, so the KV stream overlaps the
  // previous kernel. The page of the new token and the query wait for it.
  // The sequence's pages are cut into `splits` equal parts by its actual length (at most
  // pages_per_split each, the plan's bound for the block table's capacity), so a cache sized for long
  // sequences still keeps every split of a shorter one busy.
  // When the block table's row fits the page list, the whole row is requested together with the
  // sequence length (no dependent load between them); longer rows read the split's range afterwards.
  const int* bt_row = p.block_tables + (size_t)b * p.max_blocks_per_seq;
  const bool whole_row = p.max_blocks_per_seq <= kMaxPagesPerSplit;
  const bool rope = p.qkv != nullptr;
  // positions, like the lengths, are written before the step starts; the RoPE tables are constant
  const int pos = rope ? p.positions[b] : 0;
  const int seq = p.seq_lens[b];
  if (whole_row)
    for (int i = threadIdx.x; i < p.max_blocks_per_seq; i += blockDim.x) s_pages[i] = bt_row[i];
  const int npages = min((seq + kBS - 1) / kBS, p.max_blocks_per_seq);  // a length past the table is clamped
  const int pps = min(p.pages_per_split, max(1, (npages + p.splits - 1) / p.splits));
  const int pg0 = split * pps;
  const int pg1 = min(npages, pg0 + pps);
  if (!whole_row)
    for (int i = threadIdx.x; i < pg1 - pg0; i += blockDim.x) s_pages[i] = bt_row[pg0 + i];
  __syncthreads();  // page list (and the barrier initialisation) visible to every warp
  const int* my_list = s_pages + (whole_row ? pg0 : 0);  // entry i: page pg0 + i of the sequence

  T* myKV = sKV + (size_t)warp * kStages * 2 * PE;
  uint64_t* mybar = bars + warp * kStages;
  // page i of this warp is pg0 + warp + i * kWarps
  const int my_pages = pg1 - pg0 > warp ? (pg1 - pg0 - warp + kWarps - 1) / kWarps : 0;
  auto issue = [&](int i) {
    if (i >= my_pages || lane != 0) return;
    const int st = i % kStages;
    const int blk = my_list[warp + i * kWarps];
    const int row = (blk * p.nkv + kvh) * kBS;
    T* dk = myKV + (size_t)st * 2 * PE;
    T* dv = dk + PE;
    mbar_arrive_expect_tx(&mybar[st], 2 * PE * sizeof(T));
#pragma unroll
    for (int h = 0; h < D / 64; ++h) {  // boxes of 64 columns (128 bytes, the swizzle span)
      tma_load_2d(dk + h * kBS * 64, &args.tk, &mybar[st], 64 * h, row);
      tma_load_2d(dv + h * kBS * 64, &args.tv, &mybar[st], 64 * h, row);
    }
  };
  // Without the fused append, the page holding the new token is written by the previous kernel and is
  // requested after the dependency wait; with it, its cache row is stale until this kernel writes it,
  // and the warp that owns the page patches the row in shared memory once the page has landed.
  const int last_pg = npages - 1;
#pragma unroll
  for (int i = 0; i < kStages; ++i)
    if (rope || pg0 + warp + i * kWarps != last_pg) issue(i);
  if (rope) {  // the position's RoPE row, staged before the wait: after it only the projection is loaded
    for (int i = threadIdx.x; i < kD / 2; i += blockDim.x) {
      s_cs[i] = p.cos_t[(size_t)pos * (kD / 2) + i];
      s_cs[kD / 2 + i] = p.sin_t[(size_t)pos * (kD / 2) + i];
    }
    __syncthreads();
  }
  pdl_wait_then_trigger();  // the next kernel (the o_proj GEMM) may start streaming its weights
  if (!rope) {
#pragma unroll
    for (int i = 0; i < kStages; ++i)
      if (pg0 + warp + i * kWarps == last_pg) issue(i);
  }
  // the query tile is staged while the first pages are in flight (rotated here in the fused form)
  const int qkv_stride = (p.nq + 2 * p.nkv) * kD;
  for (int c = threadIdx.x; c < kRows * CH; c += blockDim.x) {
    const int r = c / CH, ch = c % CH;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G) {
      if (rope)
        v = rope_chunk<T, D>(p, reinterpret_cast<const T*>(p.qkv) + (size_t)b * qkv_stride, kvh * G + r, ch, s_cs);
      else
        v = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) + ((size_t)b * p.nq + (size_t)kvh * G + r) *
                                           kD)[ch];
    }
    *reinterpret_cast<uint4*>(sQ + swz<D>(r, ch)) = v;
  }
  __syncthreads();
  uint32_t qa[kD / 16][4];
#pragma unroll
  for (int ks = 0; ks < kD / 16; ++ks) {
    const int r = lane & 15, ch = ks * 2 + (lane >> 4);
    ldsm_x4(qa[ks], sQ + swz<D>(r, ch));
  }

  const float sl2 = p.scale * kLog2e;
  float o[kD / 8][4];
#pragma unroll
  for (int n = 0; n < kD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  bool ok = true;

  for (int i = 0; i < my_pages && ok; ++i) {
    const int st = i % kStages;
    const int pg = pg0 + warp + i * kWarps;
    if (!mbar_wait(&mybar[st], (i / kStages) & 1, 1000000000ull)) {
      ok = false;
      if (p.err) atomicOr(p.err, 1);
      break;
    }
    const T* sK = myKV + (size_t)st * 2 * PE;
    const T* sV = sK + PE;
    if (rope && pg == pos / kBS) {
      // the new token's row: k rotated, v (+ bias) from the projection, into the landed page and the cache
      const T* src = reinterpret_cast<const T*>(p.qkv) + (size_t)b * qkv_stride;
      const int r = pos % kBS, blk = my_list[pg - pg0];
      for (int c = lane; c < 2 * CH; c += 32) {
        const bool is_k = c < CH;
        const int ch = is_k ? c : c - CH;
        const uint4 v = is_k ? rope_chunk<T, D>(p, src, p.nq + kvh, ch, s_cs)
                             : plain_chunk<T>(p, src, p.nq + p.nkv + kvh, ch, kD);
        *reinterpret_cast<uint4*>(const_cast<T*>(is_k ? sK : sV) + swzp(r, ch)) = v;
        T* cache = reinterpret_cast<T*>(const_cast<void*>(is_k ? p.k_cache : p.v_cache));  // the append writes the caches
        reinterpret_cast<uint4*>(cache + (((size_t)blk * p.nkv + kvh) * kBS + r) * kD)[ch] = v;
      }
      __syncwarp();
    }
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks) {
        const int tok = nt * 8 + (lane & 7), ch = ks * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1;
        ldsm_x2(b0, b1, sK + swzp(tok, ch));
        mma16816<T>(s[nt], qa[ks], b0, b1);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tok = pg * kBS + nt * 8 + 2 * (lane & 3) + (j & 1);
        s[nt][j] = tok < seq ? s[nt][j] * sl2 : -INFINITY;
      }
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float a0 = safe_exp2_diff(m0, mn0), a1 = safe_exp2_diff(m1, mn1);
    m0 = mn0;
    m1 = mn1;
    float pr[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      pr[nt][0] = exp2f(s[nt][0] - mn0);
      pr[nt][1] = exp2f(s[nt][1] - mn0);
      pr[nt][2] = exp2f(s[nt][2] - mn1);
      pr[nt][3] = exp2f(s[nt][3] - mn1);
    }
    l0 = l0 * a0 + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    l1 = l1 * a1 + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
    uint32_t pa[4];
    pa[0] = pack2<T>(pr[0][0], pr[0][1]);
    pa[1] = pack2<T>(pr[0][2], pr[0][3]);
    pa[2] = pack2<T>(pr[1][0], pr[1][1]);
    pa[3] = pack2<T>(pr[1][2], pr[1][3]);
#pragma unroll
    for (int n = 0; n < kD / 8; ++n) {
      o[n][0] *= a0;
      o[n][1] *= a0;
      o[n][2] *= a1;
      o[n][3] *= a1;
      const int tok = lane & 15;
      uint32_t b0, b1;
      ldsm_x2_t(b0, b1, sV + swzp(tok, n));
      mma16816<T>(o[n], pa, b0, b1);
    }
    __syncwarp();   // every lane is done with this stage before it is refilled
    issue(i + kStages);
  }
  // a warp that gave up still has copies in flight: wait for them (bounded) before smem is reused
  if (!ok && lane == 0) {
    for (int i = 0; i < my_pages && i < kStages; ++i) mbar_wait(&mybar[i % kStages], 0, 1000000000ull);
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // ---- merge the warps (shared memory reused)
  __syncthreads();
  float* sO = reinterpret_cast<float*>(sKV);    // [kWarps][16][kD]
  float* sML = sO + kWarps * kRows * kD;        // [kWarps][16][2]
  {
    const int r = lane >> 2, c = 2 * (lane & 3);
#pragma unroll
    for (int n = 0; n < kD / 8; ++n) {
      float* bp = sO + ((size_t)warp * kRows) * kD + n * 8 + c;
      bp[(size_t)r * kD] = o[n][0];
      bp[(size_t)r * kD + 1] = o[n][1];
      bp[(size_t)(r + 8) * kD] = o[n][2];
      bp[(size_t)(r + 8) * kD + 1] = o[n][3];
    }
    if ((lane & 3) == 0) {
      sML[(warp * kRows + r) * 2] = m0;
      sML[(warp * kRows + r) * 2 + 1] = l0;
      sML[(warp * kRows + r + 8) * 2] = m1;
      sML[(warp * kRows + r + 8) * 2 + 1] = l1;
    }
  }
  __syncthreads();
  T* out = reinterpret_cast<T*>(p.out) + ((size_t)b * p.nq + (size_t)kvh * G) * kD;
  const size_t pair = (size_t)b * p.nkv + kvh;
  // cluster mode: this CTA's merged partial stays in shared memory for its cluster peers
  float* cO = sML + kWarps * kRows * 2;  // [G][kD]
  float* cML = cO + kRows * kD;          // [G][2]
  float* po = CLUSTER ? cO : p.part_o + (pair * p.splits + split) * (size_t)G * kD;
  float* pml = CLUSTER ? cML : p.part_ml + (pair * p.splits + split) * (size_t)G * 2;
  for (int idx = threadIdx.x; idx < G * kD; idx += blockDim.x) {
    const int g = idx / kD, d = idx - g * kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sML[(w * kRows + g) * 2]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = safe_exp2_diff(sML[(w * kRows + g) * 2], M);
      L += f * sML[(w * kRows + g) * 2 + 1];
      O += f * sO[((size_t)w * kRows + g) * kD + d];
    }
    if (p.splits == 1) {
      out[(size_t)g * kD + d] = from_f<T>(O / L);
    } else {
      po[idx] = O;
      if (d == 0) {
        pml[g * 2] = M;
        pml[g * 2 + 1] = L;
      }
    }
  }
  if (p.splits == 1) return;
  if (CLUSTER && args.push) {
    // Push merge: every CTA stores its partial of output element idx into the shared memory of the CTA
    // that owns idx (and its (max, sum) rows into every CTA), one cluster barrier, then each owner folds
    // the splits from local memory in split order - the arithmetic of the pull merge below, without its
    // remote-load round trips and its second barrier.
    cg::cluster_group cluster = cg::this_cluster();
    const int cs = p.splits, r = split, per = (G * kD + cs - 1) / cs;
    float* redML = s_red + (size_t)cs * per;  // [cs][G][2]
    __syncthreads();  // this CTA's partial (cO, cML) complete
    asm volatile("barrier.cluster.wait;" ::: "memory");  // second half of the start-up barrier
    for (int idx = threadIdx.x; idx < G * kD; idx += blockDim.x) {
      const int o = idx / per;
      cluster.map_shared_rank(s_red, o)[(size_t)split * per + (idx - o * per)] = cO[idx];
    }
    for (int i = threadIdx.x; i < cs * G; i += blockDim.x) {  // (destination CTA, row)
      const int c = i / G, g = i - c * G;
      float* ml = cluster.map_shared_rank(redML, c) + ((size_t)split * G + g) * 2;
      ml[0] = cML[g * 2];
      ml[1] = cML[g * 2 + 1];
    }
    cluster.sync();  // release / acquire: every push has landed in its owner
    for (int idx = r * per + threadIdx.x; idx < min(G * kD, (r + 1) * per); idx += blockDim.x) {
      const int g = idx / kD, li = idx - r * per;
      float M = -INFINITY;
      for (int c = 0; c < cs; ++c) M = fmaxf(M, redML[(c * G + g) * 2]);
      float L = 0.f, O = 0.f;
      for (int c = 0; c < cs; ++c) {
        const float f = safe_exp2_diff(redML[(c * G + g) * 2], M);
        L += f * redML[(c * G + g) * 2 + 1];
        O += f * s_red[(size_t)c * per + li];
      }
      out[idx] = from_f<T>(O / L);
    }
    return;  // no peer reads this CTA's shared memory after the barrier
  }
  if (CLUSTER) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int cs = p.splits, r = split;  // cluster spans the splits of this pair (<= kMaxClusterSplits)
    // every split's (max, sum) per query row, copied once into this CTA's shared memory (one DSMEM
    // load per thread, all in flight together), then each output element's partials of all splits
    // requested together; sums in split order, as one pass over the splits would give
    float* sMLall = cML + kRows * 2;  // [cs][G][2], past the buffers the peers read
    for (int i = threadIdx.x; i < cs * G * 2; i += blockDim.x) {
      const int c = i / (G * 2);
      sMLall[i] = cluster.map_shared_rank(cML, c)[i - c * G * 2];
    }
    __syncthreads();
    const int per = (G * kD + cs - 1) / cs;
    for (int idx = r * per + threadIdx.x; idx < min(G * kD, (r + 1) * per); idx += blockDim.x) {
      const int g = idx / kD;
      float ov[kMaxClusterSplits];
#pragma unroll
      for (int c = 0; c < kMaxClusterSplits; ++c)
        if (c < cs) ov[c] = cluster.map_shared_rank(cO, c)[idx];
      float M = -INFINITY;
      for (int c = 0; c < cs; ++c) M = fmaxf(M, sMLall[(c * G + g) * 2]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int c = 0; c < kMaxClusterSplits; ++c) {
        if (c < cs) {
          const float f = safe_exp2_diff(sMLall[(c * G + g) * 2], M);
          L += f * sMLall[(c * G + g) * 2 + 1];
          O += f * ov[c];
        }
      }
      out[idx] = from_f<T>(O / L);
    }
    // keeps this CTA's partial alive until every peer has read it; nothing is published after the
    // barrier above, so the arrive needs no release ordering
    asm volatile("barrier.cluster.arrive.relaxed;\n\tbarrier.cluster.wait;" ::: "memory");
    return;
  }
  // ---- the last split of this (sequence, head) pair merges all splits
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&p.counters[pair], 1);
    s_last = prev == p.splits - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* po0 = p.part_o + pair * p.splits * (size_t)G * kD;
  const float* pml0 = p.part_ml + pair * p.splits * (size_t)G * 2;
  // split weights computed once: w[sp][g] = 2^(m_sp,g - M_g), inv_l[g] = 1 / sum_sp w * l
  float* s_w = reinterpret_cast<float*>(sKV);      // [splits][G] (KV stages are free now)
  float* s_l = s_w + (size_t)p.splits * G;         // [splits][G]
  float* s_inv = s_l + (size_t)p.splits * G;       // [G]
  for (int i = threadIdx.x; i < p.splits * G; i += blockDim.x) {
    s_w[i] = __ldcg(pml0 + (size_t)i * 2);
    s_l[i] = __ldcg(pml0 + (size_t)i * 2 + 1);
  }
  __syncthreads();
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    float M = -INFINITY;
    for (int sp = 0; sp < p.splits; ++sp) M = fmaxf(M, s_w[sp * G + g]);
    float L = 0.f;
    for (int sp = 0; sp < p.splits; ++sp) {
      const float f = safe_exp2_diff(s_w[sp * G + g], M);
      s_w[sp * G + g] = f;
      L += f * s_l[sp * G + g];
    }
    s_inv[g] = 1.f / L;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * kD; idx += blockDim.x) {
    const int g = idx / kD;
    float O = 0.f;
    int sp = 0;
    for (; sp + 8 <= p.splits; sp += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcg(po0 + (size_t)(sp + u) * G * kD + idx);
#pragma unroll
      for (int u = 0; u < 8; ++u) O += s_w[(sp + u) * G + g] * v[u];
    }
    for (; sp < p.splits; ++sp) O += s_w[sp * G + g] * __ldcg(po0 + (size_t)sp * G * kD + idx);
    out[idx] = from_f<T>(O * s_inv[g]);
  }
  if (threadIdx.x == 0) p.counters[pair] = 0;
}

}  // namespace

size_t attn_scratch_bytes(int batch, int nkv, int splits, int group, int head_dim) {
  const size_t pairs = (size_t)batch * nkv;
  return pairs * splits * group * head_dim * sizeof(float) + pairs * splits * group * 2 * sizeof(float) +
         pairs * sizeof(int32_t);
}

int& attn_stage_mode() {
  static int mode = 0;
  return mode;
}

size_t attn_launch_smem_bytes(int splits, int group, int head_dim, bool cluster, int stages) {
  const bool deep = stages == kStagesDeep;
  const size_t base = head_dim == 128 ? (deep ? attn_smem_bytes<128, kStagesDeep>() : attn_smem_bytes<128, kStages>())
                                      : (deep ? attn_smem_bytes<64, kStagesDeep>() : attn_smem_bytes<64, kStages>());
  const bool cl = cluster && splits > 1 && splits <= kMaxClusterSplits;
  return base + (cl && splits <= 8 ? attn_push_bytes(splits, group, head_dim) : 0);
}

namespace {

// KV ring depth of one launch. The deep ring (all four pages of every warp of a 2048-token, 8-way split
// in flight) needs one CTA per SM at head_dim 128, so it is used only for grids that fit in one wave at
// one CTA per SM and clusters of at most 8 (portable sizes); mode kStagesDeep asks for it, any other
// mode keeps the shallow ring (two CTAs per SM).
int attn_stages_for(int ctas, int cluster_size) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return attn_stage_mode() == kStagesDeep && ctas <= sms && cluster_size <= 8 ? kStagesDeep : kStages;
}

template <int D, int S>
cudaError_t launch_attention_s(const AttnParams& p, cudaStream_t s);

template <int D>
cudaError_t launch_attention(const AttnParams& p, cudaStream_t s) {
  const int ctas = p.splits * p.nkv * p.batch;
  return attn_stages_for(ctas, p.cluster ? p.splits : 1) == kStagesDeep ? launch_attention_s<D, kStagesDeep>(p, s)
                                                                        : launch_attention_s<D, kStages>(p, s);
}

template <int D, int S>
cudaError_t launch_attention_s(const AttnParams& p, cudaStream_t s) {
  constexpr int PE = kPageElems<D>;
  if ((size_t)p.splits * (p.nq / p.nkv) * 2 + kRows > (size_t)kWarps * kStages * 2 * PE / 2)
    return cudaErrorInvalidValue;  // the global merge's split weights must fit in the KV stages
  static_assert(kWarps * kRows * D * 4 + kWarps * kRows * 2 * 4 + kRows * D * 4 + kRows * 2 * 4 +
                        kMaxClusterSplits * kRows * 2 * 4 <=
                    kWarps * kStages * 2 * PE * 2,
                "merge buffers must fit in the KV stages");
  AttnArgs a;
  a.p = p;
  a.push = 0;
  // rows of the 2-D cache view; when the caller does not know the block count a large bound is used
  // (only rows named by the block tables are ever read)
  const uint64_t rows = (uint64_t)(p.num_blocks > 0 ? p.num_blocks : (1 << 22)) * p.nkv * kBS;
  const bool bf16 = p.dtype == kBF16;
  cudaError_t e = tensor_map_2d(p.k_cache, rows, D, D * 2, kBS, 64, bf16, &a.tk);
  if (e != cudaSuccess) return e;
  e = tensor_map_2d(p.v_cache, rows, D, D * 2, kBS, 64, bf16, &a.tv);
  if (e != cudaSuccess) return e;
  const dim3 grid(p.splits, p.nkv, p.batch);
  const bool cluster = p.cluster && p.splits > 1 && p.splits <= kMaxClusterSplits;
  // the push merge for portable clusters (its buffer keeps two CTAs per SM with the shallow ring)
  a.push = cluster && p.splits <= 8;
  const size_t smem = attn_launch_smem_bytes(p.splits, p.nq / p.nkv, D, cluster, S);
  auto fn = bf16 ? (cluster ? k_decode_attn<__nv_bfloat16, true, D, S> : k_decode_attn<__nv_bfloat16, false, D, S>)
                 : (cluster ? k_decode_attn<__half, true, D, S> : k_decode_attn<__half, false, D, S>);
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (cluster && p.splits > 8) {  // clusters of 9..16 CTAs are non-portable (two CTAs per SM here)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  if (!cluster) return launch_k(fn, grid, dim3(kWarps * 32), smem, s, a);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  int na = 1;
  if (pdl_flag()) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

}  // namespace

cudaError_t paged_decode_attention(const AttnParams& p, cudaStream_t s) {
  if ((p.head_dim != 64 && p.head_dim != 128) || p.block_size != kBS || p.nkv <= 0 || p.nq % p.nkv != 0 ||
      p.nq / p.nkv > kRows || p.splits <= 0 || p.pages_per_split <= 0 || p.pages_per_split > kMaxPagesPerSplit ||
      p.batch <= 0 || (p.dtype != kBF16 && p.dtype != kF16))
    return cudaErrorInvalidValue;
  if (p.qkv != nullptr && (p.positions == nullptr || p.cos_t == nullptr || p.sin_t == nullptr)) return cudaErrorInvalidValue;
  return p.head_dim == 128 ? launch_attention<128>(p, s) : launch_attention<64>(p, s);
}

}  // namespace cob

// ------------------------------------------------------------------------------------------------
// Allocation-free entry point (see attention_noalloc.h for who calls it and its limits).
// ------------------------------------------------------------------------------------------------
#include <mutex>
#include <string>

#include "attention_noalloc.h"

// One fixed scratch area per GPU, part of the library image: split-KV partial outputs, their
// (max, sum) pairs and the per-(sequence, head) arrival counters of the kernel above.
static __device__ __align__(256) unsigned char g_noalloc_scratch[COB_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoAllocMaxDevices = 64;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;
thread_local std::string g_noalloc_err;

int noalloc_fail(int code, const std::string& msg) {
  g_noalloc_err = msg;
  return code;
}
}  // namespace

extern "C" __attribute__((visibility("default"))) size_t cob_noalloc_scratch_capacity(void) {
  return COB_NOALLOC_SCRATCH_BYTES;
}

extern "C" __attribute__((visibility("default"))) const char* cob_noalloc_last_error(void) {
  return g_noalloc_err.c_str();
}

extern "C" __attribute__((visibility("default"))) int cob_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int32_t* block_tables, const int32_t* seq_lens,
    void* out, int batch, int nq, int nkv, int head_dim, int block_size, int max_blocks_per_seq, int num_blocks,
    int splits, int pages_per_split, float scale, int dtype, void* stream) {
  g_noalloc_err.clear();
  if (batch <= 0 || nkv <= 0 || nq <= 0 || nq % nkv != 0)
    return noalloc_fail(cudaErrorInvalidValue, "invalid head geometry: need batch > 0, nkv > 0 and nq a multiple of nkv");
  if (head_dim != 64 && head_dim != 128)
    return noalloc_fail(cudaErrorInvalidValue, "head_dim must be 64 or 128, got " + std::to_string(head_dim));
  if (block_size != 16)
    return noalloc_fail(cudaErrorInvalidValue, "block_size must be 16 (tokens per KV page), got " +
                                                   std::to_string(block_size));
  if (dtype != cob::kBF16 && dtype != cob::kF16)
    return noalloc_fail(cudaErrorInvalidValue, "dtype must be 1 (fp16) or 2 (bf16)");
  if (max_blocks_per_seq <= 0)
    return noalloc_fail(cudaErrorInvalidValue, "max_blocks_per_seq must be positive");
  if (num_blocks <= 0)
    return noalloc_fail(cudaErrorInvalidValue, "num_blocks (pages in each cache) must be positive");
  if ((unsigned long long)num_blocks * (unsigned long long)nkv * 16ull >= (1ull << 32))
    return noalloc_fail(cudaErrorInvalidValue, "cache too large: num_blocks * nkv * 16 rows must stay below 2^32");
  if (splits <= 0 || pages_per_split <= 0 || pages_per_split > 512)
    return noalloc_fail(cudaErrorInvalidValue, "need splits > 0 and 0 < pages_per_split <= 512");
  if ((long long)splits * pages_per_split < max_blocks_per_seq)
    return noalloc_fail(cudaErrorInvalidValue,
                        "splits * pages_per_split (" + std::to_string((long long)splits * pages_per_split) +
                            ") does not cover max_blocks_per_seq (" + std::to_string(max_blocks_per_seq) +
                            "): the tokens beyond it would be dropped");
  const size_t need = cob::attn_scratch_bytes(batch, nkv, splits, nq / nkv, head_dim);
  if (need > COB_NOALLOC_SCRATCH_BYTES)
    return noalloc_fail(cudaErrorInvalidValue, "split-KV scratch of " + std::to_string(need) +
                                                   " bytes exceeds the built-in limit of " +
                                                   std::to_string((size_t)COB_NOALLOC_SCRATCH_BYTES) +
                                                   " bytes; use fewer splits or a smaller batch");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(e, "cudaGetDevice failed");
  if (dev < 0 || dev >= kNoAllocMaxDevices) return noalloc_fail(cudaErrorInvalidDevice, "device index too large");
  void* base = nullptr;
  {
    // set-up, once per device, with that device current: host code needs the array's device address
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      e = cudaGetSymbolAddress(&g_noalloc_addr[dev], g_noalloc_scratch);
      if (e != cudaSuccess) {
        g_noalloc_addr[dev] = nullptr;
        return noalloc_fail(e, std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
      }
    }
    base = g_noalloc_addr[dev];
  }
  const size_t pairs = (size_t)batch * nkv, group = (size_t)(nq / nkv);
  char* b = static_cast<char*>(base);
  cob::AttnParams p = {};
  p.q = q;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.block_tables = block_tables;
  p.seq_lens = seq_lens;
  p.out = out;
  p.part_o = reinterpret_cast<float*>(b);
  p.part_ml = reinterpret_cast<float*>(b + pairs * splits * group * head_dim * sizeof(float));
  p.counters = reinterpret_cast<int32_t*>(b + pairs * splits * group * head_dim * sizeof(float) +
                                          pairs * splits * group * 2 * sizeof(float));
  p.batch = batch;
  p.nq = nq;
  p.nkv = nkv;
  p.head_dim = head_dim;
  p.block_size = block_size;
  p.max_blocks_per_seq = max_blocks_per_seq;
  p.num_blocks = num_blocks;  // the K/V tensor maps end at the caller's cache: stray pages read zeros
  p.splits = splits;
  p.pages_per_split = pages_per_split;
  p.scale = scale;
  p.dtype = dtype;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the counters must start at zero (the array keeps whatever the previous call left)
  e = cudaMemsetAsync(p.counters, 0, pairs * sizeof(int32_t), s);
  if (e != cudaSuccess) return noalloc_fail(e, std::string("clearing counters failed: ") + cudaGetErrorString(e));
  e = cob::paged_decode_attention(p, s);
  if (e != cudaSuccess) return noalloc_fail(e, std::string("launch failed: ") + cudaGetErrorString(e));
  return 0;
}
