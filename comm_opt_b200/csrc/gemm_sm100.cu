// Decode-shaped GEMM on the 5th-generation tensor cores: Y[M, N] = X[M, K] * W[N, K]^T, M small.
//
// Swap-AB: a CTA owns 128 output features (the tcgen05 M dimension) and all M <= 256 batch rows
// (the tcgen05 N dimension, padded to 16..256), so the weight matrix - the bytes that bound decode -
// streams through shared memory exactly once:
//   warp 0 / one thread : TMA producer. Weight tiles (128 x 64, 128-byte swizzle) for the first ring
//                         slots are issued BEFORE the programmatic-dependent-launch wait (weights do
//                         not depend on the previous kernel); activation tiles after it.
//   warp 1 / one thread : tcgen05.mma issuer, fp32 accumulator in TMEM (BN columns), releases ring
//                         slots with tcgen05.commit -> mbarrier.
//   warps 2-5           : epilogue, tcgen05.ld of their 32 TMEM lanes, bf16 stores / partials.
// Persistent stream-K: one CTA per SM; CTA c owns an equal, contiguous share of the flattened
// (output tile, 64-wide k-step) space, so every SM streams the same number of weight bytes whatever
// the tile count (no wave quantisation). Accumulators are double-buffered in TMEM so the epilogue of
// one tile overlaps the MMAs of the next. A tile split between CTAs is finished by its last
// contributor, which sums every contributor's fp32 partial (workspace) in CTA order: deterministic.
// Every mbarrier wait is bounded by %globaltimer; a timeout sets *err and the CTA drains and exits.
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "gemm.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace cob {
namespace {

namespace cg = cooperative_groups;
using namespace sm100;

constexpr int BM = 128, BK = 64;
constexpr int kThreads = 192;  // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kSmemBudget = 220 * 1024;
constexpr int kMaxContrib = 48;  // CTAs sharing one tile (the planner keeps it below this)
// phase stamp slots per CTA (profiling only; gemm_stamps() == nullptr switches them off)
enum : int {
  kStEntry = 0,         // kernel entry
  kStSetup = 1,         // barriers initialised, TMEM allocated
  kStWeightsIssued = 2, // producer: first ring of weight tiles issued (before the dependency wait)
  kStPdlWait = 3,       // producer: previous kernel's data visible
  kStLastLoad = 4,      // producer: every load issued
  kStFirstFull = 5,     // MMA issuer: first stage landed
  kStLastMma = 6,       // MMA issuer: last MMA issued
  kStAccReady = 7,      // epilogue: last accumulator complete
  kStEpiDone = 8,       // epilogue: last tile stored (or its partial written)
  kStEnd = 9,           // all threads done (cluster reduction included), before teardown
};

// SMALL: half the shared-memory ring, so two CTAs (this kernel and the next one in the stream under
// programmatic dependent launch) fit on one SM.
// CL: cluster split-K, which adds a reduction area for the partial tiles that the cluster's CTAs push
// to each other (outside the ring, so a peer can write it while this CTA's MMAs still read the ring).
template <int BN, bool SMALL = false, bool CL = false>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;  // 16 KB weight tile
  static constexpr int B_BYTES = BN * BK * 2;  // activation tile
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int RED = CL ? ((BM + 8) * (BN + 4) * 4 + 127) / 128 * 128 : 0;
  static constexpr int STAGES_RAW = ((SMALL ? kSmemBudget / 2 : kSmemBudget) - 2048 - RED) / STAGE;
  static constexpr int STAGES = STAGES_RAW > 12 ? 12 : STAGES_RAW;
  static constexpr int PIPE = STAGES * STAGE;
  static constexpr int SMEM = PIPE + RED + 1024 + 512;  // alignment slack + barriers + contributor table
  static constexpr int TC = BN < 32 ? 32 : BN;          // TMEM columns per accumulator buffer
  static constexpr int TMEM_COLS = 2 * TC;              // double-buffered accumulator
};

// Cluster barrier halves (non-aligned forms: lanes of a warp may reach them at different points).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }

// v as the output type would hold it (the value a plain GEMM stores)
template <bool BF16>
__device__ __forceinline__ float round_out(float v) {
  return BF16 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}

template <bool BF16>
__device__ __forceinline__ void store_out(void* Y, size_t idx, float v) {
  if (BF16)
    reinterpret_cast<__nv_bfloat16*>(Y)[idx] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(Y)[idx] = __float2half_rn(v);
}

// Stream-K partition: CTA c owns flattened k-steps [beg(c), beg(c+1)) of tiles x KT.
__device__ __forceinline__ long long sk_beg(int c, long long total, int P) { return (long long)c * total / P; }
__device__ __forceinline__ int sk_owner(long long g, long long total, int P) {
  int c = (int)((g * P) / total);
  while (c + 1 < P && sk_beg(c + 1, total, P) <= g) ++c;
  while (c > 0 && sk_beg(c, total, P) > g) --c;
  return c;
}

// Named barrier among the 4 epilogue warps (ids 1.., count 128)
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// CLUSTER: instead of the stream-K partition, CTA (t, r) of grid (tiles, s) owns k-range r of tile t and
// the s CTAs of a tile form a thread-block cluster that sums its partial tiles through distributed
// shared memory (no global workspace, no L2 round trips on the tail). `kps` = k-steps per split.
// swiglu: W holds gate and up rows interleaved by 64 (tile t = gate features 64t..64t+63, then the
// matching up features), Y is [M, N / 2] = silu(gate) * up. CLUSTER (s in {2, 4, 8, 16}): CTA r of the
// cluster receives gate rows [r * 64 / s, (r + 1) * 64 / s) of the tile together with their up rows, so
// the product is formed where the sums are. Stream-K (BN = 16): the epilogue warps holding the up rows
// (TMEM lanes 64..127) hand them to the warps holding the gate rows through a per-CTA area of the
// workspace (written, epilogue barrier, read) - for whole tiles and in the finisher of split tiles.
// Either way the SiLU * up kernel and the [M, N] round trip disappear.
// SW: the stream-K SwiGLU epilogue compiled in (BN = 16, stream-K only): a separate instance, so the
// plain kernels keep their register budget (two CTAs per SM with the half ring).
template <int BN, bool BF16, bool SMALL, bool CLUSTER, bool SW = false>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_streamk(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, void* Y, int M,
                   int N, int K, int ldy, float* ws, int* tile_ctr, int* err, unsigned long long timeout_ns,
                   int kps, int l2pf, long long* stamps, const uint8_t* __restrict__ Wp, int swiglu) {
  using C = Cfg<BN, SMALL, CLUSTER>;
  static_assert(!SW || (BN == 16 && !CLUSTER), "the stream-K SwiGLU epilogue is for 16-column batch tiles");
  // optional phase stamps (%globaltimer, ns): stamps[cta * kStampSlots + phase]
  const int lin = blockIdx.x + blockIdx.y * gridDim.x;
  auto stamp = [&](int phase) {
    if (stamps != nullptr) stamps[(size_t)lin * kStampSlots + phase] = (long long)globaltimer_ordered();
  };
  if (threadIdx.x == 0) stamp(kStEntry);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  float* red = reinterpret_cast<float*>(smem + C::PIPE);  // [cs][per][BN + 4] partial rows pushed here (CLUSTER)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::PIPE + C::RED);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;  // [2] accumulator ready for the epilogue
  uint64_t* tempty = tfull + 2;         // [2] accumulator drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* s_fail = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_issued = const_cast<int*>(s_fail) + 1;
  int* s_consumed = s_issued + 1;
  int* s_last = s_consumed + 1;
  int* s_contrib = s_last + 1;  // [kMaxContrib] workspace offsets of a tile's contributors

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = gridDim.x, cta = blockIdx.x;
  const int KT = (K + BK - 1) / BK, tiles = (N + BM - 1) / BM;
  const long long total = (long long)tiles * KT;
  long long beg, end;
  if (CLUSTER) {
    beg = (long long)blockIdx.x * KT + (long long)blockIdx.y * kps;
    end = min((long long)blockIdx.x * KT + KT, beg + kps);
  } else {
    beg = sk_beg(cta, total, P);
    end = sk_beg(cta + 1, total, P);
  }
  const int first_tile = (int)(beg / KT);

  if (threadIdx.x == 0) {
    if (Wp == nullptr) prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
    *s_fail = 0;
    *s_issued = 0;
    *s_consumed = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) stamp(kStSetup);
  // cluster split-K: peers push partial rows into this CTA's reduction area; the first half of a cluster
  // barrier here, its second half before the first push, makes sure every CTA of the cluster has started
  const bool split_cluster = CLUSTER && gridDim.y > 1;
  if (split_cluster) cluster_arrive_relaxed();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      // (tile, k-step) of flattened step g advanced incrementally: no 64-bit divisions in the loop.
      // Packed weights (Wp != nullptr): tile t, k-step k is the contiguous 16 KB block t * KT + k, stored
      // as the swizzled shared-memory image, so one bulk copy replaces the 2-D tensor load and each CTA
      // reads its whole share of the weights as one contiguous range.
      const int nsteps = (int)(end - beg);
      const int pre = min(C::STAGES, nsteps);
      const int k_beg = (int)(beg % KT), t_beg = (int)(beg / KT);
      auto load_w = [&](int s, int k, int t, long long g) {
        if (Wp != nullptr)
          bulk_load(sA + s * C::A_BYTES, Wp + (size_t)g * C::A_BYTES, C::A_BYTES, &full[s]);
        else
          tma_load_2d(sA + s * C::A_BYTES, &tmW, &full[s], k * BK, t * BM);
      };
      // weights first: they do not depend on the previous kernel
      {
        int k = k_beg, t = t_beg;
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], C::STAGE);
          load_w(i, k, t, beg + i);
          if (++k == KT) k = 0, ++t;
        }
        // the next l2pf weight tiles into L2 while the previous kernel finishes (later stages hit L2)
        for (int i = pre; i < min(nsteps, pre + l2pf); ++i) {
          if (Wp != nullptr)
            bulk_prefetch_l2(Wp + (size_t)(beg + i) * C::A_BYTES, C::A_BYTES);
          else
            tma_prefetch_l2(&tmW, k * BK, t * BM);
          if (++k == KT) k = 0, ++t;
        }
      }
      stamp(kStWeightsIssued);
      pdl_wait();
      stamp(kStPdlWait);
      int k = k_beg, t = t_beg;
      for (int i = 0; i < pre; ++i) {
        tma_load_2d(sB + i * C::B_BYTES, &tmX, &full[i], k * BK, 0);
        if (++k == KT) k = 0, ++t;
      }
      int issued = pre;
      for (int i = pre, s = pre % C::STAGES, ph = (pre / C::STAGES) & 1; i < nsteps; ++i) {
        if (!mbar_wait(&empty[s], ph ^ 1, timeout_ns) || *s_fail) {
          *s_fail = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::STAGE);
        load_w(s, k, t, beg + i);
        tma_load_2d(sB + s * C::B_BYTES, &tmX, &full[s], k * BK, 0);
        issued = i + 1;
        if (++k == KT) k = 0, ++t;
        if (++s == C::STAGES) s = 0, ph ^= 1;
      }
      *s_issued = issued;
      stamp(kStLastLoad);
      pdl_trigger();  // every load is issued: the next kernel may start its prologue
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = idesc_f16(BM, BN, BF16);
      int i = 0, j = 0;
      bool ok = true;
      for (long long g = beg; g < end && ok; ++j) {
        const int k0 = (int)(g % KT);
        const int k1 = (int)(((long long)KT < k0 + (end - g)) ? (long long)KT : k0 + (end - g));
        const int acc = j & 1;
        if (!mbar_wait(&tempty[acc], ((j >> 1) & 1) ^ 1, timeout_ns)) {
          *s_fail = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * C::TC;
        for (int k = k0; k < k1; ++k, ++i) {
          const int s = i % C::STAGES;
          if (!mbar_wait(&full[s], (i / C::STAGES) & 1, timeout_ns) || *s_fail) {
            *s_fail = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          if (i == 0) stamp(kStFirstFull);
          const uint32_t a = smem_addr(sA + s * C::A_BYTES), b = smem_addr(sB + s * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16(d, desc_k_sw128(a + kk * 32), desc_k_sw128(b + kk * 32), idesc, (k > k0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        mma_commit(&tfull[acc]);
        g += k1 - k0;
      }
      *s_consumed = i;
      stamp(kStLastMma);
    }
  } else {
    // ------------------------------------------------ epilogue: warps 2..5, TMEM lane quarter = warp % 4
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int mcols = min(M, BN);
    // cluster split-K: row `row` of this CTA's partial tile goes to the CTA that owns it (rows
    // [o * per, (o + 1) * per) belong to CTA o of the cluster), slot blockIdx.y of that CTA's reduction area
    float* push_dst = nullptr;
    if (split_cluster) {
      const int per = (BM + gridDim.y - 1) / gridDim.y;
      int o = row / per, slot = row - o * per;
      if (swiglu) {  // gate row f and up row 64 + f go to the same owner: slots [0, ph) gate, [ph, 2 ph) up
        const int ph = (BM / 2) / gridDim.y, f = row & (BM / 2 - 1);
        o = f / ph;
        slot = f - o * ph + (row >= BM / 2 ? ph : 0);
      }
      cluster_wait();  // every CTA of the cluster has started: its shared memory may be written
      push_dst = cg::this_cluster().map_shared_rank(red, o) + ((size_t)blockIdx.y * per + slot) * (BN + 4);
    }
    // stream-K SwiGLU: [64][BN] up-row values of the current tile, per CTA, past the partial slots
    float* xch = ws + (size_t)P * 2 * BN * BM + (size_t)cta * (BM / 2) * BN;
    int j = 0;
    for (long long g = beg; g < end; ++j) {
      const int t = (int)(g / KT);
      const int k0 = (int)(g % KT);
      const int k1 = (int)(((long long)KT < k0 + (end - g)) ? (long long)KT : k0 + (end - g));
      const int acc = j & 1;
      const int n = t * BM + row;
      const bool whole = (k0 == 0 && k1 == KT);
      if (!mbar_wait(&tfull[acc], (j >> 1) & 1, timeout_ns)) *s_fail = 1;
      __syncwarp();
      tc_fence_after();
      if (q == 2 && lane == 0) stamp(kStAccReady);
      const uint32_t taddr = tmem + acc * C::TC + ((uint32_t)(q * 32) << 16);
      // partial segments go to workspace slot 0 (first tile of this CTA) or 1 (its last tile),
      // row-major [row][BN] so the finisher reads 16-byte vectors; in cluster mode straight into the
      // owning CTA's shared memory (distributed shared memory stores; this is the CTA's only segment)
      float* part = CLUSTER ? push_dst
                            : ws + ((size_t)cta * 2 + (t == first_tile ? 0 : 1)) * BN * BM + (size_t)row * BN;
      float sw_gate[16];  // stream-K SwiGLU, whole tile: this gate row's 16 columns
      for (int c0 = 0; c0 < mcols; c0 += 16) {
        float v[16];
        tmem_ld16(taddr + c0, v);
        if (SW && whole) {
          if (q >= 2) {  // up rows: to the exchange area
#pragma unroll
            for (int jj = 0; jj < 16; jj += 4)
              *reinterpret_cast<float4*>(xch + (size_t)(row - BM / 2) * BN + jj) =
                  make_float4(v[jj], v[jj + 1], v[jj + 2], v[jj + 3]);
          } else {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) sw_gate[jj] = v[jj];
          }
        } else if (whole) {
          if (n < N) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              if (c0 + jj < M) store_out<BF16>(Y, (size_t)(c0 + jj) * ldy + n, v[jj]);
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 16; jj += 4)
            *reinterpret_cast<float4*>(part + c0 + jj) = make_float4(v[jj], v[jj + 1], v[jj + 2], v[jj + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (q == 2 && lane == 0) stamp(kStEpiDone);
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&tempty[acc])) : "memory");
      if (SW && whole) {
        epi_sync();  // the up rows are in the exchange area
        if (q < 2) {
          const float* up = xch + (size_t)row * BN;
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            if (jj < M) {
              const float gv = round_out<BF16>(sw_gate[jj]), uv = round_out<BF16>(up[jj]);
              store_out<BF16>(Y, (size_t)jj * ldy + t * (BM / 2) + row, gv / (1.f + __expf(-gv)) * uv);
            }
          }
        }
        epi_sync();  // the area is free for the next tile
      }
      if (!CLUSTER && !whole) {
        // last contributor of tile t sums every contributor's partial in CTA order
        const int cfirst = sk_owner((long long)t * KT, total, P);
        const int clast = sk_owner((long long)(t + 1) * KT - 1, total, P);
        const int nc = clast - cfirst + 1;
        __threadfence();
        epi_sync();
        if (q == 2 && lane == 0) *s_last = (atomicAdd(&tile_ctr[t], 1) == nc - 1);
        epi_sync();
        if (*s_last) {
          __threadfence();
          // contributor slot offsets, computed once per tile (64-bit divisions off the load path)
          for (int c = threadIdx.x - 64; c < nc && c < kMaxContrib; c += 128) {
            const int cc = cfirst + c;
            s_contrib[c] = (cc * 2 + ((t == (int)(sk_beg(cc, total, P) / KT)) ? 0 : 1)) * BN * BM;
          }
          epi_sync();
          const float* base = ws + (size_t)row * BN;
          const int ncap = nc < kMaxContrib ? nc : kMaxContrib;
          auto sum4 = [&](int c0) {  // columns c0..c0+3 of this row over every contributor, in CTA order
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            int c = 0;
            for (; c + 8 <= ncap; c += 8) {
              float4 v[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) v[u] = __ldcg(reinterpret_cast<const float4*>(base + s_contrib[c + u] + c0));
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                a.x += v[u].x;
                a.y += v[u].y;
                a.z += v[u].z;
                a.w += v[u].w;
              }
            }
            for (; c < ncap; ++c) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(base + s_contrib[c] + c0));
              a.x += v.x;
              a.y += v.y;
              a.z += v.z;
              a.w += v.w;
            }
            return a;
          };
          if (SW) {
            // the up rows' sums go through the exchange area to the threads of their gate rows
            float4 sw_sum[4];
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) sw_sum[c4] = 4 * c4 < mcols ? sum4(4 * c4) : make_float4(0.f, 0.f, 0.f, 0.f);
            if (q >= 2) {
#pragma unroll
              for (int c4 = 0; c4 < 4; ++c4)
                *reinterpret_cast<float4*>(xch + (size_t)(row - BM / 2) * BN + 4 * c4) = sw_sum[c4];
            }
            epi_sync();
            if (q < 2) {
#pragma unroll
              for (int c4 = 0; c4 < 4; ++c4) {
                const float4 u4 = *reinterpret_cast<const float4*>(xch + (size_t)row * BN + 4 * c4);
                const float gs[4] = {sw_sum[c4].x, sw_sum[c4].y, sw_sum[c4].z, sw_sum[c4].w};
                const float us[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  if (4 * c4 + u < M) {
                    const float gv = round_out<BF16>(gs[u]), uv = round_out<BF16>(us[u]);
                    store_out<BF16>(Y, (size_t)(4 * c4 + u) * ldy + t * (BM / 2) + row, gv / (1.f + __expf(-gv)) * uv);
                  }
                }
              }
            }
            epi_sync();
          } else {
            for (int c0 = 0; c0 < mcols; c0 += 4) {
              const float4 a = sum4(c0);
              if (n < N) {
                const float o[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
                  if (c0 + u < M) store_out<BF16>(Y, (size_t)(c0 + u) * ldy + n, o[u]);
              }
            }
          }
          if (q == 2 && lane == 0) tile_ctr[t] = 0;
        }
        epi_sync();
      }
      g += k1 - k0;
    }
  }

  // ------------------------------------------------ cluster split-K: sum the pushed partial rows (all threads)
  if (split_cluster) {
    if (warp < 2) cluster_wait();  // second half of the start-up barrier (the epilogue warps passed it)
    __syncthreads();               // warps 0 and 1 reconverged (their lane 0 had its own role)
    cg::this_cluster().sync();     // release / acquire: every partial row has reached its owner
    const int cs = gridDim.y, r = blockIdx.y, t = blockIdx.x;
    const int mcols = min(M, BN);
    const int per = (BM + cs - 1) / cs, r0 = r * per, nr = min(BM, r0 + per) - r0;
    const int ncol4 = (mcols + 3) / 4;
    if (swiglu) {
      const int ph = (BM / 2) / cs;
      for (int idx = threadIdx.x; idx < ph * ncol4; idx += kThreads) {
        const int lr = idx % ph, c4 = (idx / ph) * 4;
        float4 ga = make_float4(0.f, 0.f, 0.f, 0.f), ua = ga;
        for (int c = 0; c < cs; ++c) {  // sources in cluster order, as the plain sums
          const float4 g4 = *reinterpret_cast<const float4*>(red + ((size_t)c * per + lr) * (BN + 4) + c4);
          const float4 u4 = *reinterpret_cast<const float4*>(red + ((size_t)c * per + ph + lr) * (BN + 4) + c4);
          ga.x += g4.x;
          ga.y += g4.y;
          ga.z += g4.z;
          ga.w += g4.w;
          ua.x += u4.x;
          ua.y += u4.y;
          ua.z += u4.z;
          ua.w += u4.w;
        }
        const int nn = t * (BM / 2) + r * ph + lr;  // output feature
        if (nn < N / 2) {
          const float gv[4] = {ga.x, ga.y, ga.z, ga.w}, uv[4] = {ua.x, ua.y, ua.z, ua.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (c4 + u < M) {
              // gate and up rounded as a plain GEMM would store them, then SiLU(gate) * up in fp32
              const float g = round_out<BF16>(gv[u]), up = round_out<BF16>(uv[u]);
              store_out<BF16>(Y, (size_t)(c4 + u) * ldy + nn, g / (1.f + __expf(-g)) * up);
            }
          }
        }
      }
    }
    for (int idx = threadIdx.x; !swiglu && idx < nr * ncol4; idx += kThreads) {
      const int lr = idx % nr, c4 = (idx / nr) * 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = 0; c < cs; ++c) {  // sources in cluster order: deterministic
        const float4 v = *reinterpret_cast<const float4*>(red + ((size_t)c * per + lr) * (BN + 4) + c4);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int nn = t * BM + r0 + lr;
      if (nn < N) {
        const float o[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c4 + u < M) store_out<BF16>(Y, (size_t)(c4 + u) * ldy + nn, o[u]);
      }
    }
    // no second cluster barrier: after the one above nobody touches another CTA's shared memory
  }

  // ------------------------------------------------ teardown
  __syncthreads();
  if (threadIdx.x == 0) stamp(kStEnd);
  if (threadIdx.x == 0 && *s_fail) {
    atomicOr(err, 1);
    // drain TMA loads that were issued but never consumed before shared memory is released
    for (int i = *s_consumed; i < *s_issued; ++i) mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, timeout_ns);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// Row-major [rows, cols] 16-bit matrix, box = 64 columns (128 bytes, one swizzle span) x box_rows.
cudaError_t tensor_map(const void* ptr, int rows, int cols, int box_rows, bool bf16, CUtensorMap* out) {
  return tensor_map_2d(ptr, (uint64_t)rows, (uint64_t)cols, (uint64_t)cols * 2, (uint32_t)box_rows, (uint32_t)BK,
                       bf16, out);
}

template <int BN, bool BF16, bool SMALL>
cudaError_t launch_bn(const CUtensorMap& mw, const CUtensorMap& mx, void* Y, int M, int N, int K, int ctas, int ldy,
                      float* ws, int* ctr, int* err, unsigned long long timeout_ns, bool pdl, int splits,
                      cudaStream_t stream, const uint8_t* Wp, bool swiglu) {
  const bool clustered = splits > 0;
  const int smem = clustered ? Cfg<BN, SMALL, true>::SMEM : Cfg<BN, SMALL, false>::SMEM;
  // stream-K SwiGLU: its own instance (BN = 16 only; the host rejects it for wider batch tiles)
  const int form = clustered ? 1 : (swiglu && BN == 16 ? 2 : 0);
  auto fn = form == 1 ? k_gemm_streamk<BN, BF16, SMALL, true>
                      : (form == 2 ? k_gemm_streamk<BN, BF16, SMALL, false, BN == 16>
                                   : k_gemm_streamk<BN, BF16, SMALL, false>);
  static bool attr_set[3] = {false, false, false};
  if (!attr_set[form]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    if (clustered) {  // 9..16 splits: non-portable cluster sizes (narrow outputs such as QKV at TP = 8)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
    }
    attr_set[form] = true;
  }
  const int KT = (K + BK - 1) / BK;
  const int kps = clustered ? (KT + splits - 1) / splits : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = clustered ? dim3((N + BM - 1) / BM, (KT + kps - 1) / kps, 1) : dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (clustered && cfg.gridDim.y > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 1;
    attrs[na].val.clusterDim.y = cfg.gridDim.y;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl || pdl_flag()) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, fn, mw, mx, Y, M, N, K, ldy, ws, ctr, err, timeout_ns, kps, l2_prefetch_tiles(),
                            next_gemm_stamps(), Wp, (int)swiglu);
}

template <bool BF16, bool SMALL>
cudaError_t launch_bn_sel(const CUtensorMap& mw, const CUtensorMap& mx, int bn, void* Y, int M, int N, int K,
                          int ctas, int ldy, float* ws, int* ctr, int* err, unsigned long long t, bool pdl,
                          int splits, cudaStream_t s, const uint8_t* Wp, bool sw) {
  switch (bn) {
    case 16: return launch_bn<16, BF16, SMALL>(mw, mx, Y, M, N, K, ctas, ldy, ws, ctr, err, t, pdl, splits, s, Wp, sw);
    case 32: return launch_bn<32, BF16, SMALL>(mw, mx, Y, M, N, K, ctas, ldy, ws, ctr, err, t, pdl, splits, s, Wp, sw);
    case 64: return launch_bn<64, BF16, SMALL>(mw, mx, Y, M, N, K, ctas, ldy, ws, ctr, err, t, pdl, splits, s, Wp, sw);
    case 128: return launch_bn<128, BF16, SMALL>(mw, mx, Y, M, N, K, ctas, ldy, ws, ctr, err, t, pdl, splits, s, Wp, sw);
    case 256: return launch_bn<256, BF16, SMALL>(mw, mx, Y, M, N, K, ctas, ldy, ws, ctr, err, t, pdl, splits, s, Wp, sw);
    default: return cudaErrorInvalidValue;
  }
}

template <bool BF16>
cudaError_t launch_typed(const CUtensorMap& mw, const CUtensorMap& mx, int bn, void* Y, int M, int N, int K, int ctas,
                         int ldy, float* ws, int* ctr, int* err, unsigned long long t, bool pdl, bool small,
                         int splits, cudaStream_t s, const uint8_t* Wp, bool sw) {
  return small ? launch_bn_sel<BF16, true>(mw, mx, bn, Y, M, N, K, ctas, ldy, ws, ctr, err, t, pdl, splits, s, Wp, sw)
               : launch_bn_sel<BF16, false>(mw, mx, bn, Y, M, N, K, ctas, ldy, ws, ctr, err, t, pdl, splits, s, Wp, sw);
}

}  // namespace

long long*& gemm_stamps() {
  static long long* p = nullptr;
  return p;
}
long long& gemm_stamp_stride() {
  static long long s = 0;
  return s;
}
long long& gemm_stamp_launches() {
  static long long n = 0;
  return n;
}
long long* next_gemm_stamps() {
  long long* p = gemm_stamps();
  if (p == nullptr) return nullptr;
  return p + gemm_stamp_stride() * gemm_stamp_launches()++;
}

GemmPlan plan_gemm(int M, int N, int K, int num_sms, int ctas_override) {
  GemmPlan p = {};
  p.bn = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256)));
  p.tiles = (N + BM - 1) / BM;
  const int KT = (K + BK - 1) / BK;
  const long long total = (long long)p.tiles * KT;
  int ctas = ctas_override > 0 ? ctas_override : num_sms;
  if (ctas_override <= 0) {
    // wide batch tiles make split tiles expensive to finish: bound the CTAs sharing one tile
    const int max_share = p.bn <= 32 ? 32 : (p.bn <= 64 ? 8 : 4);
    ctas = (int)std::min<long long>(ctas, (long long)p.tiles * max_share);
  }
  p.ctas = (int)std::min<long long>(std::max(1, ctas), total);
  // a tile is shared by at most ceil(KT / (total / ctas)) + 1 CTAs; keep that within kMaxContrib
  while (p.ctas > 1 && ((long long)KT * p.ctas + total - 1) / total + 1 > kMaxContrib) --p.ctas;
  return p;
}

size_t gemm_workspace_bytes(int num_ctas, int bn) { return (size_t)num_ctas * 2 * BM * bn * sizeof(float); }

cudaError_t gemm_decode(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, float* ws,
                        size_t ws_bytes, int* tile_ctr, int max_tiles, int* err, int num_sms, int ctas_override,
                        bool pdl, bool small_smem, int cluster_splits, unsigned long long timeout_ns,
                        cudaStream_t stream, GemmPlan* used, bool packed, bool swiglu) {
  if (cluster_splits > 16 || (cluster_splits > 0 && M > 64)) return cudaErrorInvalidValue;
  if (swiglu) {
    if (N % BM) return cudaErrorInvalidValue;
    if (cluster_splits > 0) {  // cluster split-K whose split count divides 64 (gate / up row pairs split evenly)
      const int KT = (K + BK - 1) / BK, kps = (KT + cluster_splits - 1) / cluster_splits, s = (KT + kps - 1) / kps;
      if (s < 2 || (BM / 2) % s) return cudaErrorInvalidValue;
    } else if (M > 16) {  // stream-K: the 16-column batch tile only
      return cudaErrorInvalidValue;
    }
  }
  if (M <= 0 || M > 256 || N <= 0 || K <= 0 || K % 8 || (dtype != kBF16 && dtype != kF16))
    return cudaErrorInvalidValue;
  // packed weights: whole 128 x 64 blocks, 16-byte aligned
  if (packed && (K % BK || (reinterpret_cast<uintptr_t>(W) & 15))) return cudaErrorInvalidValue;
  const GemmPlan p = plan_gemm(M, N, K, num_sms, ctas_override);
  if (used) *used = p;
  // stream-K SwiGLU also uses a [64][bn] exchange area per CTA past the partial slots
  const size_t ws_need = gemm_workspace_bytes(p.ctas, p.bn) +
                         (swiglu && cluster_splits <= 0 ? (size_t)p.ctas * (BM / 2) * p.bn * sizeof(float) : 0);
  if (p.tiles > max_tiles || ws_need > ws_bytes) return cudaErrorInvalidValue;
  const bool bf16 = dtype == kBF16;
  CUtensorMap mw = {}, mx;
  cudaError_t e = packed ? cudaSuccess : tensor_map(W, N, K, BM, bf16, &mw);
  if (e != cudaSuccess) return e;
  e = tensor_map(X, M, K, p.bn, bf16, &mx);
  if (e != cudaSuccess) return e;
  const uint8_t* Wp = packed ? static_cast<const uint8_t*>(W) : nullptr;
  return bf16 ? launch_typed<true>(mw, mx, p.bn, Y, M, N, K, p.ctas, ldy, ws, tile_ctr, err, timeout_ns, pdl,
                                   small_smem, cluster_splits, stream, Wp, swiglu)
              : launch_typed<false>(mw, mx, p.bn, Y, M, N, K, p.ctas, ldy, ws, tile_ctr, err, timeout_ns, pdl,
                                    small_smem, cluster_splits, stream, Wp, swiglu);
}

}  // namespace cob
