// Layer-boundary fusion for tensor-parallel decode on sm_100a (see fused_gemm.h for the contract).
//
// The reference stops at a fused all-reduce + residual + RMSNorm kernel between separate GEMMs
// (exp/M17_epoch_ab/fused_ar_norm_nf.cu:90-199); its design notes name the GEMM-epilogue fusion as
// the next step. Here both neighbouring GEMMs absorb the collective:
//
// gemm_push (row-parallel GEMM -> all-reduce input)
//   warp 0 : TMA producer (weights issued before the programmatic-dependent-launch wait)
//   warp 1 : tcgen05.mma issuer, fp32 accumulator in TMEM
//   warps 2-5 : epilogue. TMEM -> shared memory transposed to [batch row][feature]; the splits of a
//           tile (one thread-block cluster) sum their partial tiles through DSMEM, and every CTA
//           stores its share of the tile as 16-byte bf16 vectors, Lamport-encoded (-0 -> +0), into
//           land1[slot][this rank][row][:] of EVERY rank's heap (NVLink 5 stores; own heap locally).
//           The per-output transfer overlaps the other tiles' MMAs; no local Y is ever written.
//
// ar_norm_gemm (all-reduce + residual + RMSNorm -> column-parallel GEMM)
//   warp 0 : weight tiles for the first ring slots at once (they do not depend on anything), then
//            waits for the activation pieces of its split and streams activation + weight tiles.
//            Launched with programmatic dependent launch, the weight stream overlaps the tail of the
//            preceding gemm_push; the pieces wait for it to complete (griddepcontrol.wait) first.
//   warp 1 : tcgen05.mma issuer.
//   warps 2-5 : first the "piece" of the all-reduce this CTA owns: a [M, ~K / CTAs] block of the
//            landing buffers, polled per 16-byte vector (Lamport), summed over ranks with the
//            residual (h, rounded to the activation type, written back to the residual in place),
//            h * gamma staged to global memory for the TMA, the per-row sum of squares of the piece
//            stored, the landing vectors restored to -0, then a per-piece flag = epoch (release).
//            Then the epilogue: rstd per row from all pieces' sums (per split with a warp tree, then
//            across the cluster through DSMEM, fixed order: deterministic), partial tiles summed
//            over the cluster, scaled by rstd, stored as bf16 - or, with a paired epilogue, each CTA
//            finishes row pairs (f, 64 + f) of its tile: SiLU(gate) * up (the gate_up projection,
//            weights interleaved per tile) or RoPE + paged-KV append (the QKV projection, one head
//            per tile), which removes the separate SiLU and RoPE kernels from the decode step.
//   RMSNorm folds into the GEMM: Z = (h * gamma * rstd) W^T = rstd * ((h * gamma) W^T) per row.
//
// CTAs of ar_norm_gemm wait for pieces written by other CTAs of the same launch, so the host only
// launches grids that fit on the GPU at once (tiles x splits <= SMs x resident CTAs per SM); every
// wait is bounded (%globaltimer) and a timeout sets the rank's error word and *err.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>

#include "fused_gemm.h"
#include "sm100.cuh"
#include "tma_host.h"

namespace cob {
namespace {

namespace cg = cooperative_groups;
using namespace sm100;

constexpr int BM = 128, BK = 64;
constexpr int kThreads = 192;
constexpr int kPitch = BM + 4;     // floats per batch row of the transposed partial tile
constexpr int kQCap = 2048;        // ar_norm_gemm: floats of per-item sums of squares in shared memory

template <int BN, bool SMALL>
struct FCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BUDGET = SMALL ? 100 * 1024 : 200 * 1024;
  static constexpr int PART = BN * kPitch * 4;
  static constexpr int STAGES_RAW = BUDGET / STAGE;
  static constexpr int STAGES = STAGES_RAW > 12 ? 12 : STAGES_RAW;
  static constexpr int RING = STAGES * STAGE;
  static constexpr int PIPE = RING > PART ? RING : PART;
  static constexpr int CTRL = 1024 + BN * 8;  // barriers, flags, per-row sums / rstd
  // batch tile 16: area into which the cluster's CTAs push partial rows and row sums of squares (the
  // consumer's one-barrier reduction; outside the ring, the piece buffers and `q`)
  static constexpr int RED = BN == 16 ? (BN * BM + 16 * BN) * 4 : 0;
  static constexpr int SMEM = PIPE + 1024 + CTRL + kQCap * 4 + RED;
  static constexpr int TC = BN < 32 ? 32 : BN;  // TMEM columns per accumulator (two are allocated)
  // SMALL: two CTAs per SM (228 KB per SM, 1 KB reserved per CTA)
  static_assert(!SMALL || SMEM <= 113 * 1024, "two CTAs per SM");
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

struct Ctrl {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* tfull;   // [2]
  uint64_t* tempty;  // [2]
  uint32_t* tmem_slot;
  volatile int* fail;
  int* issued;
  int* consumed;
  float* ss;     // [BN] this split's per-row sum of squares (ar_norm_gemm)
  float* rstd;   // [BN]
  float* q;      // [kQCap] per-item sums of squares (ar_norm_gemm)
  float* red;    // batch tile 16: [cs][BN][BM / cs] partial rows pushed by the cluster (ar_norm_gemm)
  float* red_ss; // batch tile 16: [cs][BN] per-split row sums of squares pushed by the cluster
};

template <int BN, bool SMALL>
__device__ __forceinline__ Ctrl carve(uint8_t* smem) {
  using C = FCfg<BN, SMALL>;
  Ctrl c;
  uint8_t* ctrl = smem + C::PIPE;
  c.full = reinterpret_cast<uint64_t*>(ctrl);
  c.empty = c.full + C::STAGES;
  c.tfull = c.empty + C::STAGES;
  c.tempty = c.tfull + 2;
  c.tmem_slot = reinterpret_cast<uint32_t*>(c.tempty + 2);
  c.fail = reinterpret_cast<volatile int*>(c.tmem_slot + 1);
  c.issued = const_cast<int*>(c.fail) + 1;
  c.consumed = c.issued + 1;
  c.ss = reinterpret_cast<float*>(ctrl + 1024);
  c.rstd = c.ss + BN;
  c.q = reinterpret_cast<float*>(ctrl + C::CTRL);
  c.red = c.q + kQCap;
  c.red_ss = c.red + BN * BM;
  return c;
}

__device__ __forceinline__ RankState* fg_state(const FusedGemmParams& p, int r) {
  return reinterpret_cast<RankState*>(p.base[r] + p.L.state);
}
__device__ __forceinline__ uint4* fg_land(const FusedGemmParams& p, int owner, int slot, int src, int row, int v) {
  return COB_IN_RANGE(
      reinterpret_cast<uint4*>(p.base[owner] + p.L.land1) +
          ((((size_t)slot * p.L.world + src) * p.L.max_rows + row) * p.L.max_hv + v),
      (unsigned)owner < (unsigned)p.L.world && (unsigned)slot < 2u && (unsigned)src < (unsigned)p.L.world &&
          (unsigned)row < (unsigned)p.L.max_rows && (unsigned)v < (unsigned)p.L.max_hv,
      &reinterpret_cast<RankState*>(p.base[p.emulate ? blockIdx.z : p.rank] + p.L.state)->error);
}
__device__ __forceinline__ int lin_block() { return blockIdx.x + gridDim.x * blockIdx.y; }
__device__ __forceinline__ uint64_t fg_epoch(const FusedGemmParams& p, int rank) {
  return ld_vol_u64(&fg_state(p, rank)->blk_epoch[lin_block() % kMaxBlocks]) + 1;
}

__device__ __forceinline__ void fg_error(const FusedGemmParams& p, int rank, uint32_t bit, uint64_t where,
                                         uint64_t e) {
  RankState* st = fg_state(p, rank);
  if (atomicOr(&st->error, bit) == 0u) {
    st->err_detail[0] = (uint64_t)0xF6 << 32;  // fused-GEMM kernels
    st->err_detail[1] = where;
    st->err_detail[2] = lin_block();
    st->err_detail[3] = e;
  }
  atomicOr(p.err, 1);
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void st_release_u32(void* ptr, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const void* ptr) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
// Named barrier among warps 2-5.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Warp-wide wait until flags[i] == tag for every i in [0, n). Returns false on timeout.
__device__ bool wait_flags(const uint32_t* flags, int n, uint32_t tag, uint64_t timeout_ns, const volatile int* fail) {
  const int lane = threadIdx.x & 31;
  uint64_t t0 = 0;
  for (int i = lane; i < ((n + 31) & ~31); i += 32) {
    bool done = i >= n;
    uint32_t spins = 0;
    while (!__all_sync(0xffffffffu, done)) {
      if (!done) done = ld_acquire_gpu_u32(flags + i) == tag;
      if ((++spins & 63u) == 0u) {
        const uint64_t t = globaltimer();
        if (t0 == 0) t0 = t;
        const bool out = (t - t0 > timeout_ns) || (fail != nullptr && *fail);
        if (__any_sync(0xffffffffu, out)) return false;
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------------------------------------
// Main loop shared by both kernels: warp 0 producer, warp 1 MMA issuer. The CTA computes `nt` output
// tiles (rows wrow + i * wstride, i < nt) over the same k-range; accumulators alternate between two
// TMEM buffers so the epilogue of one tile overlaps the MMAs of the next.
// WAIT_ACT: the activation loads wait for the pieces of this split (ar_norm_gemm).
// ---------------------------------------------------------------------------------------------
template <int BN, bool SMALL, bool WAIT_ACT>
__device__ __forceinline__ void mainloop(const FusedGemmParams& p, const CUtensorMap* tmW, const CUtensorMap* tmB,
                                         uint8_t* smem, const Ctrl& c, uint32_t tmem, int k0, int nsteps, int wrow,
                                         int wstride, int nt, int brow, const uint32_t* split_flags, int nflags,
                                         uint32_t tag, int wtile0) {
  using C = FCfg<BN, SMALL>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  const int total = nt * nsteps;
  if (warp == 0) {
    const int pre = min(C::STAGES, total);
    auto wr = [&](int i) { return wrow + (i / nsteps) * wstride; };
    auto kx = [&](int i) { return (k0 + i % nsteps) * BK; };
    // packed weights (p.wp): 16 KB block (tile, k-step) of this rank at wp + (tile * KT + k) * 16 KB
    const int KT = p.K / BK;
    auto wblock = [&](int i) {
      return p.wp + ((size_t)(wtile0 + (i / nsteps) * (wstride / BM)) * KT + (k0 + i % nsteps)) * C::A_BYTES;
    };
    auto load_w = [&](int s, int i) {
      if (p.wp != nullptr)
        bulk_load(sA + s * C::A_BYTES, wblock(i), C::A_BYTES, &c.full[s]);
      else
        tma_load_2d(sA + s * C::A_BYTES, tmW, &c.full[s], kx(i), wr(i));
    };
    if (lane == 0) {
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&c.full[i], C::STAGE);
        load_w(i, i);
      }
      // the next weight tiles into L2 while the activations are awaited (later stages then hit L2)
      for (int i = pre; i < min(total, pre + p.l2_prefetch); ++i) {
        if (p.wp != nullptr)
          bulk_prefetch_l2(wblock(i), C::A_BYTES);
        else
          tma_prefetch_l2(tmW, kx(i), wr(i));
      }
      if (!WAIT_ACT) pdl_wait();
    }
    bool ok = true;
    if (WAIT_ACT) {
      ok = wait_flags(split_flags, nflags, tag, p.timeout_ns, c.fail);
      if (!ok && lane == 0) *c.fail = 1;
      fence_proxy_async_global();
    }
    if (lane == 0) {
      int issued = pre;
      // the ring's first stages expect activation bytes too: on failure they are loaded anyway
      // (contents unused, the CTA reports failure) so every issued stage completes and can be drained
      for (int i = 0; i < pre; ++i) tma_load_2d(sB + i * C::B_BYTES, tmB, &c.full[i], kx(i), brow);
      if (ok) {
        for (int i = pre; i < total; ++i) {
          const int s = i % C::STAGES;
          if (!mbar_wait(&c.empty[s], ((i / C::STAGES) & 1) ^ 1, p.timeout_ns) || *c.fail) {
            *c.fail = 1;
            break;
          }
          mbar_arrive_expect_tx(&c.full[s], C::STAGE);
          load_w(s, i);
          tma_load_2d(sB + s * C::B_BYTES, tmB, &c.full[s], kx(i), brow);
          issued = i + 1;
        }
      }
      *c.issued = issued;
      pdl_trigger();  // every load is issued: the next kernel may start its prologue
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BM, BN, true);
      int i = 0;
      bool ok = true;
      for (int tile = 0; tile < nt && ok; ++tile) {
        const int acc = tile & 1;
        if (!mbar_wait(&c.tempty[acc], ((tile >> 1) & 1) ^ 1, p.timeout_ns)) {
          *c.fail = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * C::TC;
        for (int k = 0; k < nsteps; ++k, ++i) {
          const int s = i % C::STAGES;
          if (!mbar_wait(&c.full[s], (i / C::STAGES) & 1, p.timeout_ns) || *c.fail) {
            *c.fail = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_addr(sA + s * C::A_BYTES), b = smem_addr(sB + s * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16(d, desc_k_sw128(a + kk * 32), desc_k_sw128(b + kk * 32), idesc, (k > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&c.empty[s]);
        }
        mma_commit(&c.tfull[acc]);
      }
      *c.consumed = i;
    }
  }
}

// Epilogue part 1 (warps 2-5): accumulator tile -> shared memory, transposed to [batch row][feature].
template <int BN, bool SMALL>
__device__ __forceinline__ void tile_to_smem(const FusedGemmParams& p, uint8_t* smem, const Ctrl& c, uint32_t tmem,
                                             int M) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, row = q * 32 + lane;
  if (!mbar_wait(&c.tfull[0], 0, p.timeout_ns)) *c.fail = 1;
  __syncwarp();
  tc_fence_after();
  float* part = reinterpret_cast<float*>(smem);  // single tile per CTA: the drained ring holds it
  const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
  const int mcols = min(M, BN);
  for (int c0 = 0; c0 < mcols; c0 += 16) {
    float v[16];
    tmem_ld16(taddr + c0, v);
#pragma unroll
    for (int j = 0; j < 16; ++j) part[(c0 + j) * kPitch + row] = v[j];
  }
  tc_fence_before();
}

// Cluster barrier halves (non-aligned forms: lanes of a warp may reach them at different points).
__device__ __forceinline__ void cl_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
__device__ __forceinline__ void cl_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }

// gemm_push with a small batch tile (BN * BM floats fit the per-item area `c.q`, unused by this kernel):
// accumulator row `row` (one output feature) goes straight from TMEM to the CTA of the cluster that
// pushes that feature - owner o = row / per - as red_o[r][b][row - o * per] (distributed shared memory
// stores), so the cluster needs one barrier and no remote loads before the owners sum and push.
template <int BN, bool SMALL>
__device__ __forceinline__ void tile_to_owners(const FusedGemmParams& p, const Ctrl& c, uint32_t tmem, int M) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, row = q * 32 + lane;
  const int cs = gridDim.y, r = blockIdx.y, per = BM / cs, o = row / per;
  if (!mbar_wait(&c.tfull[0], 0, p.timeout_ns)) *c.fail = 1;
  __syncwarp();
  tc_fence_after();
  cl_wait();  // every CTA of the cluster has started: its shared memory may be written
  float* dst = cg::this_cluster().map_shared_rank(c.q, o) + (size_t)r * BN * per + (row - o * per);
  const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
  const int mcols = min(M, BN);
  for (int c0 = 0; c0 < mcols; c0 += 16) {
    float v[16];
    tmem_ld16(taddr + c0, v);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c0 + j < mcols) dst[(size_t)(c0 + j) * per] = v[j];
  }
  tc_fence_before();
}

// ar_norm_gemm with a batch tile of 16: accumulator row `row` to the CTA that finishes it - plain
// epilogue: owner row / (BM / cs); paired epilogue (rows f and 64 + f together): owner (row % 64) / ph,
// the low half at [0, ph) and the high half at [ph, 2 ph) of the owner's per-source slice.
template <int BN, bool SMALL>
__device__ __forceinline__ void consumer_tile_to_owners(const FusedGemmParams& p, const Ctrl& c, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, row = q * 32 + lane;
  const int cs = gridDim.y, r = blockIdx.y, per = BM / cs;
  int o, lf;
  if (p.epi == kEpiPlain) {
    o = row / per;
    lf = row - o * per;
  } else {
    const int ph = (BM / 2) / cs, f = row % (BM / 2);
    o = f / ph;
    lf = (row < BM / 2 ? 0 : ph) + f - o * ph;
  }
  if (!mbar_wait(&c.tfull[0], 0, p.timeout_ns)) *c.fail = 1;
  __syncwarp();
  tc_fence_after();
  float* dst = cg::this_cluster().map_shared_rank(c.red, o) + (size_t)r * BN * per + lf;
  const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
  const int mcols = min(p.M, BN);
  for (int c0 = 0; c0 < mcols; c0 += 16) {
    float v[16];
    tmem_ld16(taddr + c0, v);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (c0 + j < mcols) dst[(size_t)(c0 + j) * per] = v[j];
  }
  tc_fence_before();
}

// Sum over the cluster's sources of 8 pushed values at owner-local index `lf` of batch row b.
template <int BN>
__device__ __forceinline__ void red_sum8(const float* red, int cs, int per, int b, int lf, float (&acc)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  for (int cc = 0; cc < cs; ++cc) {
    const float* src = red + ((size_t)cc * BN + b) * per + lf;
    const float4 u = *reinterpret_cast<const float4*>(src);
    const float4 w = *reinterpret_cast<const float4*>(src + 4);
    acc[0] += u.x;
    acc[1] += u.y;
    acc[2] += u.z;
    acc[3] += u.w;
    acc[4] += w.x;
    acc[5] += w.y;
    acc[6] += w.z;
    acc[7] += w.w;
  }
}

// Sum of this CTA's feature share [f0, f0 + 8) of batch row b over the cs CTAs of the cluster.
__device__ __forceinline__ void cluster_sum8(float* part, int cs, int b, int f, float (&acc)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  cg::cluster_group cluster = cg::this_cluster();
  for (int cc = 0; cc < cs; ++cc) {
    const float* src = (cs > 1 ? cluster.map_shared_rank(part, cc) : part) + (size_t)b * kPitch + f;
    const float4 u = *reinterpret_cast<const float4*>(src);
    const float4 w = *reinterpret_cast<const float4*>(src + 4);
    acc[0] += u.x;
    acc[1] += u.y;
    acc[2] += u.z;
    acc[3] += u.w;
    acc[4] += w.x;
    acc[5] += w.y;
    acc[6] += w.z;
    acc[7] += w.w;
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&a)[8]) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return r;
}

template <int BN, bool SMALL>
__device__ __forceinline__ void teardown(const FusedGemmParams& p, const Ctrl& c, uint32_t tmem, int rank) {
  using C = FCfg<BN, SMALL>;
  __syncthreads();
  if (threadIdx.x == 0 && *c.fail) {
    fg_error(p, rank, kErrTimeoutLanding, 0xF60000u, 0);
    // drain every TMA load still in flight before the shared memory is released
    for (int i = *c.consumed; i < *c.issued; ++i) mbar_wait(&c.full[i % C::STAGES], (i / C::STAGES) & 1, p.timeout_ns);
  }
  tc_fence_before();
  __syncthreads();
  if ((threadIdx.x >> 5) == 1) tmem_dealloc(tmem, 2 * C::TC);
}

template <int BN, bool SMALL>
__device__ __forceinline__ uint32_t setup(uint8_t* smem, const Ctrl& c, int full_count, const CUtensorMap* a,
                                          const CUtensorMap* b) {
  using C = FCfg<BN, SMALL>;
  if (threadIdx.x == 0) {
    if (a != nullptr) prefetch_tmap(a);
    prefetch_tmap(b);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&c.full[s], full_count);
      mbar_init(&c.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&c.tfull[a], 1);
      mbar_init(&c.tempty[a], 4);  // one arrival per epilogue warp
    }
    *c.fail = 0;
    *c.issued = 0;
    *c.consumed = 0;
    fence_barrier_init();
  }
  if ((threadIdx.x >> 5) == 1) tmem_alloc(c.tmem_slot, 2 * C::TC);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return *c.tmem_slot;
}

// ---------------------------------------------------------------------------------------------
// gemm_push
// ---------------------------------------------------------------------------------------------
template <int BN, bool SMALL>
__global__ void __launch_bounds__(kThreads, SMALL ? 2 : 1)
    k_gemm_push(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                const FusedGemmParams p) {
  using LP = LamportOf<__nv_bfloat16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Ctrl c = carve<BN, SMALL>(smem);
  const int rank = p.emulate ? (int)blockIdx.z : p.rank;
  const int t = blockIdx.x, r = blockIdx.y, cs = gridDim.y;
  const int KT = p.K / BK;
  const int k0 = r * p.kps, nsteps = min(KT, k0 + p.kps) - k0;
  const uint32_t tmem = setup<BN, SMALL>(smem, c, 1, p.wp != nullptr ? nullptr : &tmW, &tmX);
  // small batch tile: partial rows are pushed to their owner CTA (one cluster barrier); else every CTA
  // keeps its tile and the owners read the peers' tiles (two barriers)
  constexpr bool kPushRed = BN * BM <= kQCap;
  const bool push_red = kPushRed && cs > 1;
  if (push_red) cl_arrive_relaxed();  // first half of a start-up barrier, waited for before the first push

  mainloop<BN, SMALL, false>(p, &tmW, &tmX, smem, c, tmem, k0, nsteps, (p.emulate ? rank * p.N : 0) + t * BM, 0, 1,
                             p.emulate ? rank * p.M : 0, nullptr, 0, 0u, (p.emulate ? rank : 0) * p.w_tiles + t);
  if (threadIdx.x >= 64) {
    if (push_red)
      tile_to_owners<BN, SMALL>(p, c, tmem, p.M);
    else
      tile_to_smem<BN, SMALL>(p, smem, c, tmem, p.M);
  } else if (push_red) {
    cl_wait();  // warps 0 and 1: second half of the start-up barrier
  }
  pdl_wait();  // every thread: the epoch below was written by an earlier kernel of the stream
  const uint64_t e = fg_epoch(p, rank);
  const int slot = (int)(e & 1);
  __syncthreads();
  if (cs > 1) cg::this_cluster().sync();  // release / acquire: partial tiles (or pushed rows) complete
  // this CTA pushes features [f0, f0 + per) of the tile for every batch row, 8 per 16-byte vector
  const int per = BM / cs, f0 = r * per, groups = per / 8;
  if (!*c.fail) {
    float* part = reinterpret_cast<float*>(smem);
    for (int idx = threadIdx.x; idx < p.M * groups; idx += kThreads) {
      const int b = idx / groups, f = f0 + (idx % groups) * 8;
      const int n = t * BM + f;
      if (n >= p.N) continue;
      float acc[8];
      if (push_red) {  // sources in cluster order from the local area: the sums of cluster_sum8
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int cc = 0; cc < cs; ++cc) {
          const float* src = c.q + ((size_t)cc * BN + b) * per + (f - f0);
          const float4 u = *reinterpret_cast<const float4*>(src);
          const float4 w = *reinterpret_cast<const float4*>(src + 4);
          acc[0] += u.x;
          acc[1] += u.y;
          acc[2] += u.z;
          acc[3] += u.w;
          acc[4] += w.x;
          acc[5] += w.y;
          acc[6] += w.z;
          acc[7] += w.w;
        }
      } else {
        cluster_sum8(part, cs, b, f, acc);
      }
      const uint4 d = LP::clean(pack_bf16x8(acc));
      for (int i = 0; i < p.world; ++i) {
        const int q = (rank + i) % p.world;  // start with the own heap, then peers in ring order
        st_vol_v4(fg_land(p, q, slot, rank, b, n / 8), d);
      }
    }
  }
  // the two-barrier form keeps this CTA's tile alive until the cluster has read it
  if (cs > 1 && !push_red) cg::this_cluster().sync();
  teardown<BN, SMALL>(p, c, tmem, rank);
}

// ---------------------------------------------------------------------------------------------
// ar_norm_gemm
// ---------------------------------------------------------------------------------------------
template <int BN, bool SMALL>
__global__ void __launch_bounds__(kThreads, SMALL ? 2 : 1)
    k_ar_norm_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                   const FusedGemmParams p) {
  using LP = LamportOf<__nv_bfloat16>;
  using V = Vec<__nv_bfloat16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Ctrl c = carve<BN, SMALL>(smem);
  const int rank = p.emulate ? (int)blockIdx.z : p.rank;
  const int wsr = p.emulate ? rank : 0;  // workspace index of this rank (one set per process otherwise)
  // X CTAs along x; CTA x computes tiles x, x + X, ... (several only when splits == 1)
  const int t = blockIdx.x, r = blockIdx.y, cs = gridDim.y, tiles = gridDim.x;
  const int ntiles = (p.N + BM - 1) / BM, nt = (ntiles - t + tiles - 1) / tiles;
  const int KT = p.K / BK, KV = p.K / 8;
  const int k0 = r * p.kps, nsteps = min(KT, k0 + p.kps) - k0;
  const int piece = r * tiles + t;
  uint32_t* flags = p.flags + (size_t)wsr * kMaxPieces;
  float* pss = p.pss + (size_t)wsr * kMaxPieces * p.act_rows;
  const uint32_t tmem = setup<BN, SMALL>(smem, c, 1, p.wp != nullptr ? nullptr : &tmW, &tmA);
  // batch tile 16: the split-K partial rows and row sums of squares are pushed to the CTA that finishes
  // them (one cluster barrier, no remote loads); the first half of a start-up barrier here, its second
  // half before the first push
  const bool push_red = BN == 16 && cs > 1;
  if (push_red) cl_arrive_relaxed();
  // The weight stream needs nothing from earlier kernels and starts at once (warp 0). The pieces
  // (warps 2-5) first wait, in hardware, for the preceding kernel - this rank's gemm_push - to
  // complete, so on this GPU nothing spins on a kernel that runs concurrently; the polls that
  // follow only wait for the other ranks' pushes. The epoch was written by a kernel that completed
  // before the preceding one passed its own wait.
  const uint64_t e = fg_epoch(p, rank);
  const uint32_t tag = (uint32_t)e;
  const int slot = (int)(e & 1);

  mainloop<BN, SMALL, true>(p, &tmW, &tmA, smem, c, tmem, k0, nsteps, (p.emulate ? rank * p.N : 0) + t * BM,
                            tiles * BM, nt, wsr * p.act_rows, flags + (size_t)r * tiles, tiles, tag,
                            (p.emulate ? rank : 0) * p.w_tiles + t);

  if (threadIdx.x >= 64) {
    const int tid = threadIdx.x - 64;
    pdl_wait();
    // ---------------- this CTA's piece of the all-reduce: vectors [vb, ve) of every row
    const int s0 = k0 * 8, slen = min(KV, (k0 + p.kps) * 8) - s0;
    const int vb = s0 + (int)((long long)slen * t / tiles), ve = s0 + (int)((long long)slen * (t + 1) / tiles);
    const int len = ve - vb, items = p.M * len;
    __nv_bfloat16* res = reinterpret_cast<__nv_bfloat16*>(p.residual) + (size_t)rank * p.res_rs;
    const uint4* gam = reinterpret_cast<const uint4*>(p.gamma);
    uint4* act = reinterpret_cast<uint4*>(p.act) + (size_t)(p.emulate ? rank * p.act_rows : 0) * KV;
    Waiter w(p.timeout_ns, &fg_state(p, rank)->error);
    bool ok = !*c.fail;
    constexpr int U = 2;  // items in flight per thread
    for (int i0 = tid; i0 < items && ok; i0 += 128 * U) {
      uint4 d[U][kMaxWorld], rv[U], gv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int it = i0 + u * 128;
        if (it < items) {
          const int b = it / len, v = vb + it % len;
#pragma unroll
          for (int s = 0; s < kMaxWorld; ++s)
            if (s < p.world) d[u][s] = ld_vol_v4(fg_land(p, rank, slot, s, b, v));
          rv[u] = reinterpret_cast<const uint4*>(res + (size_t)b * p.K)[v];
          gv[u] = ld_nc_v4(gam + v);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int it = i0 + u * 128;
        if (it >= items) continue;
        const int b = it / len, v = vb + it % len;
        float a[8], f[8];
        V::to_float(rv[u], a);
#pragma unroll
        for (int s = 0; s < kMaxWorld; ++s) {
          if (s >= p.world) break;
          while (ok && !LP::ready(d[u][s])) {
            if (w.expired()) {
              fg_error(p, rank, kErrTimeoutLanding, ((uint64_t)b << 32) | (uint64_t)v, e);
              *c.fail = 1;
              ok = false;
            } else {
              d[u][s] = ld_vol_v4(fg_land(p, rank, slot, s, b, v));
            }
          }
          V::to_float(d[u][s], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] += f[j];
        }
        const uint4 hb = V::from_float(a);  // h in the activation type; the norm uses these values
        V::to_float(hb, a);
        V::to_float(gv[u], f);
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          ss += a[j] * a[j];
          f[j] *= a[j];
        }
        reinterpret_cast<uint4*>(res + (size_t)b * p.K)[v] = hb;
        act[(size_t)b * KV + v] = V::from_float(f);
        c.q[it] = ss;
#pragma unroll
        for (int s = 0; s < kMaxWorld; ++s)
          if (s < p.world) st_vol_v4(fg_land(p, rank, slot, s, b, v), LP::fill());
      }
    }
    fence_proxy_async_global();  // act is read by TMA (async proxy) in other CTAs
    epi_sync();
    // per-row sum of squares of the piece, in item order (deterministic)
    for (int b = tid; b < p.M; b += 128) {
      float s = 0.f;
      for (int j = 0; j < len; ++j) s += c.q[b * len + j];
      pss[(size_t)piece * p.act_rows + b] = s;
    }
    __threadfence();
    epi_sync();
    if (tid == 0 && !*c.fail) st_release_u32(flags + piece, tag);

    // ---------------- epilogue
    // this split's per-row sum of squares over its pieces: lanes stride the pieces, warp tree
    const int warp = (threadIdx.x >> 5) - 2, lane = threadIdx.x & 31;
    if (!wait_flags(flags + (size_t)r * tiles, tiles, tag, p.timeout_ns, c.fail)) *c.fail = 1;
    if (push_red) cl_wait();  // every CTA of the cluster has started: its shared memory may be written
    for (int b = warp; b < p.M; b += 4) {
      float s = 0.f;
      for (int j = lane; j < tiles; j += 32) s += __ldcg(pss + (size_t)(r * tiles + j) * p.act_rows + b);
      s = warp_sum(s);
      if (lane == 0) {
        c.ss[b] = s;
        c.rstd[b] = rsqrtf(s / (float)p.K + p.eps);  // final when splits == 1
      }
      if (push_red && lane < cs) cg::this_cluster().map_shared_rank(c.red_ss, lane)[r * BN + b] = s;
    }
    if (cs == 1) {
      // several tiles per CTA: accumulator -> registers -> scaled bf16 stores, row-major Y
      epi_sync();
      const int q = (threadIdx.x >> 5) & 3;  // TMEM lane quarter a warp may access: warp id % 4
      __nv_bfloat16* Y = reinterpret_cast<__nv_bfloat16*>(p.Y) + (p.emulate ? (size_t)rank * p.M * p.N : 0);
      using C = FCfg<BN, SMALL>;
      for (int i = 0; i < nt; ++i) {
        const int acc = i & 1;
        if (!mbar_wait(&c.tfull[acc], (i >> 1) & 1, p.timeout_ns)) *c.fail = 1;
        __syncwarp();
        tc_fence_after();
        const int n = (t + i * tiles) * BM + q * 32 + lane;
        const uint32_t taddr = tmem + acc * C::TC + ((uint32_t)(q * 32) << 16);
        for (int c0 = 0; c0 < min(p.M, BN); c0 += 16) {
          float v[16];
          tmem_ld16(taddr + c0, v);
          if (n < p.N && !*c.fail) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (c0 + j < p.M) Y[(size_t)(c0 + j) * p.N + n] = __float2bfloat16_rn(v[j] * c.rstd[c0 + j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&c.tempty[acc])) : "memory");
      }
    } else if (push_red) {
      consumer_tile_to_owners<BN, SMALL>(p, c, tmem);
    } else {
      tile_to_smem<BN, SMALL>(p, smem, c, tmem, p.M);
    }
  } else if (push_red) {
    cl_wait();  // warps 0 and 1: second half of the start-up barrier
  }
  __syncthreads();
  cg::cluster_group cluster = cg::this_cluster();
  if (cs > 1) {
    cluster.sync();  // release / acquire: partial tiles and row sums complete (pushed, or readable)
    for (int b = threadIdx.x; b < p.M; b += kThreads) {
      float s = 0.f;
      for (int cc = 0; cc < cs; ++cc) s += push_red ? c.red_ss[cc * BN + b] : *cluster.map_shared_rank(c.ss + b, cc);
      c.rstd[b] = rsqrtf(s / (float)p.K + p.eps);
    }
    __syncthreads();
  }
  if (cs > 1 && !*c.fail && p.epi != kEpiPlain) {
    // paired epilogue: this CTA finishes half-rows [r * ph, (r + 1) * ph) of both tile halves
    float* part = reinterpret_cast<float*>(smem);
    const int ph = (BM / 2) / cs, hgroups = ph / 8;
    for (int idx = threadIdx.x; idx < p.M * hgroups; idx += kThreads) {
      const int b = idx / hgroups, f = r * ph + (idx % hgroups) * 8;
      float lo[8], hi[8];
      if (push_red) {
        red_sum8<BN>(c.red, cs, BM / cs, b, f - r * ph, lo);
        red_sum8<BN>(c.red, cs, BM / cs, b, ph + f - r * ph, hi);
      } else {
        cluster_sum8(part, cs, b, f, lo);
        cluster_sum8(part, cs, b, BM / 2 + f, hi);
      }
      const float rs = c.rstd[b];
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // the values a plain epilogue would have stored (bf16)
        lo[j] = __bfloat162float(__float2bfloat16_rn(lo[j] * rs));
        hi[j] = __bfloat162float(__float2bfloat16_rn(hi[j] * rs));
      }
      if (p.epi == kEpiSwiglu) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = lo[j] / (1.f + __expf(-lo[j])) * hi[j];
        __nv_bfloat16* Y = reinterpret_cast<__nv_bfloat16*>(p.Y) + (p.emulate ? (size_t)rank * p.M * (p.N / 2) : 0);
        *reinterpret_cast<uint4*>(Y + (size_t)b * (p.N / 2) + t * (BM / 2) + f) = pack_bf16x8(o);
      } else {  // kEpiRopeKv: tile t is head t
        const int head = t, pos = p.positions[b];
        if (head < p.nq + p.nkv) {
          float o1[8], o2[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float cs_ = p.cos_t[(size_t)pos * (BM / 2) + f + j], sn = p.sin_t[(size_t)pos * (BM / 2) + f + j];
            o1[j] = lo[j] * cs_ - hi[j] * sn;
            o2[j] = hi[j] * cs_ + lo[j] * sn;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            lo[j] = o1[j];
            hi[j] = o2[j];
          }
        }
        __nv_bfloat16* dst;
        if (head < p.nq) {
          dst = reinterpret_cast<__nv_bfloat16*>(p.Y) + (p.emulate ? (size_t)rank * p.M * p.nq * BM : 0) +
                ((size_t)b * p.nq + head) * BM;
        } else {
          const int blk = p.block_tables[(size_t)b * p.max_blocks + pos / p.bs], off = pos % p.bs;
          const int kv = head < p.nq + p.nkv ? head - p.nq : head - p.nq - p.nkv;
          __nv_bfloat16* cache = reinterpret_cast<__nv_bfloat16*>(head < p.nq + p.nkv ? p.k_cache : p.v_cache) +
                                 (p.emulate ? (size_t)rank * p.cache_rs : 0);
          dst = cache + (((size_t)blk * p.nkv + kv) * p.bs + off) * BM;
        }
        *reinterpret_cast<uint4*>(dst + f) = pack_bf16x8(lo);
        *reinterpret_cast<uint4*>(dst + BM / 2 + f) = pack_bf16x8(hi);
      }
    }
  }
  const int per = BM / cs, f0 = r * per, groups = per / 8;
  if (cs > 1 && !*c.fail && p.epi == kEpiPlain) {
    float* part = reinterpret_cast<float*>(smem);
    __nv_bfloat16* Y = reinterpret_cast<__nv_bfloat16*>(p.Y) + (p.emulate ? (size_t)rank * p.M * p.N : 0);
    for (int idx = threadIdx.x; idx < p.M * groups; idx += kThreads) {
      const int b = idx / groups, f = f0 + (idx % groups) * 8;
      const int n = t * BM + f;
      if (n >= p.N) continue;
      float acc[8];
      if (push_red)
        red_sum8<BN>(c.red, cs, per, b, f - f0, acc);
      else
        cluster_sum8(part, cs, b, f, acc);
      const float rs = c.rstd[b];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] *= rs;
      *reinterpret_cast<uint4*>(Y + (size_t)b * p.N + n) = pack_bf16x8(acc);
    }
  }
  // the two-barrier form keeps this CTA's tile and row sums alive until the cluster has read them
  if (cs > 1 && !push_red) cluster.sync();
  // publish the epoch for the next call (same rule as the fused all-reduce kernels)
  const int G = tiles * cs;
  RankState* st = fg_state(p, rank);
  for (int j = lin_block() + threadIdx.x * G; j < kMaxBlocks; j += kThreads * G) st->blk_epoch[j] = e;
  if (lin_block() == 0 && threadIdx.x == 0) st->epoch = e;
  teardown<BN, SMALL>(p, c, tmem, rank);
}

// Clusters of `splits` consumer CTAs that can be resident on this device at once. The occupancy
// calculator places clusters on the GPCs (cudaOccupancyMaxActiveClusters), but for this kernel it
// reports one CTA per SM, while its resources (registers from the compiled function, shared memory,
// threads) admit two SMALL CTAs per SM and launches of 224 mutually waiting CTAs complete on B200; so
// its cluster count is scaled by the per-SM count computed here from the same resources. Cached per
// cluster size; COB_CLUSTER_OCCUPANCY=0 switches the check off. Returns -1 if a query failed.
template <int BN, bool SMALL>
int consumer_cluster_capacity(const void* fn, const cudaLaunchConfig_t& cfg, int splits) {
  static int cap[17] = {};
  static const bool check = [] {
    const char* v = getenv("COB_CLUSTER_OCCUPANCY");
    return v == nullptr || v[0] != '0';
  }();
  if (!check) return 1 << 20;
  if (splits < 1 || splits > 16) return -1;
  if (cap[splits] != 0) return cap[splits];
  using C = FCfg<BN, SMALL>;
  int dev = 0, regs_sm = 0, smem_sm = 0, reserved = 0, threads_sm = 0, calc = 0, clusters = 0;
  cudaFuncAttributes fa;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaFuncGetAttributes(&fa, fn) != cudaSuccess ||
      cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&calc, fn, kThreads, C::SMEM) != cudaSuccess)
    return -1;
  cudaLaunchConfig_t q = cfg;
  q.numAttrs = 1;  // the cluster shape alone
  if (cudaOccupancyMaxActiveClusters(&clusters, fn, &q) != cudaSuccess) return -1;
  const int regs_cta = ((fa.numRegs * 32 + 255) / 256) * 256 * (kThreads / 32);
  int own = std::min({regs_sm / std::max(1, regs_cta),
                      smem_sm / (C::SMEM + (int)fa.sharedSizeBytes + reserved), threads_sm / kThreads,
                      SMALL ? 2 : 1});
  own = std::max(own, calc);
  cap[splits] = calc > 0 ? clusters * own / calc : 0;
  return cap[splits];
}

template <int BN, bool SMALL, bool PUSH>
cudaError_t launch_t(const FusedGemmParams& p, const CUtensorMap& tw, const CUtensorMap& tb, const FusedGemmPlan& pl,
                     int ranks, bool pdl, cudaStream_t stream) {
  using C = FCfg<BN, SMALL>;
  auto fn = PUSH ? k_gemm_push<BN, SMALL> : k_ar_norm_gemm<BN, SMALL>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    // clusters of 16 CTAs (split-K 16 for narrow outputs such as QKV at TP=8) are non-portable
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    // the whole shared-memory carve-out, so that two SMALL CTAs fit on an SM (and the occupancy
    // calculator, which follows this preference, says so)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.xctas, pl.splits, ranks);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeClusterDimension;
  attrs[na].val.clusterDim.x = 1;
  attrs[na].val.clusterDim.y = pl.splits;
  attrs[na].val.clusterDim.z = 1;
  ++na;
  if (pdl || pdl_flag()) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  if (!PUSH) {
    // CTAs of the consumer wait for pieces that other CTAs of the same launch produce, so every cluster
    // of the grid must be resident at once: reject grids larger than that (the caller falls back).
    const int mc = consumer_cluster_capacity<BN, SMALL>(reinterpret_cast<const void*>(fn), cfg, pl.splits);
    if (mc < 0) return cudaErrorUnknown;
    if ((long long)mc < (long long)pl.xctas * ranks) return cudaErrorInvalidValue;
  }
  FusedGemmParams q = p;
  q.kps = pl.kps;
  if (q.l2_prefetch == 0) q.l2_prefetch = l2_prefetch_tiles();
  return cudaLaunchKernelEx(&cfg, fn, tw, tb, q);
}

template <bool PUSH>
cudaError_t launch_sel(const FusedGemmParams& p, const CUtensorMap& tw, const CUtensorMap& tb, const FusedGemmPlan& pl,
                       int ranks, bool pdl, cudaStream_t s) {
  switch (pl.bn) {
    case 16: return launch_t<16, true, PUSH>(p, tw, tb, pl, ranks, pdl, s);
    case 32: return launch_t<32, true, PUSH>(p, tw, tb, pl, ranks, pdl, s);
    case 64: return launch_t<64, true, PUSH>(p, tw, tb, pl, ranks, pdl, s);
    case 128: return launch_t<128, false, PUSH>(p, tw, tb, pl, ranks, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

int smem_of(int bn) {
  switch (bn) {
    case 16: return FCfg<16, true>::SMEM;
    case 32: return FCfg<32, true>::SMEM;
    case 64: return FCfg<64, true>::SMEM;
    case 128: return FCfg<128, false>::SMEM;
    default: return 0;
  }
}

cudaError_t check_common(const FusedGemmParams& p, const FusedGemmPlan& pl, int ranks) {
  if (p.M <= 0 || p.M > 128 || p.N % 8 || p.K % BK || p.N <= 0 || p.K <= 0) return cudaErrorInvalidValue;
  if (p.world < 1 || p.world > kMaxWorld || ranks < 1 || (p.emulate ? ranks != p.world : ranks != 1))
    return cudaErrorInvalidValue;
  if (pl.splits < 1 || pl.splits > 16 || BM % (8 * pl.splits) || pl.tiles != (p.N + BM - 1) / BM)
    return cudaErrorInvalidValue;
  // several tiles per CTA only without split-K (the cluster epilogue holds one tile)
  if (pl.xctas < 1 || pl.xctas > pl.tiles || (pl.splits > 1 && pl.xctas != pl.tiles)) return cudaErrorInvalidValue;
  if (p.epi != kEpiPlain) {
    if (pl.splits < 2 || pl.splits > 8 || p.N % BM) return cudaErrorInvalidValue;
    if (p.epi == kEpiRopeKv && (p.N != (p.nq + 2 * p.nkv) * BM || p.bs <= 0 || !p.positions || !p.cos_t ||
                                !p.sin_t || !p.block_tables || !p.k_cache || !p.v_cache))
      return cudaErrorInvalidValue;
  }
  if ((long long)pl.kps * (pl.splits - 1) >= p.K / BK) return cudaErrorInvalidValue;  // every split non-empty
  // packed weights: whole 16 KB blocks, one block row per 128-row tile of each rank
  if (p.wp != nullptr && ((reinterpret_cast<uintptr_t>(p.wp) & 15) || p.w_tiles != (p.N + BM - 1) / BM))
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

}  // namespace

FusedGemmPlan plan_fused_gemm(int M, int N, int K, int splits, int num_sms, bool consumer, int epi) {
  FusedGemmPlan pl = {};
  pl.bn = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
  pl.tiles = (N + BM - 1) / BM;
  const int KT = K / BK;
  const int per_sm = pl.bn <= 64 ? 2 : 1;
  // ar_norm_gemm: the whole grid resident at once and one epoch word per CTA
  const int cap = std::min(num_sms * per_sm, kMaxBlocks);
  if (splits <= 0) {
    // enough CTAs to keep every SM streaming weights, within one resident wave
    splits = 1;
    // (up to 16: a non-portable cluster size, co-scheduled as 8 SMs x 2 CTAs)
    const int smax = epi != kEpiPlain ? 8 : (per_sm == 2 ? 16 : 8);
    const int lim = consumer ? cap : num_sms * per_sm;
    while (splits < smax && pl.tiles * splits * 2 <= lim && KT / (splits * 2) >= 2) splits *= 2;
  }
  pl.kps = (KT + splits - 1) / splits;
  pl.splits = (KT + pl.kps - 1) / pl.kps;
  while (BM % (8 * pl.splits)) --pl.splits;
  pl.kps = (KT + pl.splits - 1) / pl.splits;
  pl.xctas = pl.tiles;
  if (epi != kEpiPlain) {
    // paired epilogues finish whole tiles inside a cluster of 2..8 splits, one tile per CTA
    if (pl.splits < 2 && KT >= 2 && pl.tiles * 2 <= cap) {
      pl.splits = 2;
      pl.kps = (KT + 1) / 2;
      pl.splits = (KT + pl.kps - 1) / pl.kps;
    }
    if (pl.splits < 2 || pl.splits > 8 || pl.tiles * pl.splits > cap) pl.splits = 0;  // unsupported
  }
  if (consumer && pl.splits > 0 && pl.tiles * pl.splits > cap) {
    // too many tiles for one resident wave: no split-K, each CTA loops over several tiles
    pl.splits = 1;
    pl.kps = KT;
    pl.xctas = std::min(pl.tiles, cap);
  }
  pl.smem = smem_of(pl.bn);
  pl.ctas = pl.xctas * pl.splits;
  return pl;
}

cudaError_t launch_gemm_push(const FusedGemmParams& p, const CUtensorMap& tmW, const CUtensorMap& tmX,
                             const FusedGemmPlan& pl, int ranks, bool pdl, cudaStream_t stream) {
  cudaError_t e = check_common(p, pl, ranks);
  if (e != cudaSuccess) return e;
  if (pl.xctas != pl.tiles || p.epi != kEpiPlain) return cudaErrorInvalidValue;
  if (p.M > p.L.max_rows || p.N / 8 > p.L.max_hv || p.L.world != p.world) return cudaErrorInvalidValue;
  return launch_sel<true>(p, tmW, tmX, pl, ranks, pdl, stream);
}

cudaError_t launch_ar_norm_gemm(const FusedGemmParams& p, const CUtensorMap& tmW, const CUtensorMap& tmA,
                                const FusedGemmPlan& pl, int ranks, bool pdl, cudaStream_t stream) {
  cudaError_t e = check_common(p, pl, ranks);
  if (e != cudaSuccess) return e;
  if (p.M > p.L.max_rows || p.K / 8 > p.L.max_hv || p.L.world != p.world || p.M > p.act_rows) return cudaErrorInvalidValue;
  // pieces per launch, and per-block epoch words written by every block (no two blocks share one)
  if (pl.ctas > kMaxPieces || pl.ctas > kMaxBlocks) return cudaErrorInvalidValue;
  // every piece's per-item sums of squares fit in shared memory
  const int KV = p.K / 8, slen = std::min(KV, pl.kps * 8);
  if ((long long)p.M * ((slen + pl.xctas - 1) / pl.xctas + 1) > kQCap) return cudaErrorInvalidValue;
  // CTAs wait for pieces of other CTAs of the launch: the whole grid must be resident at once (a quick
  // bound here; launch_t asks the occupancy calculator for the exact cluster configuration)
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if ((long long)pl.ctas * ranks > (long long)sms * (pl.bn <= 64 ? 2 : 1)) return cudaErrorInvalidValue;
  return launch_sel<false>(p, tmW, tmA, pl, ranks, pdl, stream);
}

namespace {
template <int BN, bool SMALL>
int consumer_clusters(int splits) {
  using C = FCfg<BN, SMALL>;
  auto fn = k_ar_norm_gemm<BN, SMALL>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess ||
      cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
      cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
          cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, splits > 0 ? splits : 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeClusterDimension;
  a.val.clusterDim.x = 1;
  a.val.clusterDim.y = splits > 0 ? splits : 1;
  a.val.clusterDim.z = 1;
  cfg.attrs = &a;
  cfg.numAttrs = 1;
  int n = 0;
  if (splits == 0) {  // CTAs per SM by the occupancy calculator (diagnostic)
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, C::SMEM) == cudaSuccess ? n : -1;
  }
  return consumer_cluster_capacity<BN, SMALL>(reinterpret_cast<const void*>(fn), cfg, splits);
}
}  // namespace

int ar_norm_gemm_resident_clusters(int bn, int splits) {
  if (splits < 0 || splits > 16) return -1;
  switch (bn) {
    case 16: return consumer_clusters<16, true>(splits);
    case 32: return consumer_clusters<32, true>(splits);
    case 64: return consumer_clusters<64, true>(splits);
    case 128: return consumer_clusters<128, false>(splits);
    default: return -1;
  }
}

}  // namespace cob
