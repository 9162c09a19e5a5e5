// Fused tensor-parallel all-reduce + residual add + RMSNorm over NVLink 5 / NVSwitch peer memory.
//
//   out, residual <- RMSNorm(residual + sum_r x_r) * gamma, residual + sum_r x_r
//
// One kernel per call, no host barrier, safe under CUDA-graph replay. Capability parity with the
// A100 prototype of the reference (exp/M17_epoch_ab/fused_ar_norm_nf.cu:90-199: start barrier ->
// pull reduce-scatter -> residual + RMSNorm -> LL128 push all-gather -> poll -> last block advances
// the epoch), re-designed for Blackwell:
//   * world 2/4/8 (the reference hard-codes 8, fused_ar_norm_nf.cu:28),
//   * every rank ends with the FULL new residual (the reference keeps it sharded by rows,
//     fused_ar_norm_nf.cu:13), because the all-gather carries h = residual + sum(x) and every rank
//     normalises locally; the two-shot variants shard columns, not rows, so T < world still uses
//     every rank, and the per-row sum of squares travels with the data,
//   * arrival detection without 128-byte line atomicity (the reference's unproven assumption A,
//     docs/method_design.md:35): Lamport negative-zero sentinels (per-element atomicity only) for
//     bulk data and {value, epoch} 8-byte words for partials,
//   * NVSwitch multicast (multimem.ld_reduce / multimem.st / multimem.red barriers), which the
//     A100 NV12 system of the reference did not have,
//   * thread-block clusters with DSMEM so a single row can be spread over up to 8 SMs,
//   * every wait bounded by %globaltimer; a timeout sets the rank's error word and the kernel
//     returns (the reference's spins are unbounded, fused_ar_norm_nf.cu:95-96, 181-183),
//   * one epoch for all blocks of a call whatever the grid size, so graphs of different grid sizes
//     interleave (the property of the reference's M16 fix, exp/M16_epoch_fix/fused_ar_norm.cu:190-198),
//     without its last-block arrival counter: each block publishes the epoch for its index class.
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"
#include "fused_ar.h"

namespace cob {
namespace {

namespace cg = cooperative_groups;

constexpr int kVPT = 4;  // max 16-byte vectors per thread per row chunk

__host__ __device__ __forceinline__ long long align_up(long long v, long long a) { return (v + a - 1) / a * a; }

__device__ __forceinline__ RankState* state_of(const ARParams& p, int r) {
  return reinterpret_cast<RankState*>(p.base[r] + p.L.state);
}
// index ranges of the heap regions (checked builds record a violation instead of accessing)
__device__ __forceinline__ bool heap_ok(const ARParams& p, int owner, int slot, int src, int row, int v, int vmax) {
  return (unsigned)owner < (unsigned)p.L.world && (unsigned)slot < 2u && (unsigned)src < (unsigned)p.L.world &&
         (unsigned)row < (unsigned)p.L.max_rows && (unsigned)v < (unsigned)vmax;
}
__device__ __forceinline__ unsigned int* err_word_of(const ARParams& p) {
  return &reinterpret_cast<RankState*>(p.base[p.emulate ? blockIdx.y : p.rank] + p.L.state)->error;
}
__device__ __forceinline__ uint4* land1_at(const ARParams& p, int owner, int slot, int src, int row, int v) {
  return COB_IN_RANGE(reinterpret_cast<uint4*>(p.base[owner] + p.L.land1) +
                          ((((size_t)slot * p.L.world + src) * p.L.max_rows + row) * p.L.max_hv + v),
                      heap_ok(p, owner, slot, src, row, v, p.L.max_hv), err_word_of(p));
}
__device__ __forceinline__ uint4* rs_at(const ARParams& p, int owner, int slot, int src, int row, int i) {
  return COB_IN_RANGE(reinterpret_cast<uint4*>(p.base[owner] + p.L.rs) +
                          ((((size_t)slot * p.L.world + src) * p.L.max_rows + row) * p.L.sv_max + i),
                      heap_ok(p, owner, slot, src, row, i, p.L.sv_max), err_word_of(p));
}
__device__ __forceinline__ uint4* ag_at(const ARParams& p, int owner, int slot, int src, int row, int i) {
  return COB_IN_RANGE(reinterpret_cast<uint4*>(p.base[owner] + p.L.ag) +
                          ((((size_t)slot * p.L.world + src) * p.L.max_rows + row) * p.L.sv_max + i),
                      heap_ok(p, owner, slot, src, row, i, p.L.sv_max), err_word_of(p));
}
// Partial sums of squares travel per "unit" of an owner slice (32 vectors, one per lane): units per
// slice ceil(sv / 32), at most pu_max(L) words per (source rank, row).
__host__ __device__ __forceinline__ int pu_max(const Layout& L) { return (L.sv_max + 31) / 32; }
__device__ __forceinline__ unsigned long long* agp_at(const ARParams& p, int owner, int slot, int src, int row, int u) {
  return reinterpret_cast<unsigned long long*>(p.base[owner] + p.L.agp) +
         ((((size_t)slot * p.L.world + src) * p.L.max_rows + row) * pu_max(p.L) + u);
}
__device__ __forceinline__ size_t hpart_idx(const ARParams& p, int row, int src, int u) {
  return ((size_t)row * p.L.world + src) * pu_max(p.L) + u;
}
__device__ __forceinline__ size_t stage_idx(const ARParams& p, int parity, int row, int v) {
  return ((size_t)parity * p.L.max_rows + row) * p.L.max_hv + v;
}
__device__ __forceinline__ uint4* stage_at(const ARParams& p, int owner, int parity, int row, int v) {
  return COB_IN_RANGE(reinterpret_cast<uint4*>(p.base[owner] + p.L.stage) + stage_idx(p, parity, row, v),
                      heap_ok(p, owner, parity, 0, row, v, p.L.max_hv), err_word_of(p));
}

__device__ void record_error(RankState* st, uint32_t bit, uint64_t variant_phase, uint64_t where,
                             uint64_t peer, uint64_t epoch) {
  if (atomicOr(&st->error, bit) == 0u) {
    st->err_detail[0] = variant_phase;
    st->err_detail[1] = where;
    st->err_detail[2] = peer;
    st->err_detail[3] = epoch;
  }
}

// Phase stamp of this block (thread 0) when stamping is enabled.
__device__ __forceinline__ void stamp(const ARParams& p, int rank, uint64_t e, int phase) {
  if (p.stamps != nullptr && threadIdx.x == 0) {
    const size_t i = (((size_t)rank * p.stamp_cap + (size_t)(e % (uint64_t)p.stamp_cap)) * kMaxBlocks + blockIdx.x) *
                         kStampPhases + phase;
    p.stamps[i] = (long long)globaltimer();
  }
}

// End of a call: publish the epoch to the blocks of the next call (see RankState::blk_epoch). No
// block waits for another, so there is no arrival counter on the critical path; the next call reads
// these words after griddepcontrol.wait, which returns once this grid has completed and its writes
// are visible. Every block of every call reads the same epoch, whatever the grid sizes (the rule
// of the reference's fix for graphs of mixed grid sizes, exp/M16_epoch_fix/fused_ar_norm.cu:190-198).
__device__ __forceinline__ uint64_t call_epoch(RankState* st) {
  return ld_vol_u64(&st->blk_epoch[blockIdx.x]) + 1;
}

__device__ __forceinline__ void finish_call(RankState* st, uint64_t e) {
  for (int j = blockIdx.x + threadIdx.x * gridDim.x; j < kMaxBlocks; j += blockDim.x * gridDim.x)
    st->blk_epoch[j] = e;
  if (blockIdx.x == 0 && threadIdx.x == 0) st->epoch = e;
}

// Cluster-wide (or block-wide when C == 1) sum with a fixed order. `it` alternates the shared
// slot so one cluster barrier per row is enough.
__device__ __forceinline__ float row_sum(float v, float* scratch, float* s_part, int it, int C) {
  float part = block_sum(v, scratch);
  if (C == 1) return part;
  cg::cluster_group cluster = cg::this_cluster();
  if (threadIdx.x == 0) s_part[it & 1] = part;
  cluster.sync();
  float tot = 0.f;
  for (int c = 0; c < C; ++c) tot += *cluster.map_shared_rank(&s_part[it & 1], c);
  return tot;
}

// Cluster-wide sum with no release-ordered barrier (variant kLamport1SX). Each CTA publishes its
// block sum as one {f32, tag} word in its own shared memory (slot it % 2, tag it + 1); lane c of warp 0
// polls CTA c's word with relaxed cluster-scope loads, and the C values are added in CTA order from
// zero, the same order as row_sum(), so every CTA of the cluster (and every rank) gets bitwise the
// same total. Nothing here orders the CTA's earlier NVLink pushes or landing restores, so the row
// sum never waits for them to be acknowledged (a release-ordered cluster barrier does).
// Slot reuse: a CTA writes row it + 2 into slot it % 2 only after it has read every CTA's row it + 1
// word, which each CTA publishes only after it has consumed all row-it words; two slots suffice. The
// words are zeroed (tag 0 = none) before a cluster barrier that every CTA passes before its first
// poll, so stale shared memory is never accepted. A CTA stops reading its peers' shared memory
// before it arrives at the final cluster barrier, which its peers pass before they exit.
__device__ __forceinline__ float row_sum_xch(float v, float* scratch, unsigned long long* s_word, float* s_tot, int it,
                                             int C, int crank, Waiter& w, RankState* st, uint64_t e, int row) {
  const float part = block_sum(v, scratch);
  if (C == 1) return part;
  const uint32_t tag = (uint32_t)it + 1u;
  if (threadIdx.x == 0) st_cluster_word(&s_word[it & 1], ((unsigned long long)tag << 32) | __float_as_uint(part));
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float pc = part;
    if (lane < C && lane != crank) {
      const uint32_t a = cluster_map(&s_word[it & 1], lane);
      unsigned long long wd = ld_cluster_word(a);
      while ((uint32_t)(wd >> 32) != tag) {
        if (w.expired()) {
          // phase 4: the row partial of cluster CTA `lane` did not arrive
          record_error(st, kErrTimeoutPartial, ((uint64_t)kLamport1SX << 32) | 4, (uint64_t)row << 32, lane, e);
          wd = 0ull;
          break;
        }
        wd = ld_cluster_word(a);
      }
      pc = __uint_as_float((uint32_t)wd);
    }
    float tot = 0.f;
    for (int c = 0; c < C; ++c) tot += __shfl_sync(0xffffffffu, pc, c);
    if (lane == 0) *s_tot = tot;
  }
  __syncthreads();
  return *s_tot;
}

template <typename T>
__device__ __forceinline__ void store_norm(const ARParams& p, T* out, T* res, int row, int v, const float* h,
                                           const uint4& hbits, float rstd, const uint4* gamma_v = nullptr) {
  using V = Vec<T>;
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * p.hidden);
  if (p.norm) {
    float g[V::N], o[V::N];
    V::to_float(gamma_v ? *gamma_v : ld_nc_v4(reinterpret_cast<const uint4*>(p.gamma) + v), g);
#pragma unroll
    for (int i = 0; i < V::N; ++i) o[i] = h[i] * rstd * g[i];
    orow[v] = V::from_float(o);
    reinterpret_cast<uint4*>(res + (size_t)row * p.hidden)[v] = hbits;
  } else {
    orow[v] = hbits;
  }
}

// Poll a Lamport vector until every element has arrived. Returns false on timeout.
template <typename T>
__device__ __forceinline__ bool poll_vec(const uint4* addr, uint4& d, Waiter& w) {
  while (!LamportOf<T>::ready(d)) {
    if (w.expired()) return false;
    d = ld_vol_v4(addr);
  }
  return true;
}

// Flag barrier between block b of every rank: each block posts its per-block call count into every
// peer's slot and waits until all peers' counts reach it. A peer can be at most one call ahead, so
// the comparison is ">=".
__device__ __forceinline__ bool flag_barrier(const ARParams& p, int rank, RankState* st, uint32_t bc, Waiter& w) {
  bool ok = true;
  if (threadIdx.x < (unsigned)p.L.world) {
    const int peer = threadIdx.x;
    unsigned long long* dst =
        reinterpret_cast<unsigned long long*>(p.base[peer] + p.L.flags) + (size_t)blockIdx.x * kMaxWorld + rank;
    st_release_u64(dst, bc);
    const unsigned long long* mine =
        reinterpret_cast<unsigned long long*>(p.base[rank] + p.L.flags) + (size_t)blockIdx.x * kMaxWorld + peer;
    while ((long long)(ld_acquire_u64(mine) - (unsigned long long)bc) < 0) {
      if (w.expired()) {
        record_error(st, kErrTimeoutFlag, ((uint64_t)p.variant << 32) | 0, blockIdx.x, peer, bc);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

// NVLS barrier k of block b: one multicast add per rank, wait for world * calls on the local copy.
__device__ __forceinline__ bool nvls_barrier(const ARParams& p, int rank, RankState* st, int k, uint32_t calls,
                                             Waiter& w) {
  bool ok = true;
  if (threadIdx.x == 0) {
    const size_t off = p.L.nvls + ((size_t)blockIdx.x * 2 + k) * sizeof(unsigned int);
    mm_red_add_u32(p.mc + off, 1u);
    const uint32_t target = calls * (uint32_t)p.L.world;
    while ((int)(ld_acquire_u32(p.base[rank] + off) - target) < 0) {
      if (w.expired()) {
        record_error(st, kErrTimeoutNvls, ((uint64_t)p.variant << 32) | (uint64_t)k, blockIdx.x, 0, calls);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

// ---------------------------------------------------------------------------------------------
// One-shot kernels: cluster of C CTAs per row, chunk of the row per CTA.
//   LAMPORT: push x to all peers' land1[slot][rank] -> poll own land1[slot][*] -> sum
//   PULL   : copy x to stage[parity] -> flag barrier -> read every peer's stage -> sum
//   NVLS   : copy x to stage[parity] -> multicast barrier -> multimem.ld_reduce -> sum
// ---------------------------------------------------------------------------------------------
// VPT: 16-byte vectors per thread per row chunk (1 when the chunk fits the block, else kVPT), so the
// common geometries (a row spread over a cluster, one vector per thread) hold one vector's state in
// registers instead of four.
// XCH (variant kLamport1SX, MODE == kLamport1S): the row sum crosses the cluster through
// row_sum_xch(), the landing cells get their sentinel back after the row's outputs are stored, and the
// final cluster barrier is relaxed; the arithmetic and the result are those of kLamport1S.
template <typename T, int W, int MODE, int VPT, bool XCH>
__global__ void __launch_bounds__(512) k_oneshot(const ARParams p) {
  using V = Vec<T>;
  using LP = LamportOf<T>;
  const int rank = p.emulate ? (int)blockIdx.y : p.rank;
  const int tid = threadIdx.x, NT = blockDim.x;
  RankState* st = state_of(p, rank);
  const T* x = reinterpret_cast<const T*>(p.x) + (size_t)rank * p.x_rs;
  T* res = reinterpret_cast<T*>(p.residual) + (size_t)rank * p.res_rs;
  T* out = reinterpret_cast<T*>(p.out) + (size_t)rank * p.out_rs;
  const int hv = p.hidden / V::N;
  const int C = p.cluster;
  const int crank = blockIdx.x % C, cl = blockIdx.x / C, ncl = gridDim.x / C;
  const int chunk = (hv + C - 1) / C;
  const int v0 = crank * chunk, v1 = min(hv, v0 + chunk);
  __shared__ float s_scr[32];
  __shared__ float s_part[2];
  __shared__ unsigned long long s_word[2];  // XCH: this CTA's {row partial, tag} by row parity
  __shared__ float s_tot;
  const bool xcl = XCH && C > 1;
  if (xcl) {
    if (tid < 2) s_word[tid] = 0ull;
    cluster_arrive_release();  // nothing of this kernel is in flight yet; waited for before the first poll
  }

  pdl_wait();
  const uint64_t e = call_epoch(st);
  const int slot = (int)(e & 1);
  Waiter w(p.timeout_ns, &st->error);
  bool ok = true;
  stamp(p, rank, e, 0);

  if (MODE == kLamport1S) {
    for (int row = cl; row < p.rows; row += ncl) {
      const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * p.hidden);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = v0 + tid + k * NT;
        if (v < v1) {
          const uint4 d = LP::clean(ld_nc_v4(xr + v));
#pragma unroll
          for (int i = 1; i < W; ++i) st_vol_v4(land1_at(p, (rank + i) % W, slot, rank, row, v), d);
        }
      }
    }
  } else {
    for (int row = cl; row < p.rows; row += ncl) {
      const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * p.hidden);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = v0 + tid + k * NT;
        if (v < v1) *stage_at(p, rank, slot, row, v) = ld_nc_v4(xr + v);
      }
    }
    __threadfence();
    __syncthreads();
    if (MODE == kPull1S) {
      const uint32_t bc = st->flag_calls[blockIdx.x] + 1u;
      ok = flag_barrier(p, rank, st, bc, w);
      if (tid == 0) st->flag_calls[blockIdx.x] = bc;
    } else {
      const uint32_t nc = st->nvls_calls[blockIdx.x][0] + 1u;
      ok = nvls_barrier(p, rank, st, 0, nc, w);
      if (tid == 0) st->nvls_calls[blockIdx.x][0] = nc;
    }
    stamp(p, rank, e, 2);
  }
  stamp(p, rank, e, 1);
  pdl_trigger();
  if (xcl) cluster_wait();

  int it = 0;
  bool arrived = false;
  for (int row = cl; row < p.rows; row += ncl, ++it) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * p.hidden);
    float h[VPT][V::N];
    uint4 hb[VPT], rv[VPT], gv[VPT];
    float ss = 0.f;
    // residual and gamma do not depend on the peers: request them before waiting for peer data
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = v0 + tid + k * NT;
      if (v < v1 && p.norm) {
        rv[k] = reinterpret_cast<const uint4*>(res + (size_t)row * p.hidden)[v];
        gv[k] = ld_nc_v4(reinterpret_cast<const uint4*>(p.gamma) + v);
      }
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = v0 + tid + k * NT;
      if (v < v1) {
        float a[V::N];
#pragma unroll
        for (int i = 0; i < V::N; ++i) a[i] = 0.f;
        if (MODE == kNvls1S) {
          const uint4 s = ok ? mm_ld_reduce<T>(p.mc + p.L.stage + stage_idx(p, slot, row, v) * 16) : make_uint4(0, 0, 0, 0);
          V::to_float(s, a);
        } else {
          uint4 d[W];
#pragma unroll
          for (int s = 0; s < W; ++s) {
            if (MODE == kLamport1S)
              d[s] = (s == rank) ? ld_nc_v4(xr + v) : ld_vol_v4(land1_at(p, rank, slot, s, row, v));
            else
              d[s] = ok ? ld_vol_v4(stage_at(p, s, slot, row, v)) : make_uint4(0, 0, 0, 0);
          }
          if (MODE == kLamport1S) {
#pragma unroll
            for (int s = 0; s < W; ++s) {
              if (s != rank && ok && !poll_vec<T>(land1_at(p, rank, slot, s, row, v), d[s], w)) {
                record_error(st, kErrTimeoutLanding, ((uint64_t)MODE << 32) | 2, ((uint64_t)row << 32) | v, s, e);
                ok = false;
              }
            }
            if (!XCH) {
#pragma unroll
              for (int s = 0; s < W; ++s)
                if (s != rank) st_vol_v4(land1_at(p, rank, slot, s, row, v), LP::fill());
            }
          }
#pragma unroll
          for (int s = 0; s < W; ++s) {
            float f[V::N];
            V::to_float(d[s], f);
#pragma unroll
            for (int i = 0; i < V::N; ++i) a[i] += f[i];
          }
        }
        if (p.norm) {
          float r[V::N];
          V::to_float(rv[k], r);
#pragma unroll
          for (int i = 0; i < V::N; ++i) a[i] += r[i];
        }
        hb[k] = V::from_float(a);  // h is stored in the element type; the norm uses the stored values
        V::to_float(hb[k], h[k]);
#pragma unroll
        for (int i = 0; i < V::N; ++i) ss += h[k][i] * h[k][i];
      }
    }
    float rstd = 0.f;
    if (p.norm) {
      const float tot = XCH ? row_sum_xch(ss, s_scr, s_word, &s_tot, it, C, crank, w, st, e, row)
                            : row_sum(ss, s_scr, s_part, it, C);
      rstd = rsqrtf(tot / (float)p.hidden + p.eps);
    }
    if (xcl && row + ncl >= p.rows) {  // last row: this CTA reads no more peer shared memory
      cluster_arrive_relaxed();
      arrived = true;
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = v0 + tid + k * NT;
      if (v < v1) {
        uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * p.hidden);
        if (p.norm) {
          float g[V::N], o[V::N];
          V::to_float(gv[k], g);
#pragma unroll
          for (int i = 0; i < V::N; ++i) o[i] = h[k][i] * rstd * g[i];
          orow[v] = V::from_float(o);
          reinterpret_cast<uint4*>(res + (size_t)row * p.hidden)[v] = hb[k];
        } else {
          orow[v] = hb[k];
        }
      }
    }
    if (XCH && MODE == kLamport1S) {  // the row's landing cells get their sentinel back
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int v = v0 + tid + k * NT;
        if (v < v1) {
#pragma unroll
          for (int s = 0; s < W; ++s)
            if (s != rank) st_vol_v4(land1_at(p, rank, slot, s, row, v), LP::fill());
        }
      }
    }
  }
  stamp(p, rank, e, 3);
  if (xcl) {
    if (!arrived) cluster_arrive_relaxed();
    cluster_wait();  // no CTA leaves while a peer CTA may still read its shared memory
  } else if (C > 1) {
    cg::this_cluster().sync();  // no CTA leaves while a peer CTA may read its shared memory
  }
  stamp(p, rank, e, 4);
  finish_call(st, e);
}

// ---------------------------------------------------------------------------------------------
// Two-shot kernels. Rank r owns columns [r*SV, (r+1)*SV) of every row (SV = HV / W vectors). The owned
// slice of a row is cut into units of 32 vectors (one per lane, ceil(SV / 32) units per slice), so
// even one row keeps several warps busy; each unit's sum of squares travels as its own
// {f32, epoch32} word and a row's W x units words are summed by one warp in phase 3.
//   phase 1 (LAMPORT): push slice d of x to rank d's rs[slot][rank]            (flat, 4 vectors / step)
//   phase 1 (PULL)   : copy this block's rows of x to stage[parity], flag barrier
//   phase 1 (NVLS)   : copy this block's rows of x to stage[parity], multicast barrier
//   phase 2 (owner)  : a warp per unit: sum over ranks (+ residual) -> h, unit sum of squares (warp
//                      reduction); LAMPORT/PULL push h + {partial, epoch} to every rank's ag/agp,
//                      NVLS multimem.st h + partial to every rank's hbuf/hpart, then barrier 2.
//                      LAMPORT spreads units over all warps of the grid; PULL / NVLS keep a row in
//                      the block that staged it (their barriers are per block).
//   phase 3          : all slices of h + all partials -> out, residual (flat for LAMPORT/PULL, the
//                      block's rows for NVLS)
// ---------------------------------------------------------------------------------------------

// Sum of the W x U unit partials of a row (epoch-tagged words), warp-wide; false on timeout.
template <int W>
__device__ __forceinline__ bool row_partials(const ARParams& p, int rank, int slot, int row, int U, uint32_t etag,
                                             bool nvls, Waiter& w, RankState* st, uint64_t e, float& tot) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  bool ok = true;
  for (int j = lane; j < W * U; j += 32) {
    const int src = j / U, u = j - src * U;
    const unsigned long long* a =
        nvls ? reinterpret_cast<const unsigned long long*>(p.base[rank] + p.L.hpart) + hpart_idx(p, row, src, u)
             : agp_at(p, rank, slot, src, row, u);
    unsigned long long wd = ld_vol_u64(a);
    while ((uint32_t)(wd >> 32) != etag) {
      if (w.expired()) {
        record_error(st, kErrTimeoutPartial, 3, row, j, e);
        ok = false;
        break;
      }
      wd = ld_vol_u64(a);
    }
    acc += __uint_as_float((uint32_t)wd);
  }
  tot = warp_sum(acc);
  return __all_sync(0xffffffffu, ok);
}

template <typename T, int W, int MODE>
__global__ void __launch_bounds__(256) k_twoshot(const ARParams p) {
  using V = Vec<T>;
  using LP = LamportOf<T>;
  constexpr int kChunk = 1;       // vectors per lane per unit
  constexpr int UV = 32 * kChunk;  // vectors per unit
  const int rank = p.emulate ? (int)blockIdx.y : p.rank;
  const int tid = threadIdx.x, NT = blockDim.x, lane = tid & 31, warp = tid >> 5, NW = NT >> 5;
  RankState* st = state_of(p, rank);
  const T* x = reinterpret_cast<const T*>(p.x) + (size_t)rank * p.x_rs;
  T* res = reinterpret_cast<T*>(p.residual) + (size_t)rank * p.res_rs;
  T* out = reinterpret_cast<T*>(p.out) + (size_t)rank * p.out_rs;
  const int hv = p.hidden / V::N, sv = hv / W, U = (sv + UV - 1) / UV;
  const long long total = (long long)p.rows * hv;
  const long long gtid = (long long)blockIdx.x * NT + tid, gthreads = (long long)gridDim.x * NT;
  const int gw = blockIdx.x * NW + warp, total_warps = gridDim.x * NW;

  pdl_wait();
  const uint64_t e = call_epoch(st);
  const int slot = (int)(e & 1);
  const uint32_t etag = (uint32_t)e;
  Waiter w(p.timeout_ns, &st->error);
  bool ok = true;
  stamp(p, rank, e, 0);

  // ---- phase 1
  if (MODE == kLamport2S) {
    for (long long u0 = gtid; u0 < total; u0 += 4 * gthreads) {
      uint4 d[4];
      int rows_[4], vs[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const long long u = u0 + k * gthreads;
        rows_[k] = -1;
        if (u < total) {
          rows_[k] = (int)(u / hv);
          vs[k] = (int)(u - (long long)rows_[k] * hv);
          d[k] = ld_nc_v4(reinterpret_cast<const uint4*>(x + (size_t)rows_[k] * p.hidden) + vs[k]);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (rows_[k] < 0) continue;
        const int dst = vs[k] / sv, i = vs[k] - dst * sv;
        if (dst != rank) st_vol_v4(rs_at(p, dst, slot, rank, rows_[k], i), LP::clean(d[k]));
      }
    }
  } else {
    for (int row = blockIdx.x; row < p.rows; row += gridDim.x) {
      const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * p.hidden);
      for (int v = tid; v < hv; v += NT) *stage_at(p, rank, slot, row, v) = ld_nc_v4(xr + v);
    }
    __threadfence();
    __syncthreads();
    if (MODE == kPull2S) {
      const uint32_t bc = st->flag_calls[blockIdx.x] + 1u;
      ok = flag_barrier(p, rank, st, bc, w);
      if (tid == 0) st->flag_calls[blockIdx.x] = bc;
    } else {
      const uint32_t nc = st->nvls_calls[blockIdx.x][0] + 1u;
      ok = nvls_barrier(p, rank, st, 0, nc, w);
      if (tid == 0) st->nvls_calls[blockIdx.x][0] = nc;
    }
  }
  stamp(p, rank, e, 1);
  pdl_trigger();

  // ---- phase 2: a warp per (row, unit of the owned slice)
  // LAMPORT: units over all warps of the grid; PULL / NVLS: the block's rows, units over its warps
  const int nunits = MODE == kLamport2S ? p.rows * U : ((p.rows - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * U;
  for (int g = (MODE == kLamport2S ? gw : warp); MODE != kNvls2S && g < nunits;
       g += (MODE == kLamport2S ? total_warps : NW)) {
    const int row = MODE == kLamport2S ? g / U : (int)blockIdx.x + (g / U) * (int)gridDim.x;
    const int c0 = (g % U) * UV;
    float ss = 0.f;
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * p.hidden);
    const uint4* rr = reinterpret_cast<const uint4*>(res + (size_t)row * p.hidden);
    uint4 rv[kChunk];
    float a[kChunk][V::N];
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
      const int i = c0 + k * 32 + lane;
#pragma unroll
      for (int q = 0; q < V::N; ++q) a[k][q] = 0.f;
      if (i < sv && p.norm) rv[k] = rr[rank * sv + i];  // issued before the peer data is awaited
    }
    {
      // every source's vector of every chunk element is requested before any is awaited
      uint4 d[kChunk][W];
#pragma unroll
      for (int k = 0; k < kChunk; ++k) {
        const int i = c0 + k * 32 + lane;
        if (i >= sv) continue;
#pragma unroll
        for (int s = 0; s < W; ++s) {
          if (MODE == kLamport2S)
            d[k][s] = (s == rank) ? ld_nc_v4(xr + rank * sv + i) : ld_vol_v4(rs_at(p, rank, slot, s, row, i));
          else
            d[k][s] = ok ? ld_vol_v4(stage_at(p, s, slot, row, rank * sv + i)) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int k = 0; k < kChunk; ++k) {
        const int i = c0 + k * 32 + lane;
        if (i >= sv) continue;
        if (MODE == kLamport2S) {
#pragma unroll
          for (int s = 0; s < W; ++s) {
            if (s != rank && ok && !poll_vec<T>(rs_at(p, rank, slot, s, row, i), d[k][s], w)) {
              record_error(st, kErrTimeoutLanding, ((uint64_t)MODE << 32) | 2, ((uint64_t)row << 32) | i, s, e);
              ok = false;
            }
          }
#pragma unroll
          for (int s = 0; s < W; ++s)
            if (s != rank) st_vol_v4(rs_at(p, rank, slot, s, row, i), LP::fill());
        }
#pragma unroll
        for (int s = 0; s < W; ++s) {
          float f[V::N];
          V::to_float(d[k][s], f);
#pragma unroll
          for (int q = 0; q < V::N; ++q) a[k][q] += f[q];
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
      const int i = c0 + k * 32 + lane;
      if (i >= sv) continue;
      if (p.norm) {
        float r[V::N];
        V::to_float(rv[k], r);
#pragma unroll
        for (int q = 0; q < V::N; ++q) a[k][q] += r[q];
      }
      const uint4 hb = LP::clean(V::from_float(a[k]));
      float hf[V::N];
      V::to_float(hb, hf);
#pragma unroll
      for (int q = 0; q < V::N; ++q) ss += hf[q] * hf[q];
#pragma unroll
      for (int dd = 0; dd < W; ++dd) st_vol_v4(ag_at(p, (rank + dd) % W, slot, rank, row, i), hb);
    }
    const float part = warp_sum(ss);
    const unsigned long long word = ((unsigned long long)etag << 32) | __float_as_uint(part);
    if (lane < W) st_vol_u64(agp_at(p, lane, slot, rank, row, g % U), word);
  }
  if (MODE == kNvls2S) {
    // kNvB units per warp and step: one 16-byte multimem.ld_reduce per lane and unit is a round trip
    // through the switch, so every unit's load is issued before the first is used (the per-unit
    // arithmetic, and so the result, is the same as one unit at a time)
    constexpr int kNvB = 4;
    for (int g0 = warp; g0 < nunits; g0 += NW * kNvB) {
      uint4 sred[kNvB], rv[kNvB];
      int rowj[kNvB];
#pragma unroll
      for (int j = 0; j < kNvB; ++j) {
        const int g = g0 + j * NW, i = (g % U) * UV + lane;
        rowj[j] = g < nunits ? (int)blockIdx.x + (g / U) * (int)gridDim.x : -1;
        sred[j] = make_uint4(0, 0, 0, 0);
        if (rowj[j] >= 0 && i < sv) {
          if (p.norm) rv[j] = reinterpret_cast<const uint4*>(res + (size_t)rowj[j] * p.hidden)[rank * sv + i];
          if (ok) sred[j] = mm_ld_reduce<T>(p.mc + p.L.stage + stage_idx(p, slot, rowj[j], rank * sv + i) * 16);
        }
      }
#pragma unroll
      for (int j = 0; j < kNvB; ++j) {
        if (rowj[j] < 0) continue;  // warp-uniform: g depends on the warp only
        const int g = g0 + j * NW, i = (g % U) * UV + lane;
        float ss = 0.f;
        if (i < sv) {
          float a[V::N];
          V::to_float(sred[j], a);
          if (p.norm) {
            float r[V::N];
            V::to_float(rv[j], r);
#pragma unroll
            for (int q = 0; q < V::N; ++q) a[q] += r[q];
          }
          const uint4 hb = LP::clean(V::from_float(a));
          float hf[V::N];
          V::to_float(hb, hf);
#pragma unroll
          for (int q = 0; q < V::N; ++q) ss += hf[q] * hf[q];
          mm_st_v4(p.mc + p.L.hbuf + ((size_t)rowj[j] * p.L.max_hv + rank * sv + i) * 16, hb);
        }
        const float part = warp_sum(ss);
        if (lane == 0)
          mm_st_u64(p.mc + p.L.hpart + hpart_idx(p, rowj[j], rank, g % U) * 8,
                    ((unsigned long long)etag << 32) | __float_as_uint(part));
      }
    }
  }
  stamp(p, rank, e, 2);

  if (MODE == kNvls2S) {
    __threadfence_system();
    __syncthreads();
    const uint32_t nc = st->nvls_calls[blockIdx.x][1] + 1u;
    ok = nvls_barrier(p, rank, st, 1, nc, w) && ok;
    if (tid == 0) st->nvls_calls[blockIdx.x][1] = nc;
    // phase 3 (NVLS): this block's rows (the barrier covered exactly these rows), in groups of up to
    // 32: first each row's norm from its partial words (a warp per row), then every thread of the
    // block over the group's vectors with four 16-byte loads (and their gamma vectors) in flight
    __shared__ float s_rstd[32];
    const int nrows_b = (p.rows - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    for (int r0 = 0; r0 < nrows_b; r0 += 32) {
      const int nr = min(32, nrows_b - r0);
      for (int rl = warp; rl < nr; rl += NW) {
        const int row = (int)blockIdx.x + (r0 + rl) * (int)gridDim.x;
        float tot = 0.f;
        if (p.norm && ok && !row_partials<W>(p, rank, slot, row, U, etag, true, w, st, e, tot)) ok = false;
        if (lane == 0) s_rstd[rl] = rsqrtf(tot / (float)p.hidden + p.eps);
      }
      __syncthreads();
      const int items = nr * hv;
      for (int i0 = tid; i0 < items; i0 += 4 * NT) {
        uint4 hb[4], gv[4];
        int rowk[4], vk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int idx = i0 + k * NT;
          rowk[k] = -1;
          if (idx < items) {
            const int rl = idx / hv;
            vk[k] = idx - rl * hv;
            rowk[k] = rl;
            hb[k] = ld_vol_v4(p.base[rank] + p.L.hbuf +
                              ((size_t)((int)blockIdx.x + (r0 + rl) * (int)gridDim.x) * p.L.max_hv + vk[k]) * 16);
            if (p.norm) gv[k] = ld_nc_v4(reinterpret_cast<const uint4*>(p.gamma) + vk[k]);
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (rowk[k] < 0) continue;
          float hf[V::N];
          V::to_float(hb[k], hf);
          store_norm<T>(p, out, res, (int)blockIdx.x + (r0 + rowk[k]) * (int)gridDim.x, vk[k], hf, hb[k],
                        s_rstd[rowk[k]], &gv[k]);
        }
      }
      __syncthreads();  // s_rstd is rewritten by the next group
    }
  } else {
    // phase 3 (LAMPORT/PULL): flat over (row, v), two vectors per lane per step; a warp shares one
    // row per step (hv % 32 == 0)
    for (long long u0 = gtid - lane; u0 < total; u0 += 2 * gthreads) {
      uint4 hb[2], gv[2];
      uint4* at[2];
      int rowk[2], vk[2];
      float tot[2] = {0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const long long ub = u0 + k * gthreads;
        rowk[k] = -1;
        if (ub < total) {
          rowk[k] = (int)(ub / hv);
          vk[k] = (int)(ub + lane - (long long)rowk[k] * hv);
          const int s = vk[k] / sv, i = vk[k] - s * sv;
          at[k] = ag_at(p, rank, slot, s, rowk[k], i);
          hb[k] = ld_vol_v4(at[k]);
          if (p.norm) gv[k] = ld_nc_v4(reinterpret_cast<const uint4*>(p.gamma) + vk[k]);  // before any wait
        }
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (rowk[k] < 0 || !p.norm) continue;  // warp-uniform
        if (ok && !row_partials<W>(p, rank, slot, rowk[k], U, etag, false, w, st, e, tot[k])) ok = false;
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (rowk[k] < 0) continue;
        if (ok && !poll_vec<T>(at[k], hb[k], w)) {
          record_error(st, kErrTimeoutLanding, ((uint64_t)MODE << 32) | 3, ((uint64_t)rowk[k] << 32) | vk[k], 0, e);
          ok = false;
        }
        st_vol_v4(at[k], LP::fill());
        float hf[V::N];
        V::to_float(hb[k], hf);
        const float rstd = rsqrtf(tot[k] / (float)p.hidden + p.eps);
        store_norm<T>(p, out, res, rowk[k], vk[k], hf, hb[k], rstd, &gv[k]);
      }
    }
  }
  stamp(p, rank, e, 3);
  stamp(p, rank, e, 4);
  finish_call(st, e);
}

// Fill a region with a 32-bit pattern.
__global__ void k_fill_u32(uint32_t* p, uint32_t v, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    p[i] = v;
}

// Small all-gather with LL words {data32, epoch32}: one block, tags make clearing unnecessary.
__global__ void __launch_bounds__(1024) k_allgather_u32(const GatherParams p) {
  const int rank = p.emulate ? (int)blockIdx.y : p.rank;
  RankState* st = reinterpret_cast<RankState*>(p.base[rank] + p.L.state);
  const uint32_t* in = p.in + (size_t)rank * p.in_rs;
  uint32_t* out = p.out + (size_t)rank * p.out_rs;
  pdl_wait_then_trigger();
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&st->gather_epoch) + 1u;
  const int slot = (int)(e & 1u);
  auto at = [&](int owner, int src, int i) {
    return reinterpret_cast<unsigned long long*>(p.base[owner] + p.L.gather) +
           (((size_t)slot * p.L.world + src) * p.L.max_gather + i);
  };
  for (int i = threadIdx.x; i < p.n; i += blockDim.x) {
    const unsigned long long word = ((unsigned long long)e << 32) | in[i];
    for (int d = 0; d < p.world; ++d) st_vol_u64(at(d, rank, i), word);
  }
  Waiter w(p.timeout_ns, &st->error);
  bool ok = true;
  for (int idx = threadIdx.x; idx < p.n * p.world; idx += blockDim.x) {
    const int src = idx / p.n, i = idx - src * p.n;
    const unsigned long long* a = at(rank, src, i);
    unsigned long long wd = ld_vol_u64(a);
    while ((uint32_t)(wd >> 32) != e && ok) {
      if (w.expired()) {
        record_error(st, kErrTimeoutGather, 0, i, src, e);
        ok = false;
        break;
      }
      wd = ld_vol_u64(a);
    }
    out[idx] = (uint32_t)wd;
  }
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(&st->gather_epoch) = e;
}

template <typename T, int W>
cudaError_t launch_typed(const ARParams& p, cudaStream_t stream) {
  void (*fn)(const ARParams);
  // one-shot: a thread holds one vector of its CTA's row chunk when the chunk fits the block
  const int hv = p.hidden / Vec<T>::N, chunk = (hv + std::max(p.cluster, 1) - 1) / std::max(p.cluster, 1);
  const bool one = chunk <= p.threads;
  switch (p.variant) {
    case kLamport1S: fn = one ? k_oneshot<T, W, kLamport1S, 1, false> : k_oneshot<T, W, kLamport1S, kVPT, false>; break;
    case kLamport1SX: fn = one ? k_oneshot<T, W, kLamport1S, 1, true> : k_oneshot<T, W, kLamport1S, kVPT, true>; break;
    case kPull1S: fn = one ? k_oneshot<T, W, kPull1S, 1, false> : k_oneshot<T, W, kPull1S, kVPT, false>; break;
    case kNvls1S: fn = one ? k_oneshot<T, W, kNvls1S, 1, false> : k_oneshot<T, W, kNvls1S, kVPT, false>; break;
    case kLamport2S: fn = k_twoshot<T, W, kLamport2S>; break;
    case kPull2S: fn = k_twoshot<T, W, kPull2S>; break;
    case kNvls2S: fn = k_twoshot<T, W, kNvls2S>; break;
    default: return cudaErrorInvalidValue;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.blocks, p.emulate ? p.world : 1, 1);
  cfg.blockDim = dim3(p.threads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (p.cluster > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = p.cluster;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (p.pdl || pdl_flag()) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, fn, p);
}

template <typename T>
cudaError_t launch_world(const ARParams& p, cudaStream_t s) {
  switch (p.world) {
    case 2: return launch_typed<T, 2>(p, s);
    case 4: return launch_typed<T, 4>(p, s);
    case 8: return launch_typed<T, 8>(p, s);
    default: return cudaErrorInvalidValue;
  }
}

int elems_per_vec(int dtype) { return dtype == kF32 ? 4 : 8; }

}  // namespace

Layout plan_layout(int world, int max_rows, int max_hidden, int esize, int max_gather) {
  Layout L = {};
  L.world = world;
  L.max_rows = max_rows;
  L.esize = esize;
  L.max_hv = (int)((long long)max_hidden * esize / 16);
  L.sv_max = (L.max_hv + world - 1) / world;
  L.max_gather = max_gather;
  long long off = 0;
  auto take = [&](long long bytes) {
    const long long o = off;
    off = align_up(off + bytes, 4096);
    return o;
  };
  const long long R = max_rows, W = world, HV = L.max_hv, SV = L.sv_max;
  L.state = take(sizeof(RankState));
  L.flags = take((long long)kMaxBlocks * kMaxWorld * 8);
  L.nvls = take((long long)kMaxBlocks * 2 * 4);
  L.land1 = take(2 * W * R * HV * 16);
  L.rs = take(2 * W * R * SV * 16);
  L.ag = take(2 * W * R * SV * 16);
  L.agp = take(2 * W * R * pu_max(L) * 8);
  L.stage = take(2 * R * HV * 16);
  L.hbuf = take(R * HV * 16);
  L.hpart = take(R * W * pu_max(L) * 8);
  L.gather = take(2 * W * (long long)max_gather * 8);
  L.total = align_up(off, 2 << 20);
  return L;
}

cudaError_t init_heap(char* heap, const Layout& L, int dtype, cudaStream_t stream) {
  const uint32_t fill = dtype == kF32 ? 0x80000000u : 0x80008000u;
  cudaError_t err = cudaMemsetAsync(heap, 0, L.total, stream);
  if (err != cudaSuccess) return err;
  const long long lam_begin = L.land1, lam_end = L.agp;  // land1, rs, ag are contiguous
  const long long n = (lam_end - lam_begin) / 4;
  k_fill_u32<<<592, 256, 0, stream>>>(reinterpret_cast<uint32_t*>(heap + lam_begin), fill, n);
  return cudaGetLastError();
}

cudaError_t resolve_config(ARParams& p, int num_sms) {
  const int epv = elems_per_vec(p.dtype);
  if (p.world < 2 || p.world > kMaxWorld || (p.world & (p.world - 1)) != 0) return cudaErrorInvalidValue;
  if (p.hidden <= 0 || p.hidden % epv != 0) return cudaErrorInvalidValue;
  if (p.rows <= 0 || p.rows > p.L.max_rows) return cudaErrorInvalidValue;
  const int hv = p.hidden / epv;
  if (hv > p.L.max_hv) return cudaErrorInvalidValue;
  const bool two = p.variant == kLamport2S || p.variant == kPull2S || p.variant == kNvls2S;
  const bool nvls = p.variant == kNvls1S || p.variant == kNvls2S;
  if (nvls && p.mc == nullptr) return cudaErrorNotSupported;
  if (two && (hv % p.world != 0 || hv % 32 != 0)) return cudaErrorInvalidValue;
  const int ranks_per_gpu = p.emulate ? p.world : 1;
  const int budget = std::max(1, num_sms / ranks_per_gpu);  // resident CTAs (one per SM) per rank
  if (!two) {
    if (p.cluster <= 0) {
      // spread a row over enough CTAs that small batches still engage several SMs, and over at
      // least enough that each thread holds <= kVPT vectors of 512 threads
      int c = 1;
      while (c < 8 && (long long)p.rows * c * 2 <= budget) c *= 2;
      while (c < 8 && (hv + c - 1) / c > 512 * kVPT) c *= 2;
      while (c > 1 && p.blocks > 0 && p.blocks % c != 0) c /= 2;  // must divide a given block count
      p.cluster = c;
    }
    const int chunk = (hv + p.cluster - 1) / p.cluster;
    if (p.threads <= 0) p.threads = std::min(512, std::max(64, (chunk + 31) / 32 * 32));
    if (chunk > p.threads * kVPT) return cudaErrorInvalidValue;
    if (p.blocks <= 0) {
      const int clusters = std::max(1, std::min(p.rows, budget / p.cluster));
      p.blocks = clusters * p.cluster;
    }
    if (p.blocks % p.cluster != 0) return cudaErrorInvalidValue;
  } else {
    if (p.threads <= 0) p.threads = 256;
    p.threads = std::max(p.threads, 32);
    if (p.threads > 256) return cudaErrorInvalidValue;
    p.cluster = 1;
    if (p.blocks <= 0) {
      // LAMPORT: enough CTAs that every (row, unit) has a warp and the flat push / gather phases
      // have ~1 vector per thread; PULL: a CTA per row for the staging and reduce phases (their
      // barriers are per CTA), more when the flat all-gather phase wants them (CTAs without a row
      // pass their barrier and only gather); NVLS: a CTA per row; capped by one resident CTA per SM
      const int warps = p.threads / 32;
      const int units = (hv / p.world + 31) / 32;
      const long long by_units = ((long long)p.rows * units + warps - 1) / warps;
      const long long by_flat = ((long long)p.rows * hv + p.threads - 1) / p.threads;
      const long long b = p.variant == kLamport2S ? std::max(by_units, by_flat)
                          : p.variant == kPull2S  ? std::max((long long)p.rows, by_flat)
                                                  : (long long)p.rows;
      p.blocks = (int)std::max<long long>(1, std::min<long long>(b, budget));
    }
  }
  if (p.blocks > kMaxBlocks || p.blocks > budget) return cudaErrorInvalidValue;
  if (p.threads > 512 || p.threads % 32 != 0) return cudaErrorInvalidValue;
  return cudaSuccess;
}

cudaError_t launch_fused_ar(ARParams p, cudaStream_t stream) {
  switch (p.dtype) {
    case kF32: return launch_world<float>(p, stream);
    case kF16: return launch_world<__half>(p, stream);
    case kBF16: return launch_world<__nv_bfloat16>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_allgather_u32(GatherParams p, cudaStream_t stream) {
  if (p.n <= 0 || p.n > p.L.max_gather || p.world < 1 || p.world > kMaxWorld) return cudaErrorInvalidValue;
  return launch_k(k_allgather_u32, dim3(1, p.emulate ? p.world : 1, 1), dim3(1024), 0, stream, p);
}

}  // namespace cob
