// Host/device interface of the fused all-reduce + residual-add + RMSNorm family.
//
// Every rank owns one "symmetric heap": a device allocation that every other rank has mapped
// (NVLink 5 peer mapping) and, when NVSwitch multicast is available, that is also bound to one
// multicast object. All buffers sit at the same byte offset in every rank's heap, so a kernel
// reaches buffer B on rank r at `base[r] + L.B` and the in-switch reduced view of B at `mc + L.B`.
//
// The same kernels run in two modes:
//   * real   : one process per GPU, gridDim.y == 1, `rank` = this process's rank;
//   * emulate: all `world` ranks in ONE launch on one GPU (gridDim.y == world, rank = blockIdx.y),
//              each rank's heap a separate region of that GPU. This is how the multi-rank
//              protocol is exercised on a single GPU without separate launches that wait on one
//              another.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cob {

constexpr int kMaxWorld = 8;
constexpr int kMaxBlocks = 296;  // per-block barrier slots and epoch words: two CTAs on each of 148 SMs

enum Variant : int {
  kAuto = 0,
  kLamport1S = 1,  // one-shot push: every rank pushes its x to every peer, sums locally
  kLamport2S = 2,  // two-shot push: reduce-scatter push -> owner sums -> all-gather push of h
  kNvls1S = 3,     // one-shot NVSwitch multimem.ld_reduce of the whole message
  kNvls2S = 4,     // two-shot: multimem.ld_reduce of the owned slice -> multimem.st of h
  kPull1S = 5,     // one-shot pull: start barrier, every rank reads every peer's x
  kPull2S = 6,     // two-shot: pull reduce-scatter (start barrier) -> all-gather push of h
  kLamport1SX = 7, // kLamport1S whose row sums cross the cluster without a release-ordered barrier
  kNumVariants = 8,
};

// Per-rank control block (in the rank's own heap). Only this rank's kernels write it, except
// `flags` (separate region) which peers write.
struct alignas(256) RankState {
  unsigned long long epoch;          // number of completed fused calls on this rank (written by block 0)
  unsigned int unused;
  unsigned int error;                // sticky ErrBits (see common.cuh)
  unsigned long long err_detail[4];  // where the first error happened
  unsigned int flag_calls[kMaxBlocks];     // per-block call counter of the flag barrier
  unsigned int nvls_calls[kMaxBlocks][2];  // per-block call counters of the two NVLS barriers
  unsigned int gather_epoch;               // epoch of the small all-gather primitive
  unsigned int pad[3];
  // Epoch as read by block b of the next call. Block b of a call with G blocks writes entries
  // b, b + G, b + 2G, ... at its end, so every entry holds the same value whatever the grid size of
  // the next call; that call reads them only after this one has completed (stream order).
  unsigned long long blk_epoch[kMaxBlocks];
};

// Byte offsets of every region inside a heap (identical on all ranks). Sizes in comments use
// HV = max hidden size in 16-byte vectors, R = max rows, W = world, SV = HV / W.
struct Layout {
  long long state;   // RankState
  long long flags;   // u64 [kMaxBlocks][kMaxWorld]  flag barrier slots, written by peers
  long long nvls;    // u32 [kMaxBlocks][2] (padded)  multicast barrier counters
  long long land1;   // vec [2][W][R][HV]     one-shot push landing (Lamport fill)
  long long rs;      // vec [2][W][R][SV]     two-shot reduce-scatter landing (Lamport fill)
  long long ag;      // vec [2][W][R][SV]     two-shot all-gather landing (Lamport fill)
  long long agp;     // u64 [2][W][R][PU]     per-unit partial sums of squares {f32, epoch32},
                     //                       PU = ceil(SV / 32) units of 32 vectors per owner slice
  long long stage;   // vec [2][R][HV]        staged copy of x for pull / NVLS variants
  long long hbuf;    // vec [R][HV]           NVLS two-shot all-gathered h
  long long hpart;   // u64 [R][W][PU]        NVLS two-shot per-unit partials {f32, epoch32}
  long long gather;  // u64 [2][W][G]         small all-gather (LL words {u32 data, u32 epoch})
  long long total;   // heap size in bytes
  int world, max_rows, max_hv, sv_max, esize, max_gather;
};

struct ARParams {
  char* base[kMaxWorld];  // per-rank heap base as seen from this GPU
  char* mc;               // multicast view of the heaps (nullptr when NVLS is unavailable)
  Layout L;
  const void* x;          // this rank's partial sums [rows, hidden]
  void* residual;         // [rows, hidden], updated in place to residual + sum(x)
  const void* gamma;      // [hidden]
  void* out;              // [rows, hidden] = RMSNorm(residual + sum(x)) * gamma
  long long x_rs, res_rs, out_rs;  // emulate mode: element stride between ranks' tensors
  int rank, world, rows, hidden;
  float eps;
  int variant, blocks, threads, cluster;
  int emulate, pdl, dtype, norm;   // norm == 0: plain all-reduce into `out`, residual untouched
  unsigned long long timeout_ns;
  // Optional phase stamps (%globaltimer, ns): [rank][call % stamp_cap][kMaxBlocks][kStampPhases];
  // nullptr = off. Phase 0 start, 1 inputs sent / staged, 2 barrier passed or owner slice reduced,
  // 3 all data received, 4 block done.
  long long* stamps;
  int stamp_cap;
};

constexpr int kStampPhases = 5;

Layout plan_layout(int world, int max_rows, int max_hidden, int esize, int max_gather);

// Resolves kAuto and 0-valued geometry fields in place; returns cudaSuccess or an error code.
cudaError_t resolve_config(ARParams& p, int num_sms);
cudaError_t launch_fused_ar(ARParams p, cudaStream_t stream);
// Fill the Lamport landing regions with the dtype's sentinel and zero the control regions.
cudaError_t init_heap(char* heap, const Layout& L, int dtype, cudaStream_t stream);

// Small all-gather of 32-bit words (used for the distributed argmax of greedy decoding):
// out[src * n + i] = in_rank_src[i] for every rank src.
struct GatherParams {
  char* base[kMaxWorld];
  Layout L;
  const uint32_t* in;
  uint32_t* out;
  long long in_rs, out_rs;  // emulate strides (elements)
  int rank, world, n, emulate;
  unsigned long long timeout_ns;
};
cudaError_t launch_allgather_u32(GatherParams p, cudaStream_t stream);

}  // namespace cob
