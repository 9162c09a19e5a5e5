// Primitive probes (see probes.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cob {

struct RsProbeParams {
  char* base[8];          // per-rank probe heap (accumulator at acc_off, arrival counter at ctr_off)
  long long acc_off, ctr_off;
  const void* x;          // this rank's input: world slices of n elements (f32 or bf16)
  long long x_rank_bytes; // emulate mode: bytes between ranks' inputs (unused, and 0, on a real rank)
  int rank, world, n, variant, emulate;  // variant 0 red.f32, 1 red.v4.f32, 2 red.bf16x2, 3 red.v4.bf16x2
  unsigned long long timeout_ns;
  int* err;
};

cudaError_t rs_atomic_probe(const RsProbeParams& p, int blocks, cudaStream_t s);

// Push-vs-pull primitives over NVLink (all-gather and reduce-scatter of n 32-bit words per rank).
// Probe heap per rank (same offsets on every rank):
//   [0, 8 * kPrimMaxBlocks)                   u64 per-block epoch words (this rank only)
//   flags: u64 [kPrimMaxBlocks][8]            flag-barrier slots written by peers (pull forms)
//   stage: u32 [2][n]                         staged input for the pull forms (by epoch parity)
//   land : u32 [2][8][n / world]              Lamport landing for the push forms (sentinel 0x80000000)
//   nvls : u32 [kPrimMaxBlocks]               multicast-barrier counters (NVSwitch forms)
// Payload words are a hash of (source rank, index, epoch) so data of an earlier call is detected.
// NVSwitch forms: RS stages the whole vector and reduces its own slice in the switch
// (multimem.ld_reduce.add.u32); AG stores its slice into every rank's stage through the switch
// (multimem.st); both meet at a per-block multicast barrier (one multimem.red per rank, wait for
// epoch x world on the local copy, so a heap runs either these forms or the others, not both).
constexpr int kPrimMaxBlocks = 256;
enum PrimMode : int { kAgPull = 0, kAgPush = 1, kRsPull = 2, kRsPush = 3, kRsNvls = 4, kAgNvls = 5 };
struct PrimParams {
  char* base[8];
  char* mc;                                  // multicast view of the heaps (NVSwitch forms), or nullptr
  long long flags_off, stage_off, land_off, nvls_off;  // byte offsets in every heap
  int rank, world, n, mode, emulate;
  unsigned long long timeout_ns;
  unsigned int* bad;  // [ranks] words whose value did not match the expected payload
  int* err;           // set on a timed-out wait
};
size_t prim_heap_bytes(int world, int n, long long* flags_off, long long* stage_off, long long* land_off,
                       long long* nvls_off);
cudaError_t prim_probe(const PrimParams& p, int blocks, int threads, cudaStream_t s);
// Line-atomicity probe (the premise behind LL128-style flag-in-line protocols): writer ranks hit every
// 128-byte line (32 u32 words; word 31 is the line's flag) of the target rank's buffer with one warp-wide
// operation per line while the target's observer warps read each line with one warp-wide load and
// count lines whose flag says "complete" but whose other words do not.
//   mode 0: every writer adds to all 32 words (red.relaxed.sys.add.u32; flag += 1, data += rank + 1);
//           complete = flag == number of writers, data must then equal the sum of (rank + 1).
//   mode 1: one writer per line stores 32 x 4 bytes (flag = epoch, data = hash(word, line, epoch)).
//   mode 2: one writer per line stores 8 x 16 bytes (4 lines per warp instruction), same contents.
// Store modes run in steady state (the buffer is never cleared; the epoch grows per launch), so data
// of the previous launch under a new flag is a violation. Writers never wait; the observer gives up
// at one deadline for the whole launch and counts the lines it did not reach as timeouts.
// counters (u64, target rank's device memory): [0] violations [1] lines seen in progress before they
// completed [2] timeouts [3] lines observed complete [4] lines wrong after the launch (check kernel).
enum LineMode : int { kLineAtomic = 0, kLineStore4 = 1, kLineStore16 = 2 };
struct LineProbeParams {
  char* base[8];
  long long lines_off;  // byte offset of the lines in the target's heap (multiple of 128)
  long long n_lines;
  int rank, world, target, mode, emulate;
  int observer_blocks, writer_blocks;  // blocks of the target's observer / of every writer rank
  unsigned int epoch;                  // store modes: this launch's flag value (>= 1)
  unsigned long long timeout_ns;
  unsigned long long* counters;
};
// Runs this rank's role (emulate: every role in one launch, which must be co-resident on this GPU).
cudaError_t line_probe(const LineProbeParams& p, cudaStream_t s);
// Counts lines of the target's buffer that differ from their final expected contents into counters[4].
cudaError_t line_check(const LineProbeParams& p, cudaStream_t s);
// out[0] = SM cycles, out[1] = %globaltimer nanoseconds over a spin of `ns` nanoseconds
cudaError_t clock_calibration(unsigned long long ns, long long* out, cudaStream_t s);

}  // namespace cob
