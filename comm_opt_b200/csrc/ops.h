// Host entry points of the single-GPU decode kernels (plain CUDA, no torch types).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cob {

// out = x * rsqrt(mean(x^2) + eps) * gamma                      (rows x hidden, one CTA per row)
cudaError_t rmsnorm(const void* x, const void* gamma, void* out, int rows, int hidden, float eps, int dtype,
                    cudaStream_t s);
// residual += x; out = RMSNorm(residual) * gamma  (world-size-1 form of the fused op)
cudaError_t add_rmsnorm(const void* x, void* residual, const void* gamma, void* out, int rows, int hidden,
                        float eps, int dtype, cudaStream_t s);
// out[i] = table[ids[i]]                                        (bf16/fp16/fp32 rows, int32 ids)
cudaError_t embedding(const int32_t* ids, const void* table, void* out, int rows, int hidden, int dtype,
                      cudaStream_t s);
// qkv: [B, (nq + 2*nkv) * D]; rotates q and k by position (rotate-half RoPE, cos/sin tables
// [max_pos, D/2] fp32), writes rotated q to q_out [B, nq, D] and k, v into the paged caches
// [num_blocks, nkv, block, D] at slot (block_tables[b][pos / block], pos % block). `bias`
// ([(nq + 2*nkv) * D] of the qkv dtype, or nullptr) is added to q, k and v first.
cudaError_t rope_append_kv(const void* qkv, const void* bias, const int32_t* positions, const float* cos_t,
                           const float* sin_t, const int32_t* block_tables, int max_blocks_per_seq, void* q_out,
                           void* k_cache, void* v_cache, int batch, int nq, int nkv, int head_dim, int block_size,
                           int dtype, cudaStream_t s);
// out[b, i] = silu(gu[b, i]) * gu[b, I + i]; with interleave = c > 0 the row holds blocks of c gate
// then c up features: out[b, i] = silu(gu[b, 2c (i / c) + i % c]) * gu[b, 2c (i / c) + c + i % c]
cudaError_t silu_mul(const void* gu, void* out, int rows, int inter, int dtype, cudaStream_t s, int interleave = 0);
// Per row: fold max over the local vocabulary into keys[row] (atomicMax of an order-preserving
// 64-bit key: value high, inverted global index low; keys must be zero before).
cudaError_t argmax_local(const void* logits, unsigned long long* keys, int rows, int vocab, int vocab_offset,
                         int dtype, cudaStream_t s);
// gathered: [world, rows] keys from every rank -> ids[row] (ties: lowest index); when given,
// positions/seq_lens are incremented (decode-step feedback inside a CUDA graph) and local_keys cleared
cudaError_t argmax_combine(const unsigned long long* gathered, int32_t* ids, int rows, int world, int32_t* positions,
                           int32_t* seq_lens, unsigned long long* local_keys, cudaStream_t s);

// Paged GQA decode attention (split-KV with in-kernel combine by the last split).
struct AttnParams {
  const void* q;             // [B, nq, D]
  const void* k_cache;       // [num_blocks, nkv, block, D]
  const void* v_cache;
  const int32_t* block_tables;  // [B, max_blocks_per_seq]
  const int32_t* seq_lens;      // [B]
  void* out;                 // [B, nq, D]
  float* part_o;             // scratch [B, nkv, splits, G, D] fp32
  float* part_ml;            // scratch [B, nkv, splits, G, 2] fp32
  int32_t* counters;         // scratch [B * nkv] int32, zero between calls (kernel restores it)
  int batch, nq, nkv, head_dim, block_size, max_blocks_per_seq, splits, pages_per_split;
  float scale;
  int dtype;
  int num_blocks;            // rows of the caches / (nkv * block); 0 = unknown
  int* err;                  // optional: set to 1 if a bounded wait gave up
  int cluster;               // 1: merge splits (<= 8) inside a thread-block cluster, no scratch used
  // Optional RoPE + KV append of the new token (qkv != nullptr; q is then not read): the query heads of
  // each KV group and the new token's k / v head come from the QKV projection output, the bias (if any)
  // is added, RoPE is applied at positions[b], and the new k / v row is written into the caches at
  // positions[b] and used for the newest token (one kernel instead of the append kernel + attention).
  const void* qkv;           // [B, (nq + 2 nkv) * D]
  const void* qkv_bias;      // [(nq + 2 nkv) * D] or nullptr
  const int32_t* positions;  // [B]: position of the new token (= seq_lens[b] - 1)
  const float* cos_t;        // [max_pos, D / 2]
  const float* sin_t;
};
// bytes of scratch needed for a given geometry
size_t attn_scratch_bytes(int batch, int nkv, int splits, int group, int head_dim);
cudaError_t paged_decode_attention(const AttnParams& p, cudaStream_t s);
// KV ring depth of the attention kernel, read at launch: 6 = the deep ring (one CTA per SM) where the
// grid fits one wave at one CTA per SM and clusters of at most 8; any other value = 3 pages per warp.
int& attn_stage_mode();
// Dynamic shared memory of one attention launch (the KV ring of `stages` pages per warp, the query tile,
// barriers, the page list, the RoPE row, and the push merge's buffer for clusters of 2..8).
size_t attn_launch_smem_bytes(int splits, int group, int head_dim, bool cluster, int stages);

}  // namespace cob
