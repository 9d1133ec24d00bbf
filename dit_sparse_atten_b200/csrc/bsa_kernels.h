// Internal launcher declarations shared by the kernel translation units and the
// C ABI (abi.cu).  Not part of the public interface (include/bsa.h is).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "bsa_common.cuh"

namespace bsa {

// ---- (c) reorder ----------------------------------------------------------
// dst_rows (optional): destination row of output index i, in [0, tokens_dst).
cudaError_t launch_reorder_rows(int n_tensors, const void* const* src, void* const* dst,
                                const int32_t* perm, int64_t batch, int64_t tokens_out,
                                int64_t tokens_in, int64_t row_bytes, int* err_word,
                                cudaStream_t stream, int num_sms,
                                const int32_t* dst_rows = nullptr, int64_t tokens_dst = 0);
// Head-parallel input exchange: packed rows of this call's heads pulled from
// the ranks' input shards (peer memory) into dst[0..2] (reorder.cu).
cudaError_t launch_pull_rows(const void* const* peers, int n_peers, int64_t peer_tokens,
                             int64_t src_row_bytes, int64_t src_tensor_bytes,
                             int64_t src_offset, const int32_t* perm, int64_t tokens,
                             int64_t row_bytes, void* const* dst, int* err_word,
                             cudaStream_t stream, int num_sms);

// ---- (b) route selection / CSR pack ----------------------------------------
struct SelectArgs {
  const float* mass;        // [rows, cols] fp32, or nullptr for a pure pack
  const uint8_t* prev;      // [rows, cols] 0/1, or nullptr
  const uint8_t* route_in;  // [rows, cols] 0/1 when packing an existing route
  float persistence;
  float target;
  int32_t cap;              // max(1, ceil(cols * keep))
  int32_t sink_blocks;
  int64_t rows;
  int32_t cols;
  int32_t rows_per_group;   // rows that share one kept counter (Qb)
  uint8_t* route_out;       // [rows, cols] or nullptr
  int32_t* counts;          // [rows] or nullptr
  int32_t* indices;         // [rows, cols] or nullptr
  unsigned long long* kept; // [rows / rows_per_group] or nullptr (accumulated)
};
cudaError_t launch_route_select(const SelectArgs& args, cudaStream_t stream);

// ---- (f4) attention prologue ------------------------------------------------
struct PrologueArgs {
  const __nv_bfloat16* q_in;      // [B, T, H * D] projections, row strides below (elements)
  const __nv_bfloat16* k_in;
  const __nv_bfloat16* v_in;
  int64_t batch, tokens;
  int32_t heads, head_dim;
  int64_t in_stride_b, in_stride_t;
  bool norm_q, norm_k;            // RMSNorm of Q / K over H * D
  const float* weight_q;          // [H * D] or nullptr (no affine)
  const float* weight_k;
  float eps;
  const float* rope_cos;          // [T, D / 2] or nullptr (no rotary embedding)
  const float* rope_sin;
  const int32_t* perm;            // [T] output row -> input token, or nullptr
  __nv_bfloat16* q_out;           // [B, T, H, D] contiguous, packed order
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  int* err_word;
};
cudaError_t launch_qkv_prologue(const PrologueArgs& args, cudaStream_t stream, int num_sms);

// ---- (f3) directional frontier update ---------------------------------------
enum DirectionalExpand : int { kExpandQ = 1, kExpandK = 2, kExpandJoint = 4 };

struct DirectionalArgs {
  const float* mass;              // [planes, n, n] fp32 block mass
  const uint8_t* prev;            // [planes, n, n] 0/1 previous route
  const int32_t* neighbors;       // [n, 4] spatial neighbour block ids, -1 = none
  const uint8_t* prev_frontier;   // [planes, n, n] 0/1, or nullptr (from prev)
  int64_t planes;
  int32_t n;
  float persistence, min_ratio, candidate_bonus, budget_scale;
  int32_t cap;                    // max(1, ceil(n * keep))
  int32_t explore_count;          // max(1, ceil(n * fraction)), 0 = no exploration
  int32_t expand;                 // DirectionalExpand bits
  int32_t sink_blocks;
  int32_t rows_per_group;         // rows that share one kept counter
  uint8_t* candidates;            // [planes, n, n]: zeroed, scattered, then final
  uint8_t* route_out;             // [planes, n, n] route after the sink
  uint8_t* exploration;           // [planes, n, n] or nullptr
  uint8_t* dropped;               // [planes, n, n] or nullptr (before the sink)
  uint8_t* added;                 // [planes, n, n] or nullptr (before the sink)
  int32_t* counts;                // [planes * n] or nullptr
  int32_t* indices;               // [planes * n, n] or nullptr
  unsigned long long* kept;       // [planes * n / rows_per_group] or nullptr (accumulated)
  int* err_word;
};
// Candidate scatter, then per-row selection; candidates must be zero on entry.
cudaError_t launch_directional_update(const DirectionalArgs& args, cudaStream_t stream,
                                      int num_sms);
cudaError_t launch_frontier_mask(const uint8_t* route, const int32_t* neighbors, int64_t planes,
                                 int32_t n, uint8_t* frontier, int* err_word,
                                 cudaStream_t stream, int num_sms);

// ---- (b) sampled block mass ------------------------------------------------
struct MassArgs {
  int64_t batch, heads, n_rows;   // rows of the [B, n_rows, H, D] inputs
  int32_t samples, q_blocks;      // rows (and keys) per block; blocks per row
  float scale;
  int32_t round_bf16;
  const float* block_bias;        // [Qb] additive key weight per key block, or null (0)
  float mass_scale;               // multiplies each block sum (1/S: mean over query samples)
  const float* lse;               // [B, H, n_rows] natural-log LSE per query row, or null
  float* mass;                    // [B, H, Qb, Qb]
  int* err_word;
  // One-pass mode (S <= 32, lse null): instead of `mass`, the kernel writes
  // block_lse[B, H, Qb, n_rows] = log2 of each row's exponential sum over each
  // key block's S keys (absolute: stabiliser included) and row_lse[B, H, n_rows]
  // = log2 of the row's total; launch_sampled_mass_reduce then forms the mass.
  float* block_lse;
  float* row_lse;
};
cudaError_t launch_sampled_mass(const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                                const MassArgs& args, cudaStream_t stream);
// mass[b, h, qb, kb] = mass_scale * sum_{s < S} 2^(block_lse[b, h, kb, qb S + s]
//                                                 - row_lse[b, h, qb S + s])
cudaError_t launch_sampled_mass_reduce(const MassArgs& args, cudaStream_t stream);
// One pass with the per-block sums kept in TMEM and shared memory (no
// workspace, no reduction launch): 16 or 32 samples and up to 473 blocks
// (sampled_mass_on_chip); block_lse and lse must be null.
bool sampled_mass_on_chip(int32_t q_blocks, int32_t samples);
cudaError_t launch_sampled_mass_on_chip(const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                                        const MassArgs& args, cudaStream_t stream);

// ---- (b) sampled block mass without a caller workspace ---------------------
// Size of the module-level scratch (a static __device__ array) that
// bsa_sampled_mass_noalloc gathers a chunk of heads' sampled Q/K rows and the
// key-block weights into: 2 * N * hc * 256 bytes + Qb * 4 for N = Qb * S
// sampled rows and hc heads per chunk.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
// Address of that scratch on the current device.
cudaError_t noalloc_scratch(void** ptr);
// Gathers the S sampled tokens of every block of heads [h0, h0 + hc) of batch
// element b of q and k (bf16 [B, T, H, 128] contiguous) into the scratch as
// [N, hc, 128] each, followed by the Qb key-block weights.
cudaError_t launch_gather_samples(const void* q, const void* k, int64_t T, int64_t H, int b,
                                  int h0, int hc, int block, int samples, int q_blocks,
                                  float bias_full, float bias_tail, void* scratch,
                                  cudaStream_t stream);

// ---- (a) block-sparse attention --------------------------------------------
constexpr int kMaxPeers = 8;   // ranks of one head-parallel group the attention stores to

struct AttnArgs {
  int64_t batch, tokens, heads;
  int32_t q_blocks, k_blocks;     // ceil(T / block)
  int32_t block;                  // 64 or 128
  int32_t route_cols;             // row stride of indices (>= k_blocks)
  int64_t route_batch_stride;     // in rows of [H * Qb]; 0 = one route for all batches
  const int32_t* counts;          // [RB, H, Qb]
  const int32_t* indices;         // [RB, H, Qb, route_cols]
  const __nv_bfloat16* q;         // [B, T, H, D] with the input strides below (elements)
  int64_t in_stride_b, in_stride_t, in_stride_h;
  float scale;
  __nv_bfloat16* out;             // [B, T, H, D] with strides below (elements)
  int64_t out_stride_b, out_stride_t, out_stride_h;
  float* lse;                     // [B, H, T] or nullptr (packed row order)
  int* err_word;
  // Output row of each packed query row: row i of every batch element goes
  // to token out_rows[i] of out (the reorder's permutation, folding the
  // unpack into the epilogue); nullptr writes row i to token i.
  const int32_t* out_rows;
  // Dense attention with block mass: non-null selects every key block in
  // order (counts / indices unused) and receives [B, H, Kb, T] per-row,
  // per-key-block log2 exponential sums (block == 128).
  float* block_lse;
  // Output shards on the ranks of a head-parallel group (batch 1): with
  // n_peer > 0 the row of token t goes to rank d = t / peer_tokens, token
  // t - d * peer_tokens of out_peer[d] (out_stride_t / out_stride_h apply),
  // out_peer[d] being rank d's buffer mapped into this process.  out unused.
  int32_t n_peer;
  int64_t peer_tokens;
  __nv_bfloat16* out_peer[kMaxPeers];
};
cudaError_t launch_attention(const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                             const CUtensorMap& tm_v, const AttnArgs& args,
                             cudaStream_t stream);
// The 128-token-block kernel that gives each CTA two adjacent query blocks
// (attention_pair.cu); launch_attention uses it for block == 128.
cudaError_t launch_attention_pair(const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                                  const CUtensorMap& tm_v, const AttnArgs& args,
                                  cudaStream_t stream);
// mass [B, H, Kb, Kb] from block_lse [B, H, Kb, T] and the natural-log row LSE
// [B, H, T] of the same dense pass (128-token blocks).
cudaError_t launch_block_mass(const float* block_lse, const float* lse, int64_t batch,
                              int64_t tokens, int64_t heads, int32_t blocks, float* mass,
                              cudaStream_t stream);

}  // namespace bsa
