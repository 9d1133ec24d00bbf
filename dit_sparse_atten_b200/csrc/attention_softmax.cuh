// Softmax helpers shared by the attention kernels (attention.cu,
// attention_pair.cu): a thread owns one query row of a 128-lane TMEM S tile
// and reads it in 32-column chunks.  Scores are handled in the log2 domain
// (scale * log2 e folded into one multiplier) with a running stabiliser.
#pragma once

#include "bsa_common.cuh"

namespace bsa {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: O is rescaled only past 2^8

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// The softmax reads a BK-column S row from TMEM in 32-column chunks: a first
// pass for the row max (all chunks loaded, one wait), then the exponentials,
// for which the first chunks are read again (the whole row does not fit the
// 168-register budget next to the exponential pass's own state).

// Columns of a chunk at or past `valid` (keys beyond the sequence) -> -inf.
__device__ __forceinline__ void mask_chunk(uint32_t* r, int c0, int64_t valid) {
#pragma unroll
  for (int x = 0; x < 32; ++x)
    if (c0 + x >= valid) r[x] = __float_as_uint(-INFINITY);
}

// Running row max of a chunk in 8 independent three-input chains.
__device__ __forceinline__ void max_chunk(float* m8, const uint32_t* r) {
#pragma unroll
  for (int x = 0; x < 32; x += 16) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      m8[q] = fmax3(m8[q], __uint_as_float(r[x + 2 * q]), __uint_as_float(r[x + 2 * q + 1]));
  }
}

// p = 2^(s*c - m) for one chunk: packed FMA for the argument, MUFU (or, for
// kEmulated of every 8 pairs, the FMA-pipe polynomial); the pairs are rounded
// to bf16 (nearest even, one conversion per pair) into 16 TMEM columns at
// pdst, and summed in fp32 into four packed accumulators.
template <int kEmulated>
__device__ __forceinline__ void exp_chunk(const uint32_t* r, float2 c2, float2 neg_m,
                                          float2* acc, uint32_t pdst) {
  uint32_t pk[16];
#pragma unroll
  for (int x = 0; x < 32; x += 2) {
    const float2 t =
        __ffma2_rn(make_float2(__uint_as_float(r[x]), __uint_as_float(r[x + 1])), c2, neg_m);
    float2 p;
    if (((x >> 1) & 7) >= 8 - kEmulated) {
      p = exp2_poly2(t);
    } else {
      p.x = ex2_approx(t.x);
      p.y = ex2_approx(t.y);
    }
    acc[(x >> 1) & 3] = __fadd2_rn(acc[(x >> 1) & 3], p);
    pk[x >> 1] = pack_bf16x2(p.x, p.y);
  }
  tmem_st_32x32b_x16(pdst, pk);
}

// Chunks of a row the first pass keeps in registers for the second (the
// rest are read from TMEM again): as many as the register budget allows.
template <int BK>
constexpr int kKeptChunks = BK == 128 ? 2 : 1;

// First pass: the row max (raw scores) of the BK-column S row at sbuf, all
// chunks loaded at once; the last kKeptChunks chunks stay in `keep` (masked)
// for the second pass.
// kBatched: the chunks re-read later are loaded and reduced first (one TMEM
// wait), then the kept ones (a second wait), so at most half a row is live at
// once (for register budgets below a full row plus working set).
template <int BK, int kKeep = kKeptChunks<BK>, bool kBatched = false>
__device__ __forceinline__ float row_max(uint32_t sbuf, bool partial, int64_t valid,
                                         uint32_t (&keep)[kKeep][32]) {
  constexpr int kChunks = BK / 32;
  constexpr int kFirst = kChunks - kKeep;
  uint32_t r[kFirst > 0 ? kFirst : 1][32];
  float m8[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) m8[q] = -INFINITY;
#pragma unroll
  for (int k = 0; k < kFirst; ++k) tmem_ld_32x32b_x32(sbuf + k * 32, r[k]);
  if constexpr (kBatched) {
    tmem_wait_ld();
#pragma unroll
    for (int k = 0; k < kFirst; ++k) {
      reg_fence<32>(r[k]);
      if (partial) mask_chunk(r[k], k * 32, valid);
      max_chunk(m8, r[k]);
    }
  }
#pragma unroll
  for (int k = 0; k < kKeep; ++k) tmem_ld_32x32b_x32(sbuf + (kFirst + k) * 32, keep[k]);
  tmem_wait_ld();
#pragma unroll
  for (int k = 0; k < (kBatched ? 0 : kFirst); ++k) {
    reg_fence<32>(r[k]);
    if (partial) mask_chunk(r[k], k * 32, valid);
    max_chunk(m8, r[k]);
  }
#pragma unroll
  for (int k = 0; k < kKeep; ++k) {
    reg_fence<32>(keep[k]);
    if (partial) mask_chunk(keep[k], (kFirst + k) * 32, valid);
    max_chunk(m8, keep[k]);
  }
  return fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
}

// Second pass: P (bf16) of the row into the first BK/2 columns of its own S
// buffer (chunk k's P goes to columns [16k, 16k + 16), which only chunks
// already read hold).  The first chunks are read from TMEM again (two buffers
// alternate so a load overlaps the previous chunk's arithmetic); the kept
// ones come from `keep`, already masked.  Returns the row's partial sums.
template <int BK, int kEmulated, int kKeep = kKeptChunks<BK>>
__device__ __forceinline__ float2 row_exp(uint32_t sbuf, bool partial, int64_t valid, float2 c2,
                                          float2 neg_m,
                                          const uint32_t (&keep)[kKeep][32], uint32_t pbuf = ~0u) {
  if (pbuf == ~0u) pbuf = sbuf;   // P of chunk k goes to columns pbuf + [16k, 16k + 16)
  constexpr int kChunks = BK / 32;
  constexpr int kReload = kChunks - kKeep;
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                   make_float2(0.f, 0.f)};
  uint32_t r[2][32];
  if constexpr (kReload > 0) {
    tmem_ld_32x32b_x32(sbuf, r[0]);
    tmem_wait_ld();
    reg_fence<32>(r[0]);
  }
#pragma unroll
  for (int k = 0; k < kReload; ++k) {
    if (k + 1 < kReload) tmem_ld_32x32b_x32(sbuf + (k + 1) * 32, r[(k + 1) & 1]);
    if (partial) mask_chunk(r[k & 1], k * 32, valid);
    exp_chunk<kEmulated>(r[k & 1], c2, neg_m, acc, pbuf + k * 16);
    if (k + 1 < kReload) {
      tmem_wait_ld();
      reg_fence<32>(r[(k + 1) & 1]);
    }
  }
#pragma unroll
  for (int k = 0; k < kKeep; ++k)
    exp_chunk<kEmulated>(keep[k], c2, neg_m, acc, pbuf + (kReload + k) * 16);
  return __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
}

}  // namespace attn
}  // namespace bsa
