// (b) Block mass on tcgen05: the sampled mass of the route update and the
// exact mass of the dense bootstrap.
//
// Sampled (attention_backends/flex.py:205-251): for every head, the sampled
// queries ([Qb*S, D], S evenly spaced tokens per block) attend to all sampled
// keys ([Qb*S, D]) with an additive per-key weight log(block_size / S); the
// softmax row is then summed over the S key samples of each key block and
// averaged over the S query samples of each query block:
//   mass[h, qb, kb] = (1/S) * sum_{r in qb} sum_{k in kb} softmax_r(k).
// With round_bf16 set, scores are rounded like the reference's bf16 matmul
// output and bf16 `* score_scale` (flex.py:245) before the fp32 softmax.
//
// Exact (flex.py:97-108,167-202): the same with S = block over all tokens,
// no weights, no rounding and no mean: the probability summed over each
// block x block tile.  Given the per-query log-sum-exp of the dense pass
// (MassArgs::lse) only the second pass runs, as in the reference.
//
// One CTA per (128 query rows, head, batch).  The 128-key tiles stream through
// a TMA ring: pass 1 computes every row's log-sum-exp, pass 2 the normalised
// per-block sums.
#include <atomic>

#include "bsa_kernels.h"

namespace bsa {
namespace {

constexpr int kSlots = 5;
constexpr int kTile = 128;
constexpr float kLog2eM = 1.4426950408889634f;
constexpr int kQBytes = kTile * 256;
constexpr int kSlotBytes = kTile * 256;
constexpr int kPanel = kTile * 128;
constexpr int kMaxBlocks = 4096;

struct MassBarriers {
  uint64_t q_full;
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t drain;
  uint64_t slot_full[kSlots];
  uint64_t slot_empty[kSlots];
  uint64_t red_full[2];   // S > 32: eight warps' partials of a group of tiles written
  uint64_t red_free[2];   // S > 32: the group's slots summed and free again
  uint32_t tmem_base;
  int abort;
};

// ---------------------------------------------------------------------------
// Softmax warps (MassShape): warp w owns rows 32*(w%4).. and column part w/4
// of every S tile (quarters for S <= 32, halves for S = 64, 128), keeps its
// own running (max, sum) over its part of the row in pass 1 and combines it
// with the other parts once, through shared memory, before pass 2 (or before
// writing the row's log-sum-exp in one-pass mode).  All score arithmetic is
// packed (f32x2); the reference's two bf16 roundings (matmul output, then
// `* score_scale`) are split between the conversion unit (the first) and the
// FMA pipe (the second, by Veltkamp splitting), so that neither pipe carries
// both next to the exponentials; a share of the exponentials runs on the FMA
// pipe too (exp2_poly2).  For S <= 32 a query block's S rows are S
// consecutive lanes, reduced with shuffles.  For S = 64, 128 (exact mass) a
// query block spans several warps: each warp sums its 32 rows with shuffles
// and writes one partial per key tile into shared memory; every kRedTiles
// tiles warp 0 adds the eight partials in a fixed order (deterministic) and
// writes the mass.  The hand-over uses mbarriers with bounded waits
// (red_full / red_free, double-buffered).  After the softmax warps: the TMA
// producer warp, then the TMEM allocator + tcgen05.mma issuer warp.
constexpr int kRedTiles = 16;

// Shared-memory layout.  kOnChip (one pass, the per-block log sums kept on
// chip instead of a workspace): a two-slot K ring, and after the barriers a
// [block - kTmemVals][row] float area for the blocks past the first
// kTmemVals, whose values live in TMEM columns 256 + block.
template <bool kOnChip>
struct MassLayout {
  static constexpr int kRingSlots = kOnChip ? 2 : kSlots;
  static constexpr int kRing = kQBytes;
  static constexpr int kBias = kRing + kRingSlots * kSlotBytes;
  static constexpr int kXchg = kBias + kMaxBlocks * 4;
  static constexpr int kRed = kXchg + 4 * 128 * 2 * 4;          // [2][kRedTiles][8] floats
  static constexpr int kBar = kRed + 2 * kRedTiles * 8 * 4;
  static constexpr int kVals = kBar + 256;
  static constexpr int kBytes = kVals + 1024;                   // + base alignment slack
};
constexpr int kTmemVals = 256;     // on-chip mode: block log sums in TMEM columns [256, 512)
constexpr int kMaxDynSmem = 232448;
// Blocks the on-chip mode holds: TMEM, then shared memory (473 at 227 KB).
constexpr int kOnChipMaxBlocks =
    kTmemVals + (kMaxDynSmem - MassLayout<true>::kBytes) / (128 * 4);
constexpr int kMassEmulated = 2;  // of every 8 column pairs, exponentials on the FMA pipe

// Warp layout.  S = 16, 32: sixteen softmax warps, four per SM sub-partition,
// warp w owning rows 32*(w%4).. and column quarter w/4 of every S tile (more
// warps to hide the TMEM-load -> exponential -> sum chain; 18 warps cap a
// thread at 96 registers, which the per-block state of S <= 8 exceeds).
// Other S: eight softmax warps on column halves.  Then the TMA producer warp
// and the MMA warp (TMEM allocator).
template <int LOG2S>
struct MassShape {
  static constexpr int kParts = (LOG2S == 4 || LOG2S == 5) ? 4 : 2;  // column parts of a row
  static constexpr int kSoftWarps = 4 * kParts;
  static constexpr int kThreads = 32 * kSoftWarps + 64;
  static constexpr int kProdWarp = kSoftWarps;
  static constexpr int kMmaWarp = kSoftWarps + 1;
  static constexpr int kCols = kTile / kParts;          // columns per softmax thread
  static constexpr int kPairs = kCols / 2;
};

// The same rounding through the conversion unit: one cvt.rn.bf16x2 packs both
// values, two integer operations unpack them.  The kernel rounds the raw score
// this way and the scaled score by Veltkamp splitting, which balances the
// conversion/ALU pipes against the FMA pipe (4.9 -> 4.3 ms on config 4).
__device__ __forceinline__ float2 round2_bf16_cvt(float2 x) {
  const uint32_t p = pack_bf16x2(x.x, x.y);
  return make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
}

template <int kEmulate>
__device__ __forceinline__ float2 exp2_pair(float2 t) {
  if constexpr (kEmulate) {
    return exp2_poly2(t);
  } else {
    return make_float2(ex2_approx(t.x), ex2_approx(t.y));
  }
}

// Log2-domain scores of 64 keys starting at key0 (bias = log(size/S) per key
// block, keys past n_rows -> -inf), from the raw fp32 accumulators r.
template <int LOG2S, bool kRound, int kPairs>
__device__ __forceinline__ void mass_scores(const uint32_t* r, float2* y, int64_t key0,
                                            int64_t n_rows, const float* sBiasL, float scale) {
  const float2 sc2 = make_float2(scale, scale);
  const float2 l2e = make_float2(kLog2eM, kLog2eM);
  const int64_t kb0 = key0 >> LOG2S;
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    float2 v = make_float2(__uint_as_float(r[2 * p]), __uint_as_float(r[2 * p + 1]));
    if constexpr (kRound) {
      v = round2_bf16(__fmul2_rn(round2_bf16_cvt(v), sc2));
    } else {
      v = __fmul2_rn(v, sc2);
    }
    float2 bl;
    if constexpr (LOG2S == 0) {
      bl = make_float2(sBiasL[kb0 + 2 * p], sBiasL[kb0 + 2 * p + 1]);
    } else {
      const float bb = sBiasL[kb0 + ((2 * p) >> LOG2S)];
      bl = make_float2(bb, bb);
    }
    y[p] = __ffma2_rn(v, l2e, bl);
  }
  if (key0 + 2 * kPairs > n_rows) {
#pragma unroll
    for (int p = 0; p < kPairs; ++p) {
      if (key0 + 2 * p >= n_rows) y[p].x = -INFINITY;
      if (key0 + 2 * p + 1 >= n_rows) y[p].y = -INFINITY;
    }
  }
}

// The reference's rounded and scaled scores of 2 * kPairs keys starting at
// key0 (keys past n_rows -> -inf), before the log2(e) factor and the block
// bias: one-pass mode folds both, and its stabiliser, into one FMA per pair.
template <bool kRound, int kPairs>
__device__ __forceinline__ void mass_scores_scaled(const uint32_t* r, float2* v, int64_t key0,
                                                   int64_t n_rows, float scale) {
  const float2 sc2 = make_float2(scale, scale);
#pragma unroll
  for (int p = 0; p < kPairs; ++p) {
    float2 x = make_float2(__uint_as_float(r[2 * p]), __uint_as_float(r[2 * p + 1]));
    if constexpr (kRound) {
      x = round2_bf16(__fmul2_rn(round2_bf16_cvt(x), sc2));
    } else {
      x = __fmul2_rn(x, sc2);
    }
    v[p] = x;
  }
  if (key0 + 2 * kPairs > n_rows) {
#pragma unroll
    for (int p = 0; p < kPairs; ++p) {
      if (key0 + 2 * p >= n_rows) v[p].x = -INFINITY;
      if (key0 + 2 * p + 1 >= n_rows) v[p].y = -INFINITY;
    }
  }
}

// Of every 8 pairs, exponentials on the FMA pipe in one-pass mode.  Measured
// at config 4: 0, 1, 2 -> 3.02, 2.97, 2.97 ms; 1 keeps the polynomial's
// error on the fewest terms.
constexpr int kOnePassEmulated = 1;

// The sum of S values over S consecutive lanes, for S values at once:
// afterwards x[0] of lane l is the sum over its S-lane group of value
// (l mod S) (a butterfly that halves the values kept at each step).
template <int S>
__device__ __forceinline__ void lane_group_sums(float (&x)[S]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int half = S / 2; half >= 1; half >>= 1) {
    const bool up = (lane & half) != 0;
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float send = up ? x[j] : x[j + half];
      const float keep = up ? x[j + half] : x[j];
      x[j] = keep + __shfl_xor_sync(0xffffffffu, send, half);
    }
  }
}

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&x)[N]) {
  uint32_t r[32];
  if constexpr (N == 32) {
    tmem_ld_32x32b_x32(taddr, r);
  } else if constexpr (N == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
  } else if constexpr (N == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
  } else {
    static_assert(N == 4, "4, 8, 16 or 32 columns");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
  }
  tmem_wait_ld();
  reg_fence<N>(r);
#pragma unroll
  for (int j = 0; j < N; ++j) x[j] = __uint_as_float(r[j]);
}

// kOnChip: one pass with no workspace.  Each sampled row keeps the log2 of
// its exponential sum over every key block (running stabiliser folded in) in
// TMEM columns 256 + block (the first kTmemVals blocks) and in shared memory
// (the rest); once the row's log-sum-exp is known the CTA forms the mass of
// its S-row query blocks itself: 2^(block value - row), summed over the S
// rows (lanes) of each query block, times 1/S.
template <int LOG2S, bool kRound, bool kOnChip = false>
__global__ void __launch_bounds__(MassShape<LOG2S>::kThreads, 1)
    sampled_mass_kernel2(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k, const MassArgs a) {
  constexpr int S = 1 << LOG2S;
  constexpr bool kWide = S > 32;              // a query block spans several warps
  using Shape = MassShape<LOG2S>;
  constexpr int kParts = Shape::kParts;
  constexpr int kCols = Shape::kCols;
  constexpr int kPairs = Shape::kPairs;
  constexpr int kPartBlocks = kWide ? 1 : kCols / S;  // key blocks in a part of a tile row
  static_assert(S <= 128, "at most 128 rows per block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  using L = MassLayout<kOnChip>;
  constexpr int kRing = L::kRingSlots;
  uint8_t* sQ = smem;
  uint8_t* sRing = smem + L::kRing;
  float* sBiasL = reinterpret_cast<float*>(smem + L::kBias);
  float2* sX = reinterpret_cast<float2*>(smem + L::kXchg);  // [part][row] (max, sum)
  float* sRed = reinterpret_cast<float*>(smem + L::kRed);    // [buf][tile][warp] (S > 32)
  MassBarriers* bar = reinterpret_cast<MassBarriers*>(smem + L::kBar);
  float* sVals = reinterpret_cast<float*>(smem + L::kVals);  // kOnChip: [block - 256][row]
  volatile int* abort_flag = &bar->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int n_tiles = static_cast<int>((a.n_rows + kTile - 1) / kTile);
  // With the log-sum-exp given, pass 1 is skipped; in one-pass mode pass 1
  // emits per-block log sums and pass 2 is left to the reduction kernel.
  // (S <= 2 has one or two keys per block: the per-block state of one-pass
  // mode would not fit the registers, so those take two passes.)
  constexpr bool kOnePass = !kWide && LOG2S >= 2;
  static_assert(!kOnChip || kOnePass, "on-chip mode is one-pass");
  const bool emit = kOnePass && a.block_lse != nullptr;
  const bool one = emit || kOnChip;           // a single pass over the keys
  const int pass1 = a.lse != nullptr ? 0 : n_tiles;
  const int steps = one ? n_tiles : pass1 + n_tiles;

  if (threadIdx.x == 0) {
    mbar_init(&bar->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->s_free[i], Shape::kSoftWarps * 32);
      mbar_init(&bar->red_full[i], 8);
      mbar_init(&bar->red_free[i], 1);
    }
    mbar_init(&bar->drain, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&bar->slot_full[s], 1);
      mbar_init(&bar->slot_empty[s], 1);
    }
    bar->abort = prior_timeout(a.err_word) ? 1 : 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (bar->abort) return;  // uniform: set before the barrier, read after it
  for (int i = threadIdx.x; i < a.q_blocks; i += Shape::kThreads)
    sBiasL[i] = a.block_bias != nullptr ? a.block_bias[i] * kLog2eM : 0.f;
  if (warp == Shape::kMmaWarp) tmem_alloc(&bar->tmem_base, kOnChip ? 512 : 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;

  if (warp == Shape::kProdWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      mbar_arrive_expect_tx(&bar->q_full, kQBytes);
      tma_load_4d(sQ, &tm_q, &bar->q_full, 0, h, qt * kTile, b);
      tma_load_4d(sQ + kPanel, &tm_q, &bar->q_full, 64, h, qt * kTile, b);
      uint32_t armed = 0, armed_phase = 0;
      for (int i = 0; i < steps; ++i) {
        const int s = i % kRing;
        const uint32_t ph = (i / kRing) & 1;
        if (!mbar_wait(&bar->slot_empty[s], ph ^ 1, abort_flag, a.err_word)) break;
        const int kt = i % n_tiles;
        uint8_t* dst = sRing + s * kSlotBytes;
        mbar_arrive_expect_tx(&bar->slot_full[s], kSlotBytes);
        tma_load_4d(dst, &tm_k, &bar->slot_full[s], 0, h, kt * kTile, b);
        tma_load_4d(dst + kPanel, &tm_k, &bar->slot_full[s], 64, h, kt * kTile, b);
        armed |= 1u << s;
        armed_phase = (armed_phase & ~(1u << s)) | (ph << s);
      }
      int never = 0;
      mbar_wait(&bar->q_full, 0, &never, a.err_word);
#pragma unroll
      for (int s = 0; s < kRing; ++s)
        if (armed & (1u << s)) mbar_wait(&bar->slot_full[s], (armed_phase >> s) & 1u, &never, a.err_word);
    }
  } else if (warp == Shape::kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, kTile, false);
      const uint64_t qdesc = sdesc_sw128(smem_u32(sQ), 16, 1024);
      const uint64_t kdesc0 = sdesc_sw128(smem_u32(sRing), 16, 1024);
      bool ok = mbar_wait(&bar->q_full, 0, abort_flag, a.err_word);
      for (int i = 0; ok && i < steps; ++i) {
        const int s = i % kRing;
        ok = mbar_wait(&bar->slot_full[s], (i / kRing) & 1, abort_flag, a.err_word);
        if (ok && i >= 2) ok = mbar_wait(&bar->s_free[i & 1], ((i >> 1) - 1) & 1, abort_flag, a.err_word);
        if (!ok) break;
        tc_fence_after();
        const uint64_t kd = kdesc0 + static_cast<uint64_t>((s * kSlotBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk >> 2) * kPanel + (kk & 3) * 32) >> 4);
          umma_bf16_ss(tmem + (i & 1) * 128, qdesc + off, kd + off, idesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar->s_full[i & 1]);
        umma_commit(&bar->slot_empty[s]);
      }
      int never = 0;
      umma_commit(&bar->drain);
      mbar_wait(&bar->drain, 0, &never, a.err_word);
    }
  } else {
    const int part = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
    const int64_t qrow = static_cast<int64_t>(qt) * kTile + row;
    const int64_t out_rows = (static_cast<int64_t>(b) * a.heads + h) * a.q_blocks;
    float m2 = -INFINITY, l = 0.f, m_fold = 0.f;
    if (a.lse != nullptr && qrow < a.n_rows)
      m_fold = a.lse[(static_cast<int64_t>(b) * a.heads + h) * a.n_rows + qrow] * kLog2eM;
    bool combined = pass1 == 0;   // pass 1's row parts met (named barrier 1 + wq)
    bool ok = true;
    for (int i = 0; i < steps; ++i) {
      if (!mbar_wait(&bar->s_full[i & 1], (i >> 1) & 1, abort_flag, a.err_word)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[kCols];
#pragma unroll
      for (int c = 0; c < kCols; c += 32)
        tmem_ld_32x32b_x32(tmem + lane_addr + (i & 1) * 128 + part * kCols + c, r + c);
      tmem_wait_ld();
      reg_fence<kCols>(r);
      tc_fence_before();
      mbar_arrive(&bar->s_free[i & 1]);
      const int64_t key0 = static_cast<int64_t>(i % n_tiles) * kTile + part * kCols;
      if (kOnePass && one) {
        // One pass.  Stabiliser: the running max of (score * log2 e + the
        // largest block bias of this part), an upper bound of every argument,
        // so each exponential's argument is a single FMA with a per-block
        // constant (bias - m).
        float2 v[kPairs];
        mass_scores_scaled<kRound, kPairs>(r, v, key0, a.n_rows, a.scale);
        const int64_t kb0 = key0 >> LOG2S;
        // Block kb0 + gi covers pairs [gi * S / 2, (gi + 1) * S / 2) of this
        // part.
        auto bias = [&](int gi) { return kb0 + gi < a.q_blocks ? sBiasL[kb0 + gi] : 0.f; };
        float bmax = -INFINITY;
#pragma unroll
        for (int gi = 0; gi < kPartBlocks; ++gi)
          if (kb0 + gi < a.q_blocks) bmax = fmaxf(bmax, sBiasL[kb0 + gi]);
        float m8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) m8[q] = fmaxf(v[q].x, v[q].y);
#pragma unroll
        for (int p = 8; p < kPairs; p += 8) {
#pragma unroll
          for (int q = 0; q < 8; ++q) m8[q] = fmax3(m8[q], v[p + q].x, v[p + q].y);
        }
        const float vmax = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]),
                                 fmaxf(m8[6], m8[7]));
        const float m_tile = vmax == -INFINITY ? -INFINITY : __fmaf_rn(vmax, kLog2eM, bmax);
        const float m_new = fmaxf(m2, m_tile);
        if (m_new != -INFINITY) {
          const float2 l2e = make_float2(kLog2eM, kLog2eM);
          float* dst = kOnChip ? nullptr : a.block_lse + (out_rows + kb0) * a.n_rows + qrow;
          const bool write = qrow < a.n_rows;
          float tot = 0.f;
          constexpr int kBlockPairs = S / 2;
#pragma unroll
          for (int gi = 0; gi < kPartBlocks; ++gi) {
            const float c = __fsub_rn(bias(gi), m_new);
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int u = 0; u < kBlockPairs; ++u) {
              const int p = gi * kBlockPairs + u;
              const float2 t = __ffma2_rn(v[p], l2e, make_float2(c, c));
              const float2 e =
                  (p & 7) >= 8 - kOnePassEmulated ? exp2_pair<1>(t) : exp2_pair<0>(t);
              acc = __fadd2_rn(acc, e);
            }
            const float g = acc.x + acc.y;
            tot += g;
            const float val = m_new + __log2f(g);
            if constexpr (kOnChip) {
              const int kb = static_cast<int>(kb0) + gi;     // the same for the whole warp
              if (kb < kTmemVals)
                tmem_st_32x32b_x1(tmem + lane_addr + kTmemVals + kb, __float_as_uint(val));
              else if (kb < a.q_blocks)
                sVals[(kb - kTmemVals) * 128 + row] = val;
            } else if (write && kb0 + gi < a.q_blocks) {
              dst[gi * a.n_rows] = val;
            }
          }
          l = l * ex2_approx(m2 - m_new) + tot;
          m2 = m_new;
        }
      } else if (i < pass1) {
        float2 y[kPairs];
        mass_scores<LOG2S, kRound, kPairs>(r, y, key0, a.n_rows, sBiasL, a.scale);
        // Pass 1: running max and sum of this part of the row.
        float m8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) m8[q] = fmaxf(y[q].x, y[q].y);
#pragma unroll
        for (int p = 8; p < kPairs; p += 8) {
#pragma unroll
          for (int q = 0; q < 8; ++q) m8[q] = fmax3(m8[q], y[p + q].x, y[p + q].y);
        }
        const float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]),
                               fmaxf(m8[6], m8[7]));
        const float m_new = fmaxf(m2, mx);
        // A row part whose keys so far are all past the sequence (few sampled
        // rows) keeps (-inf, 0): -inf - -inf would be NaN.
        if (m_new != -INFINITY) {
          const float2 nm = make_float2(-m_new, -m_new);
          float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                           make_float2(0.f, 0.f)};
#pragma unroll
          for (int p = 0; p < kPairs; ++p) {
            const float2 t = __fadd2_rn(y[p], nm);
            const float2 e = (p & 7) >= 8 - kMassEmulated ? exp2_pair<1>(t) : exp2_pair<0>(t);
            acc[p & 3] = __fadd2_rn(acc[p & 3], e);
          }
          const float2 a03 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
          l = l * ex2_approx(m2 - m_new) + (a03.x + a03.y);
          m2 = m_new;
        }
      }
      if ((one || i < pass1) && i == n_tiles - 1) {
        {
          // End of the pass over the keys.  Combine the row's parts: the warps of these rows meet at named
          // barrier 1 + wq; every part adds the partial sums in part order.
          sX[part * 128 + row] = make_float2(m2, l);
          if constexpr (kOnChip) {
            tmem_wait_st();
            tc_fence_before();
          }
          asm volatile("bar.sync %0, %1;" ::"r"(1 + wq), "r"(32 * kParts) : "memory");
          if constexpr (kOnChip) tc_fence_after();
          combined = true;
          float m_all, l_all;
          if constexpr (kParts == 2) {
            const float2 o = sX[(part ^ 1) * 128 + row];
            m_all = fmaxf(m2, o.x);
            l_all = l * ex2_approx(m2 - m_all) + o.y * ex2_approx(o.x - m_all);
          } else {
            float2 o[kParts];
#pragma unroll
            for (int q = 0; q < kParts; ++q) o[q] = sX[q * 128 + row];
            m_all = o[0].x;
#pragma unroll
            for (int q = 1; q < kParts; ++q) m_all = fmaxf(m_all, o[q].x);
            l_all = o[0].y * ex2_approx(o[0].x - m_all);
#pragma unroll
            for (int q = 1; q < kParts; ++q) l_all += o[q].y * ex2_approx(o[q].x - m_all);
          }
          // 2^(y - m_fold) = 2^(y - m_all) / l_all
          m_fold = m_all + __log2f(l_all);
          if (emit && part == 0 && qrow < a.n_rows)
            a.row_lse[(static_cast<int64_t>(b) * a.heads + h) * a.n_rows + qrow] = m_fold;
        }
        if constexpr (kOnChip) {
          // The mass of this CTA's query blocks: the warps of a lane quarter
          // take groups of S key blocks in turn (group g by part g mod
          // kParts), read the rows' block values, normalise them and sum
          // each query block's S rows (lanes).
          const bool vrow = qrow < a.n_rows;
          const int64_t qblock = qrow >> LOG2S;
          const int n_groups = (a.q_blocks + S - 1) / S;
#pragma unroll 1
          for (int g = part; g < n_groups; g += kParts) {
            const int kbg = g * S;
            float x[S];
            if (kbg < kTmemVals) {
              tmem_ld_cols<S>(tmem + lane_addr + kTmemVals + kbg, x);
            } else {
#pragma unroll
              for (int j = 0; j < S; ++j)
                x[j] = kbg + j < a.q_blocks ? sVals[(kbg + j - kTmemVals) * 128 + row] : 0.f;
            }
#pragma unroll
            for (int j = 0; j < S; ++j)
              x[j] = (vrow && kbg + j < a.q_blocks) ? ex2_approx(x[j] - m_fold) : 0.f;
            lane_group_sums<S>(x);
            const int kb = kbg + (lane & (S - 1));
            if (kb < a.q_blocks && qblock < a.q_blocks)
              a.mass[(out_rows + qblock) * a.q_blocks + kb] = x[0] * a.mass_scale;
          }
        }
      }
      if (!emit && i >= pass1) {
        // Pass 2: normalised probabilities summed per key block, then over the
        // S sampled rows of each query block.
        float2 y[kPairs];
        mass_scores<LOG2S, kRound, kPairs>(r, y, key0, a.n_rows, sBiasL, a.scale);
        const float2 nf = make_float2(-m_fold, -m_fold);
        float g[kPartBlocks];
#pragma unroll
        for (int gi = 0; gi < kPartBlocks; ++gi) g[gi] = 0.f;
#pragma unroll
        for (int p = 0; p < kPairs; ++p) {
          const float2 t = __fadd2_rn(y[p], nf);
          const float2 e = (p & 7) >= 8 - kMassEmulated ? exp2_pair<1>(t) : exp2_pair<0>(t);
          if constexpr (LOG2S == 0) {
            g[2 * p] += e.x;
            g[2 * p + 1] += e.y;
          } else {
            g[(2 * p) >> LOG2S] += e.x + e.y;
          }
        }
        if (qrow >= a.n_rows) {
#pragma unroll
          for (int gi = 0; gi < kPartBlocks; ++gi) g[gi] = 0.f;
        }
        if constexpr (!kWide) {
          if constexpr (S > 1) {
#pragma unroll
            for (int gi = 0; gi < kPartBlocks; ++gi) {
#pragma unroll
              for (int off = 1; off < S; off <<= 1)
                g[gi] += __shfl_xor_sync(0xffffffffu, g[gi], off);
            }
          }
          const int64_t qblock = qrow >> LOG2S;
          const int64_t kb0 = key0 >> LOG2S;
          if ((lane & (S - 1)) == 0 && qblock < a.q_blocks) {
            float* dst = a.mass + (out_rows + qblock) * a.q_blocks;
#pragma unroll
            for (int gi = 0; gi < kPartBlocks; ++gi)
              if (kb0 + gi < a.q_blocks) dst[kb0 + gi] = g[gi] * a.mass_scale;
          }
        } else {
          // This warp's 32 rows, then the eight warps' partials of the tile.
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) g[0] += __shfl_xor_sync(0xffffffffu, g[0], off);
          const int t2 = i - pass1;                    // key tile of pass 2
          const int grp_i = t2 / kRedTiles, slot = t2 % kRedTiles, buf = grp_i & 1;
          if (slot == 0 && grp_i >= 2 &&
              !mbar_wait(&bar->red_free[buf], ((grp_i >> 1) - 1) & 1, abort_flag, a.err_word)) {
            ok = false;
            break;
          }
          if (lane == 0) sRed[(buf * kRedTiles + slot) * 8 + warp] = g[0];
          const bool last = slot == kRedTiles - 1 || t2 == n_tiles - 1;
          if (last) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->red_full[buf]);
          }
          if (last && warp == 0) {
            if (!mbar_wait(&bar->red_full[buf], (grp_i >> 1) & 1, abort_flag, a.err_word)) {
              ok = false;
              break;
            }
            if (lane <= slot) {
              const float* pr = sRed + (buf * kRedTiles + lane) * 8;
              const int64_t kt = static_cast<int64_t>(grp_i) * kRedTiles + lane;
              if constexpr (S == 128) {
                // warps: half * 4 + row quarter; one query and one key block
                float v = pr[0];
#pragma unroll
                for (int w = 1; w < 8; ++w) v += pr[w];
                if (qt < a.q_blocks && kt < a.q_blocks)
                  a.mass[(out_rows + qt) * a.q_blocks + kt] = v * a.mass_scale;
              } else {
                // S = 64: query block 2 qt + (quarter >> 1), key block 2 kt + half
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const int qbl = c >> 1, kbl = c & 1;
                  const float v = pr[kbl * 4 + 2 * qbl] + pr[kbl * 4 + 2 * qbl + 1];
                  const int64_t qb = 2 * static_cast<int64_t>(qt) + qbl, kb = 2 * kt + kbl;
                  if (qb < a.q_blocks && kb < a.q_blocks)
                    a.mass[(out_rows + qb) * a.q_blocks + kb] = v * a.mass_scale;
                }
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->red_free[buf]);
          }
        }
      }
    }
    // A warp that left pass 1 early (a timed-out wait) still arrives at the
    // row-part barrier, so that the other warps of these rows are not held there.
    if (!combined) asm volatile("bar.arrive %0, %1;" ::"r"(1 + wq), "r"(32 * kParts) : "memory");
    (void)ok;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == Shape::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kOnChip ? 512 : 256);
  }
}

// One-pass mode, second step: one CTA per 32 x 32 (query block, key block)
// tile of one (b, h); warp w sums key blocks kb0 + 4w .. 4w + 3 for the 32
// query blocks (one per lane, its S rows contiguous in block_lse), rows in
// order; the tile is written row-major through shared memory.
template <int LOG2S>
__global__ void __launch_bounds__(256) sampled_mass_reduce_kernel(const MassArgs a) {
  constexpr int S = 1 << LOG2S;
  __shared__ float tile[32][33];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qb0 = blockIdx.x * 32;
  const int kb0 = blockIdx.y * 32;
  const int64_t bh = blockIdx.z;
  const int Qb = a.q_blocks;
  const int qb = qb0 + lane;
  float lse[S];
  if (qb < Qb) {
    const float* lr = a.row_lse + bh * a.n_rows + static_cast<int64_t>(qb) * S;
#pragma unroll
    for (int s = 0; s < S; ++s) lse[s] = lr[s];
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int kl = warp * 4 + c;
    const int kb = kb0 + kl;
    float sum = 0.f;
    if (qb < Qb && kb < Qb) {
      const float* v = a.block_lse + (bh * Qb + kb) * a.n_rows + static_cast<int64_t>(qb) * S;
      float x[S];
      if constexpr (S >= 4) {
#pragma unroll
        for (int s = 0; s < S; s += 4) {
          const float4 t = __ldcs(reinterpret_cast<const float4*>(v + s));
          x[s] = t.x;
          x[s + 1] = t.y;
          x[s + 2] = t.z;
          x[s + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int s = 0; s < S; ++s) x[s] = __ldcs(v + s);
      }
#pragma unroll
      for (int s = 0; s < S; ++s) sum += ex2_approx(x[s] - lse[s]);
    }
    tile[kl][lane] = sum * a.mass_scale;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 32 * 32; idx += 256) {
    const int ql = idx >> 5, kl = idx & 31;
    if (qb0 + ql < Qb && kb0 + kl < Qb)
      a.mass[(bh * Qb + qb0 + ql) * Qb + kb0 + kl] = tile[kl][ql];
  }
}

template <int LOG2S, bool kRound, bool kOnChip>
cudaError_t launch_log2s_v2(const CUtensorMap& tq, const CUtensorMap& tk, const MassArgs& a,
                            cudaStream_t stream) {
  // Per-device flag; concurrent callers may both set the attribute, which is
  // harmless, but the flag itself must not be a data race.  The on-chip mode
  // sets the largest size once; each launch asks for what its blocks need.
  using L = MassLayout<kOnChip>;
  static std::atomic<bool> configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int max_bytes = kOnChip ? kMaxDynSmem : L::kBytes;
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(sampled_mass_kernel2<LOG2S, kRound, kOnChip>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, max_bytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev].store(true, std::memory_order_release);
  }
  int bytes = L::kBytes;
  if (kOnChip && a.q_blocks > kTmemVals) bytes += (a.q_blocks - kTmemVals) * 128 * 4;
  if (bytes > max_bytes) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>((a.n_rows + kTile - 1) / kTile),
                  static_cast<unsigned>(a.heads), static_cast<unsigned>(a.batch));
  sampled_mass_kernel2<LOG2S, kRound, kOnChip>
      <<<grid, MassShape<LOG2S>::kThreads, bytes, stream>>>(tq, tk, a);
  return cudaGetLastError();
}

template <int LOG2S, bool kOnChip = false>
cudaError_t launch_s(const CUtensorMap& tq, const CUtensorMap& tk, const MassArgs& a,
                           cudaStream_t stream) {
  return a.round_bf16 ? launch_log2s_v2<LOG2S, true, kOnChip>(tq, tk, a, stream)
                      : launch_log2s_v2<LOG2S, false, kOnChip>(tq, tk, a, stream);
}

template <int LOG2S>
cudaError_t launch_reduce_s(const MassArgs& a, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>((a.q_blocks + 31) / 32),
                  static_cast<unsigned>((a.q_blocks + 31) / 32),
                  static_cast<unsigned>(a.batch * a.heads));
  sampled_mass_reduce_kernel<LOG2S><<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_sampled_mass_reduce(const MassArgs& a, cudaStream_t stream) {
  if (a.batch == 0 || a.heads == 0 || a.n_rows == 0) return cudaSuccess;
  if (a.block_lse == nullptr || a.row_lse == nullptr || a.batch * a.heads > 65535)
    return cudaErrorInvalidValue;
  switch (a.samples) {
    case 1: return launch_reduce_s<0>(a, stream);
    case 2: return launch_reduce_s<1>(a, stream);
    case 4: return launch_reduce_s<2>(a, stream);
    case 8: return launch_reduce_s<3>(a, stream);
    case 16: return launch_reduce_s<4>(a, stream);
    case 32: return launch_reduce_s<5>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

bool sampled_mass_on_chip(int32_t q_blocks, int32_t samples) {
  // S = 16, 32: four column parts of 32 keys; fewer samples per block keep
  // more per-block state per thread than the on-chip pass has registers for.
  return (samples == 16 || samples == 32) && q_blocks >= 1 && q_blocks <= kOnChipMaxBlocks;
}

cudaError_t launch_sampled_mass_on_chip(const CUtensorMap& tq, const CUtensorMap& tk,
                                        const MassArgs& a, cudaStream_t stream) {
  if (a.batch == 0 || a.heads == 0 || a.n_rows == 0) return cudaSuccess;
  if (!sampled_mass_on_chip(a.q_blocks, a.samples) || a.lse != nullptr ||
      a.block_lse != nullptr)
    return cudaErrorInvalidValue;
  return a.samples == 16 ? launch_s<4, true>(tq, tk, a, stream)
                         : launch_s<5, true>(tq, tk, a, stream);
}

cudaError_t launch_sampled_mass(const CUtensorMap& tq, const CUtensorMap& tk, const MassArgs& a,
                                cudaStream_t stream) {
  if (a.batch == 0 || a.heads == 0 || a.n_rows == 0) return cudaSuccess;
  if (a.q_blocks > kMaxBlocks) return cudaErrorInvalidValue;
  switch (a.samples) {
    case 1: return launch_s<0>(tq, tk, a, stream);
    case 2: return launch_s<1>(tq, tk, a, stream);
    case 4: return launch_s<2>(tq, tk, a, stream);
    case 8: return launch_s<3>(tq, tk, a, stream);
    case 16: return launch_s<4>(tq, tk, a, stream);
    case 32: return launch_s<5>(tq, tk, a, stream);
    case 64: return launch_s<6>(tq, tk, a, stream);
    case 128: return launch_s<7>(tq, tk, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace bsa
