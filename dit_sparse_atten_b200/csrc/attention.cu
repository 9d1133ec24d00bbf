// (a) Block-sparse flash attention over a per-[batch, head, query-block] CSR
// route, for sm_100a.
//
// Reference semantics: FlexAttention with full blocks only, as driven by
// attention_backends/flex.py:308-355 (route -> BlockMask) and :379-399
// (padding, kernel call, trim); equivalently the gather/softmax/PV of
// attention_backends/sparse.py:670-751.  A query in block qb of head h attends
// to every valid key (< T) in the key blocks listed in its CSR row.
//
// One CTA handles one (qb, h, b) work item: 128 query rows (the MMA M), key
// blocks of BK = 128 (or 64) tokens.
//   warp 8      TMA producer: K/V tiles by routed block id into a ring of
//               shared-memory slots (consumption order K0, K1, V0, K2, V1, ...)
//   warp 9      TMEM allocator; one thread TMA-loads Q into shared memory and
//               issues S_j = Q K_j^T (A and B from shared memory)
//   warp 10     one thread issues O += P_j V_j (A = P from tensor memory)
//               Two issuing threads keep the tensor pipe fed while either
//               waits on a barrier (the pipe queues only about one
//               128x128x16 MMA ahead).
//   warps 0-7   softmax, two groups of four warps taking alternate key blocks
//               (group g = w/4 handles blocks j with j % 2 == g), so a group
//               has two block periods for its softmax.  Warp w owns TMEM lanes
//               32*(w%4).. (query rows), one full row per thread, read from
//               TMEM twice (row max, then exponentials in 32-column chunks).
//               Scores are handled in the log2 domain with a running
//               stabiliser that only moves when the max grows by more than 2^8
//               (then O is rescaled in TMEM); it passes from group to group
//               through shared memory (m_full barriers), each group keeps its
//               own row sum and the epilogue combines the two.  P_j (bf16) is
//               written into the first BK/2 columns of S_j's own TMEM buffer;
//               the epilogue normalises O and stores it (group g writes
//               features 64 g .. 64 g + 63).
// TMEM columns: three S (and P) buffers at [0,128), [128,256), [256,384), O at
// [384,512).  Shared memory: Q (32 KB) and the K/V ring.
// Ordering: S_{j+3} overwrites P_j, so the S issuer waits for PV_j (o_done);
// with three buffers a group's next S never waits for its own softmax.  The
// softmax waits for the previous PV only when it rescales O.  Barriers of a
// buffer complete once per three blocks, and no waiter can fall two phases
// behind (each next phase needs the waiter's own progress).
// Every mbarrier wait is bounded (bsa::mbar_wait); on a timeout the CTA sets
// kErrWaitTimeout in the caller's error word, drains its in-flight copies and
// MMAs, frees TMEM and exits.
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "attention_softmax.cuh"
#include "bsa_kernels.h"

namespace bsa {
namespace {

using namespace attn;

// Softmax groups of four warps; group g takes the key blocks j with
// j % kGroups == g.  Three groups run with a register split (setmaxnreg):
// 512 threads launched with kLaunchRegs each, the control warpgroup (TMA
// producer, the two MMA issuers, one idle warp) gives registers back and the
// three softmax warpgroups take them.
#ifndef BSA_SOFTMAX_GROUPS
#define BSA_SOFTMAX_GROUPS 2
#endif
constexpr int kGroups = BSA_SOFTMAX_GROUPS;
static_assert(kGroups == 2 || kGroups == 3, "two or three softmax groups");
constexpr int kSoftmaxWarps = 4 * kGroups;
constexpr int kProducerWarp = kSoftmaxWarps;
constexpr int kMmaWarp = kSoftmaxWarps + 1;   // S issuer, TMEM owner
constexpr int kPvWarp = kSoftmaxWarps + 2;    // PV issuer
constexpr int kAttnThreads = kGroups == 2 ? 352 : 512;
constexpr bool kRegSplit = kGroups == 3;
constexpr uint32_t kLaunchRegs = 128;         // 512 threads x 128 = 65,536
constexpr uint32_t kSoftRegs = 144;
constexpr uint32_t kCtrlRegs = 64;
static_assert(!kRegSplit || 3 * 128 * kSoftRegs + 128 * kCtrlRegs <= kAttnThreads * kLaunchRegs,
              "register split must stay within the launch total");
constexpr int kHeadDim = 128;
constexpr int kSBuffers = 3;            // S/P buffers in TMEM
constexpr uint32_t kTmemO = 384;
// Of every 8 column pairs of a full key block, this many take their
// exponentials on the FMA pipe (exp2_poly2) instead of MUFU.  Measured on
// B200: the softmax is bound by instruction issue, not by MUFU, so the default
// keeps every exponential on MUFU (one instruction per value).
#ifndef BSA_EMULATED_PAIRS
#define BSA_EMULATED_PAIRS 0
#endif
constexpr int kEmulatedPairsPer8 = BSA_EMULATED_PAIRS;
// S-row chunks kept in registers between the max and exponential passes.
#ifndef BSA_KEPT_CHUNKS
#define BSA_KEPT_CHUNKS 0
#endif
template <int BK>
constexpr int kKeep = BSA_KEPT_CHUNKS > 0 && BK == 128 ? BSA_KEPT_CHUNKS : kKeptChunks<BK>;

template <int BK>
struct AttnLayout {
  static constexpr int kSlotPanel = BK * 128;            // one 64-column panel of K or V
  static constexpr int kSlotBytes = 2 * kSlotPanel;
  static constexpr int kSlots = BK == 128 ? (kGroups == 2 ? 6 : 5) : 12;
  static constexpr int kQOff = 0;                                // Q tile, 128 rows x 256 B
  static constexpr int kRingOff = kQOff + 128 * 256;
  static constexpr int kXOff = kRingOff + kSlots * kSlotBytes;   // stabiliser hand-over
  static constexpr int kXBytes = 2 * kGroups * 128 * 4;          // [2][groups][row] floats
  static constexpr int kBarOff = kXOff + kXBytes;
  static constexpr int kBarBytes = 320;
  static constexpr int kUsed = kBarOff + kBarBytes;
};

struct AttnBarriers {
  uint64_t q_full;
  uint64_t s_full[kSBuffers];
  uint64_t p_full[kSBuffers];
  uint64_t m_full[2];
  uint64_t o_done[kSBuffers];
  uint64_t drain[2];
  uint64_t slot_full[12];
  uint64_t slot_empty[12];
  uint32_t tmem_base;
  int abort;
};

// kDenseMass: every key block in order (no CSR), and each query row also
// writes, per key block kb, v = log2 of its exponential sum over the block's
// keys (the online softmax's block row sum, shifted back by the stabiliser it
// used) to a.block_lse[b, h, kb, row]; block_mass_kernel turns these and the
// row LSE into the exact block mass.
template <int BK, bool kDenseMass>
__global__ void __launch_bounds__(kAttnThreads, 1)
    bsa_attention_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const AttnArgs a) {
  using L = AttnLayout<BK>;
  static_assert(sizeof(AttnBarriers) <= L::kBarBytes, "barrier area");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sRing = smem + L::kRingOff;
  float* sX = reinterpret_cast<float*>(smem + L::kXOff);
  AttnBarriers* bar = reinterpret_cast<AttnBarriers*>(smem + L::kBarOff);
  volatile int* abort_flag = &bar->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qb = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int64_t rb = a.route_batch_stride ? b : 0;
  const int64_t route_row = (rb * a.heads + h) * a.q_blocks + qb;
  const int32_t* kv_list = kDenseMass ? nullptr : a.indices + route_row * a.route_cols;
  int n = kDenseMass ? a.k_blocks : a.counts[route_row];
  if (n < 0 || n > a.route_cols || n > a.k_blocks) {
    if (threadIdx.x == 0) atomicOr(a.err_word, kErrBadRoute);
    n = n < 0 ? 0 : min(n, min(a.route_cols, a.k_blocks));
  }

  if constexpr (BK < 128) {
    // The S MMA always reads 128 Q rows; rows past a 64-token block are zero
    // (TMA writes rows [0, BK) of each 64-feature panel).
    for (int i = threadIdx.x; i < 2 * (128 - BK) * 8; i += kAttnThreads) {
      const int panel = i / ((128 - BK) * 8);
      const int chunk = i % ((128 - BK) * 8);
      reinterpret_cast<uint4*>(sQ + panel * 16384 + BK * 128)[chunk] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    uint32_t dyn_bytes;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_bytes));
    const bool fits = (smem - smem_raw) + L::kUsed <= static_cast<int>(dyn_bytes);
    mbar_init(&bar->q_full, 1);
    for (int i = 0; i < kSBuffers; ++i) {
      mbar_init(&bar->s_full[i], 1);
      mbar_init(&bar->p_full[i], 128);   // one group (128 threads) per block
      mbar_init(&bar->o_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->m_full[i], 128);
      mbar_init(&bar->drain[i], 1);
    }
    for (int s = 0; s < L::kSlots; ++s) {
      mbar_init(&bar->slot_full[s], 1);
      mbar_init(&bar->slot_empty[s], 1);
    }
    bar->abort = (prior_timeout(a.err_word) || !fits) ? 1 : 0;
    if (!fits) atomicOr(a.err_word, kErrSmemLayout);
    fence_mbar_init();
  }
  __syncthreads();
  if (bar->abort) return;  // uniform: set before the barrier, read after it
  if (warp == kMmaWarp) tmem_alloc(&bar->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;

  auto block_id = [&](int j) -> int {
    if constexpr (kDenseMass) return j;
    int kb = __ldg(kv_list + j);
    if (kb < 0 || kb >= a.k_blocks) {
      atomicOr(a.err_word, kErrBadRoute);
      kb = kb < 0 ? 0 : a.k_blocks - 1;
    }
    return kb;
  };

  if (warp >= kSoftmaxWarps) {
   if constexpr (kRegSplit) setmaxnreg_dec<kCtrlRegs>();
   if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      // Per slot: a load was issued / its parity (bit masks: a run-time
      // indexed array would live in local memory, whose traffic slows TMA).
      uint32_t armed = 0, armed_phase = 0;
      int seq = 0;
      bool ok = true;
      auto load = [&](const CUtensorMap* tm, int kb) {
        const int s = seq % L::kSlots;
        const uint32_t ph = (seq / L::kSlots) & 1;
        if (!mbar_wait(&bar->slot_empty[s], ph ^ 1, abort_flag, a.err_word)) return false;
        uint8_t* dst = sRing + s * L::kSlotBytes;
        mbar_arrive_expect_tx(&bar->slot_full[s], L::kSlotBytes);
        tma_load_4d(dst, tm, &bar->slot_full[s], 0, h, kb * BK, b);
        tma_load_4d(dst + L::kSlotPanel, tm, &bar->slot_full[s], 64, h, kb * BK, b);
        armed |= 1u << s;
        armed_phase = (armed_phase & ~(1u << s)) | (ph << s);
        ++seq;
        return true;
      };
      ok = load(&tm_k, block_id(0));
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n) ok = load(&tm_k, block_id(j + 1));
        if (ok) ok = load(&tm_v, block_id(j));
      }
      // Never leave a copy in flight into shared memory.
      int never = 0;
#pragma unroll
      for (int s = 0; s < L::kSlots; ++s)
        if (armed & (1u << s)) mbar_wait(&bar->slot_full[s], (armed_phase >> s) & 1u, &never, a.err_word);
    }
   } else if (warp == kMmaWarp || warp == kPvWarp) {
    // ------------------------------------------------------------ MMA issuers
    // Load sequence of the producer: K0, then K_{j+1}, V_j for every j.
    auto seq_k = [](int j) { return j == 0 ? 0 : 2 * j - 1; };
    auto seq_v = [n](int j) { return j + 1 < n ? 2 * j + 2 : 2 * j + 1; };
    const uint32_t ring_addr = smem_u32(sRing);
    if (warp == kMmaWarp && lane == 0 && n > 0) {
      const uint32_t idesc_s = idesc_bf16_f32(128, BK, false);
      const uint64_t kdesc0 = sdesc_sw128(ring_addr, 16, 1024);
      const uint64_t qdesc0 = sdesc_sw128(smem_u32(sQ), 16, 1024);
      tma_prefetch_desc(&tm_q);
      mbar_arrive_expect_tx(&bar->q_full, BK * 256);
      tma_load_4d(sQ, &tm_q, &bar->q_full, 0, h, qb * BK, b);
      tma_load_4d(sQ + 16384, &tm_q, &bar->q_full, 64, h, qb * BK, b);
      bool ok = mbar_wait(&bar->q_full, 0, abort_flag, a.err_word);
      for (int j = 0; ok && j < n; ++j) {
        const int sq = seq_k(j);
        const int s = sq % L::kSlots;
        ok = mbar_wait(&bar->slot_full[s], (sq / L::kSlots) & 1, abort_flag, a.err_word);
        // S_j overwrites P_{j-3} (same TMEM buffer): PV_{j-3} must be done.
        const int sb = j % kSBuffers;
        if (ok && j >= kSBuffers)
          ok = mbar_wait(&bar->o_done[sb], ((j - kSBuffers) / kSBuffers) & 1, abort_flag,
                         a.err_word);
        if (!ok) break;
        tc_fence_after();
        const uint64_t kd = kdesc0 + static_cast<uint64_t>((s * L::kSlotBytes) >> 4);
        const uint32_t d = tmem + sb * 128;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {
          const uint64_t db = kd + static_cast<uint64_t>(((kk >> 2) * L::kSlotPanel + (kk & 3) * 32) >> 4);
          const uint64_t da = qdesc0 + static_cast<uint64_t>(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
          umma_bf16_ss(d, da, db, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar->s_full[sb]);
        umma_commit(&bar->slot_empty[s]);
      }
      int never = 0;
      umma_commit(&bar->drain[0]);
      mbar_wait(&bar->drain[0], 0, &never, a.err_word);
    } else if (warp == kPvWarp && lane == 0 && n > 0) {
      const uint32_t idesc_o = idesc_bf16_f32(128, kHeadDim, true);
      const uint64_t vdesc0 = sdesc_sw128(ring_addr, L::kSlotPanel, 1024);
      bool ok = true;
      for (int j = 0; ok && j < n; ++j) {
        const int sq = seq_v(j);
        const int s = sq % L::kSlots;
        ok = mbar_wait(&bar->slot_full[s], (sq / L::kSlots) & 1, abort_flag, a.err_word);
        const int sb = j % kSBuffers;
        if (ok) ok = mbar_wait(&bar->p_full[sb], (j / kSBuffers) & 1, abort_flag, a.err_word);
        if (!ok) break;
        tc_fence_after();
        const uint64_t vd = vdesc0 + static_cast<uint64_t>((s * L::kSlotBytes) >> 4);
        const uint32_t pa = tmem + sb * 128;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          umma_bf16_ts(tmem + kTmemO, pa + kk * 8, vd + static_cast<uint64_t>((kk * 16 * 128) >> 4),
                       idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bar->o_done[sb]);
        umma_commit(&bar->slot_empty[s]);
      }
      int never = 0;
      umma_commit(&bar->drain[1]);
      mbar_wait(&bar->drain[1], 0, &never, a.err_word);
    }
   }
  } else {
    if constexpr (kRegSplit) setmaxnreg_inc<kSoftRegs>();
    // ------------------------------------------------------------ softmax
    // kGroups groups of four warps take turns over the key blocks: group
    // g = warp / 4 handles blocks j with j % kGroups == g, one full row per
    // thread (warp w owns TMEM lanes 32*(w%4)..), so each group has kGroups
    // block periods for its softmax.  The stabiliser moves from group to
    // group through m_buf and the m_full barriers; each group keeps its own
    // row sum.
    const int grp = warp >> 2;
    const int wq = warp & 3;                   // TMEM lane quarter
    const int row = wq * 32 + lane;            // query row == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t pair_barrier = 1 + wq;      // the warps (one per group) of these lanes
    const bool warp_active = (BK == 128) || (wq < 2);
    const int64_t token = static_cast<int64_t>(qb) * BK + row;
    const bool row_valid = warp_active && row < BK && token < a.tokens;

    float* m_buf = sX;                  // [parity][row]: stabiliser used at the block
    const float c = a.scale * kLog2e;
    const float2 c2 = make_float2(c, c);
    float m_mine = -INFINITY;           // stabiliser of this group's latest block
    float l = 0.f;                      // this group's row sum, relative to m_mine
    bool ok = true;
    int kb_next = (warp_active && grp < n) ? block_id(grp) : 0;
    for (int j = grp; ok && j < n; j += kGroups) {
      const int sb = j % kSBuffers;
      ok = mbar_wait(&bar->s_full[sb], (j / kSBuffers) & 1, abort_flag, a.err_word);
      if (!ok) break;
      tc_fence_after();
      const uint32_t sbuf = tmem + lane_addr + sb * 128;
      const int kb = kb_next;
      if (warp_active && j + kGroups < n) kb_next = block_id(j + kGroups);  // hide its latency
      const int64_t valid = a.tokens - static_cast<int64_t>(kb) * BK;
      const bool partial = valid < BK;
      uint32_t keep[kKeep<BK>][32];
      const float mrow =
          warp_active ? row_max<BK, kKeep<BK>, kRegSplit>(sbuf, partial, valid, keep) * c
                      : -INFINITY;
      // The previous block's stabiliser (decided by the other group).
      float m_prev = -INFINITY;
      if (j > 0) {
        ok = mbar_wait(&bar->m_full[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, a.err_word);
        if (!ok) break;
        m_prev = m_buf[((j - 1) & 1) * 128 + row];
      }
      const bool need = mrow > m_prev + kRescaleThreshold;
      const float m_used = need ? mrow : m_prev;
      m_buf[(j & 1) * 128 + row] = m_used;
      mbar_arrive(&bar->m_full[j & 1]);
      if (warp_active) {
        l *= ex2_approx(m_mine - m_used);  // m_mine = -inf at this group's first block: l = 0
        m_mine = m_used;
        const float2 neg_m = make_float2(-m_used, -m_used);
        // Partial blocks (masked columns) take every exponential on MUFU.
        const float2 rs =
            partial ? row_exp<BK, 0, kKeep<BK>>(sbuf, true, valid, c2, neg_m, keep)
                    : row_exp<BK, kEmulatedPairsPer8, kKeep<BK>>(sbuf, false, valid, c2, neg_m, keep);
        l += rs.x + rs.y;
        if constexpr (kDenseMass) {
          if (row_valid) {
            float* dst = a.block_lse + static_cast<int64_t>(kb) * a.tokens + token;
            dst[(static_cast<int64_t>(b) * a.heads + h) * a.k_blocks * a.tokens] =
                m_used + __log2f(rs.x + rs.y);
          }
        }
      }
      // O holds the blocks before j relative to m_prev: a moved stabiliser
      // rescales it once PV_{j-1} is done (rare after the first blocks).
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        ok = mbar_wait(&bar->o_done[(j - 1) % kSBuffers], ((j - 1) / kSBuffers) & 1, abort_flag,
                       a.err_word);
        if (!ok) break;
        tc_fence_after();
        if (warp_active) {
          const float p_scale = need ? ex2_approx(m_prev - m_used) : 1.f;
#pragma unroll 1
          for (int cc = 0; cc < kHeadDim / 32; ++cc) {
            uint32_t o[32];
            const uint32_t addr = tmem + lane_addr + kTmemO + cc * 32;
            tmem_ld_32x32b_x32(addr, o);
            tmem_wait_ld();
            reg_fence<32>(o);
#pragma unroll
            for (int x = 0; x < 32; ++x) o[x] = __float_as_uint(__uint_as_float(o[x]) * p_scale);
            tmem_st_32x32b_x32(addr, o);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bar->p_full[sb]);
    }
    // ---------------------------------------------------------- epilogue
    // All groups' (stabiliser, sum) meet through shared memory; the final
    // stabiliser is the largest (it never decreases along the blocks).
    // Groups 0 and 1 then write output features [64 g, 64 g + 64).
    float* xs = sX;  // [group][row] stabilisers, then [group][row] sums
    named_bar_sync(pair_barrier, 32 * kGroups);    // every group is past its last m_buf read
    xs[grp * 128 + row] = m_mine;
    xs[kGroups * 128 + grp * 128 + row] = l;
    named_bar_sync(pair_barrier, 32 * kGroups);
    float m_fin = -INFINITY;
#pragma unroll
    for (int g = 0; g < kGroups; ++g) m_fin = fmaxf(m_fin, xs[g * 128 + row]);
    float l_row = 0.f;
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      const float m_g = xs[g * 128 + row];
      if (m_g != -INFINITY) l_row += xs[kGroups * 128 + g * 128 + row] * ex2_approx(m_g - m_fin);
    }
    // O is final once every PV has completed: drain[1] (one phase) is the PV
    // issuer's commit after its last MMA.  (A wait on o_done of the last
    // block could return early for a group that last saw that barrier two
    // phases back.)
    if (ok && n > 0) {
      ok = mbar_wait(&bar->drain[1], 0, abort_flag, a.err_word);
      tc_fence_after();
    }
    // Destination token of this row (the unpack folded into the store).
    int64_t out_token = token;
    bool row_store = row_valid;
    if (a.out_rows != nullptr && row_valid) {
      out_token = __ldg(a.out_rows + token);
      if (out_token < 0 || out_token >= a.tokens) {
        atomicOr(a.err_word, kErrBadRoute);
        row_store = false;
      }
    }
    // Multi-GPU: the row's token lives on rank out_token / peer_tokens, whose
    // output shard is mapped into this process (the stores cross NVLink; they
    // are complete when the kernel is, and the host joins the ranks with a
    // collective after it before any shard is read).
    __nv_bfloat16* out_base = a.out + b * a.out_stride_b;
    if (a.n_peer > 0 && row_store) {
      const int64_t d = out_token / a.peer_tokens;
      if (d >= a.n_peer) {
        atomicOr(a.err_word, kErrBadRoute);
        row_store = false;
      } else {
        out_base = a.out_peer[d];
        out_token -= d * a.peer_tokens;
      }
    }
    if (warp_active && grp < 2) {
      __nv_bfloat16* out = out_base + out_token * a.out_stride_t + h * a.out_stride_h + grp * 64;
      const float inv_l = (n > 0 && l_row > 0.f) ? 1.f / l_row : 0.f;
#pragma unroll 1
      for (int cc = 0; cc < kHeadDim / 64; ++cc) {
        uint32_t o[32];
        if (ok && n > 0) {
          tmem_ld_32x32b_x32(tmem + lane_addr + kTmemO + grp * 64 + cc * 32, o);
          tmem_wait_ld();
          reg_fence<32>(o);
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x) o[x] = 0u;
        }
        if (row_store) {
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint4 pk;
            pk.x = pack_bf16x2(__uint_as_float(o[v4 * 8 + 0]) * inv_l,
                               __uint_as_float(o[v4 * 8 + 1]) * inv_l);
            pk.y = pack_bf16x2(__uint_as_float(o[v4 * 8 + 2]) * inv_l,
                               __uint_as_float(o[v4 * 8 + 3]) * inv_l);
            pk.z = pack_bf16x2(__uint_as_float(o[v4 * 8 + 4]) * inv_l,
                               __uint_as_float(o[v4 * 8 + 5]) * inv_l);
            pk.w = pack_bf16x2(__uint_as_float(o[v4 * 8 + 6]) * inv_l,
                               __uint_as_float(o[v4 * 8 + 7]) * inv_l);
            *reinterpret_cast<uint4*>(out + cc * 32 + v4 * 8) = pk;
          }
        }
      }
      if (row_valid && grp == 0 && a.lse != nullptr) {
        a.lse[(static_cast<int64_t>(b) * a.heads + h) * a.tokens + token] =
            (n > 0 && l_row > 0.f) ? (m_fin + __log2f(l_row)) * kLn2 : -INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int BK, bool kDenseMass>
cudaError_t launch_bk(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                      const AttnArgs& a, cudaStream_t stream) {
  using L = AttnLayout<BK>;
  // The layout needs kUsed bytes from a 1024-byte-aligned base; ask for up to
  // 1 KB of slack within the opt-in limit (the kernel checks and reports).
  static std::atomic<int> smem_bytes[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int bytes = (dev >= 0 && dev < 64) ? smem_bytes[dev].load(std::memory_order_acquire) : 0;
  if (bytes == 0) {
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    bytes = optin < L::kUsed + 1024 ? optin : L::kUsed + 1024;
    if (bytes < L::kUsed) return cudaErrorInvalidConfiguration;
    if constexpr (kRegSplit) {
      // The register split assumes exactly kLaunchRegs per thread at launch.
      cudaFuncAttributes attr{};
      e = cudaFuncGetAttributes(&attr, bsa_attention_kernel<BK, kDenseMass>);
      if (e != cudaSuccess) return e;
      if (attr.numRegs != static_cast<int>(kLaunchRegs)) return cudaErrorInvalidConfiguration;
    }
    e = cudaFuncSetAttribute(bsa_attention_kernel<BK, kDenseMass>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) smem_bytes[dev].store(bytes, std::memory_order_release);
  }
  const dim3 grid(static_cast<unsigned>(a.q_blocks), static_cast<unsigned>(a.heads),
                  static_cast<unsigned>(a.batch));
  bsa_attention_kernel<BK, kDenseMass><<<grid, kAttnThreads, bytes, stream>>>(tq, tk, tv, a);
  return cudaGetLastError();
}

}  // namespace

namespace {

// mass[b, h, qb, kb] = sum over the rows r < T of query block qb of
// 2^(block_lse[b, h, kb, r] - lse[b, h, r] * log2(e)): one warp per
// (query block, key block) cell, rows added in a fixed order.
__global__ void __launch_bounds__(256) block_mass_kernel(const float* __restrict__ block_lse,
                                                         const float* __restrict__ lse,
                                                         int64_t tokens, int heads, int blocks,
                                                         float* __restrict__ mass) {
  const int kb = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t bh = static_cast<int64_t>(b) * heads + h;
  const float* v = block_lse + (bh * blocks + kb) * tokens;
  const float* l = lse + bh * tokens;
  for (int qb = warp; qb < blocks; qb += 8) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t r = static_cast<int64_t>(qb) * 128 + i * 32 + lane;
      if (r < tokens) acc += ex2_approx(__ldg(v + r) - __ldg(l + r) * kLog2e);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) mass[(bh * blocks + qb) * blocks + kb] = acc;
  }
}

}  // namespace

cudaError_t launch_block_mass(const float* block_lse, const float* lse, int64_t batch,
                              int64_t tokens, int64_t heads, int32_t blocks, float* mass,
                              cudaStream_t stream) {
  if (batch == 0 || heads == 0 || blocks == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(heads),
                  static_cast<unsigned>(batch));
  block_mass_kernel<<<grid, 256, 0, stream>>>(block_lse, lse, tokens, static_cast<int>(heads),
                                              blocks, mass);
  return cudaGetLastError();
}

cudaError_t launch_attention(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const AttnArgs& a, cudaStream_t stream) {
  if (a.batch == 0 || a.heads == 0 || a.q_blocks == 0) return cudaSuccess;
  // BSA_ATTENTION_KERNEL=pair selects the two-query-block kernel for
  // 128-token blocks (attention_pair.cu); the default is the one-block kernel.
  static const bool pair = [] {
    const char* v = getenv("BSA_ATTENTION_KERNEL");
    return v != nullptr && strcmp(v, "pair") == 0;
  }();
  if (a.n_peer > 0 && (a.batch != 1 || a.block_lse != nullptr || a.peer_tokens <= 0 ||
                      a.n_peer > kMaxPeers))
    return cudaErrorInvalidValue;
  if (a.block == 128 && pair && a.n_peer == 0) return launch_attention_pair(tq, tk, tv, a, stream);
  if (a.block_lse != nullptr) {
    if (a.block == 128) return launch_bk<128, true>(tq, tk, tv, a, stream);
    return cudaErrorInvalidValue;
  }
  if (a.block == 128) return launch_bk<128, false>(tq, tk, tv, a, stream);
  if (a.block == 64) return launch_bk<64, false>(tq, tk, tv, a, stream);
  return cudaErrorInvalidValue;
}

}  // namespace bsa
